"""The multi-GPU plan (vbsr_multi_plan_*, MultiPlan) against the oracle, through the C ABI.

Shards may share a GPU, so the partition, the B replication tree and the C gather are exercised
on a one-GPU box too: with several shards on device 0 the replica copies are plain
device-to-device copies and every shard's kernel runs independently (no shard waits on another).
The test on two distinct GPUs runs where the box has them.
"""
import numpy as np
import pytest

import varblockspmm_b200 as vb
from helpers import assert_within_bound, spec_case

pytestmark = pytest.mark.gpu


def _check_shards(mp, host, shards):
    """Shards cover the block rows in order, and their C row ranges tile the M rows."""
    bounds = vb.partition_rows(host, shards, mp.rhs)
    c0 = 0
    for r in range(shards):
        sh = mp.shard(r)
        assert (sh.row_begin, sh.row_end) == (bounds[r], bounds[r + 1])
        assert sh.c_row0 == c0
        assert sh.c_rows == host.row_scalar_off[sh.row_end] - host.row_scalar_off[sh.row_begin]
        c0 += sh.c_rows
    assert c0 == host.scalar_rows()


@pytest.mark.parametrize("shards,rhs", [(1, 32), (3, 32), (4, 8), (5, 64), (2, 16)])
def test_multi_plan_host_buffers(cuda, shards, rhs):
    """Shards on device 0; B replicated from host memory; C gathered into host memory."""
    host = spec_case(512, 8, 2, False, 3)
    B = vb.fill_uniform(3, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    mp = vb.MultiPlan(host, [0] * shards, vb.PlanOptions(rhs))
    assert len(mp) == shards
    _check_shards(mp, host, shards)
    mp.replicate_B(B)
    mp.execute()
    ms = mp.synchronize()
    assert ms > 0.0
    got = mp.gather_C()
    assert np.isfinite(got).all()
    assert_within_bound(host, B, rhs, got)


def test_multi_plan_device_buffers_and_repeat(cuda):
    """B replicated from a device tensor, C gathered into a device tensor; a second replicate
    with a different B and a second execute give the new product (replicas are rewritten in
    stream order)."""
    torch = cuda
    rhs = 32
    host = spec_case(384, 6, 3, True, 7)
    K, M = host.scalar_cols(), host.scalar_rows()
    mp = vb.MultiPlan(host, [0, 0, 0], vb.PlanOptions(rhs))
    for seed in (11, 12):
        B = vb.fill_uniform(seed, vb.STREAM_DENSE, 0, K * rhs)
        dB = torch.from_numpy(B).cuda()
        mp.replicate_B(dB)
        mp.execute()
        mp.synchronize()
        dC = torch.full((M * rhs,), float("nan"), device="cuda")
        mp.gather_C(dC)
        got = dC.cpu().numpy()
        assert_within_bound(host, B, rhs, got)


def test_multi_plan_generated_values(cuda):
    """Shard values generated on the device (counter stream of the seed) equal the host
    generator's, so the multi-plan built without host values matches the oracle on the
    host-generated matrix."""
    rhs = 16
    host = spec_case(256, 4, 0, False, 5)
    structure = spec_case(256, 4, 0, False, 5, with_values=False)
    B = vb.fill_uniform(5, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    mp = vb.MultiPlan(structure, [0, 0], vb.PlanOptions(rhs), generated_seed=5)
    mp.replicate_B(B)
    mp.execute()
    mp.synchronize()
    assert_within_bound(host, B, rhs, mp.gather_C())


def test_multi_plan_rejects_bad_arguments(cuda):
    host = spec_case(64, 2, 0, True, 1)
    with pytest.raises(vb.InvalidArgument, match="more shards than block rows"):
        vb.MultiPlan(host, [0] * 65, vb.PlanOptions(8))
    with pytest.raises(vb.InvalidArgument, match="device ordinal"):
        vb.MultiPlan(host, [0, 4096], vb.PlanOptions(8))
    with pytest.raises(vb.InvalidArgument, match="rhs_width must be 8,16,32,64"):
        vb.MultiPlan(host, [0], vb.PlanOptions(12))
    mp = vb.MultiPlan(host, [0, 0], vb.PlanOptions(8))
    with pytest.raises(vb.InvalidArgument, match="rank out of range"):
        mp.shard(2)


def test_multi_plan_two_gpus(cuda):
    """Two distinct GPUs: peer-to-peer replica copy and peer gather into device 0."""
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rhs = 64
    host = spec_case(1024, 16, 3, False, 1)
    K, M = host.scalar_cols(), host.scalar_rows()
    B = vb.fill_uniform(1, vb.STREAM_DENSE, 0, K * rhs)
    mp = vb.MultiPlan(host, [0, 1], vb.PlanOptions(rhs))
    assert {mp.shard(0).device, mp.shard(1).device} == {0, 1}
    mp.replicate_B(torch.from_numpy(B).cuda(0))
    mp.execute()
    mp.synchronize()
    dC = torch.empty(M * rhs, device="cuda:0")
    mp.gather_C(dC)
    assert_within_bound(host, B, rhs, dC.cpu().numpy())


def _replica_rank(rank, world, port, result_path):
    import os
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    import json
    import torch
    import torch.distributed as dist

    import oracle
    import varblockspmm_b200 as vb
    from varblockspmm_b200.replica import PeerReplica

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    rhs = 32
    host = spec_case(700, 8, 2, False, 5)
    K = host.scalar_cols()
    B = vb.fill_uniform(5, vb.STREAM_DENSE, 0, K * rhs)
    rep = PeerReplica(K * rhs, rank, world, dev, dist.group.WORLD, buffers=2)
    out = {}
    # setup form: the root holds B, everyone pulls
    if rank == 0:
        vb.fill_uniform_device(5, vb.STREAM_DENSE, 0, K * rhs, rep.ptr(0))
        torch.cuda.synchronize()
    rep.replicate_from(0, 0)
    got = torch.empty(K * rhs, device="cuda")
    from varblockspmm_b200.replica import copy_async
    copy_async(got.data_ptr(), rep.ptr(0), 4 * K * rhs)
    torch.cuda.synchronize()
    g = got.cpu().numpy()
    out["replicate_equal"] = bool(np.array_equal(g.view(np.uint32), B.view(np.uint32)))
    out["replicate_mismatch"] = int(np.count_nonzero(g.view(np.uint32) != B.view(np.uint32)))
    # per-step form: own chunk from pinned host memory, the rest from the peers
    hB = torch.from_numpy(B).pin_memory()
    up = rep.upload_own_chunk(hB.data_ptr(), 1)
    torch.cuda.synchronize()
    rep.barrier()
    pulled = rep.pull_peers(1)
    torch.cuda.synchronize()
    rep.barrier()
    out["bytes"] = up + pulled
    copy_async(got.data_ptr(), rep.ptr(1), 4 * K * rhs)
    torch.cuda.synchronize()
    out["upload_pull_equal"] = bool(np.array_equal(got.cpu().numpy().view(np.uint32),
                                                   B.view(np.uint32)))
    # this rank's shard multiplied with the replica
    bounds = vb.partition_rows(host, world, rhs)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    m = vb.Matrix(host, device=dev, rows=(r0, r1))
    p = vb.Plan(m, vb.PlanOptions(rhs))
    M_r = int(host.row_scalar_off[r1] - host.row_scalar_off[r0])
    dC = torch.full((M_r * rhs,), float("nan"), device="cuda")
    p.execute(rep.ptr(1), dC)
    torch.cuda.synchronize()
    p.check_status()
    ratio, _, bad = oracle.compare(host, B, rhs, dC.cpu().numpy(), r0, r1)
    out["violations"] = int(bad)
    del p, m
    rep.close()
    with open(f"{result_path}.{rank}", "w") as f:
        json.dump(out, f)
    dist.barrier()
    dist.destroy_process_group()


def test_peer_replica_two_processes(cuda, tmp_path):
    """Two processes (one per GPU, or both on GPU 0 on a one-GPU box) share their B buffers
    through CUDA IPC: replicate_from(root) and the upload-own-chunk + pull-peers form both give
    every rank all of B bit for bit, and each rank's shard multiplied with its replica meets the
    bound."""
    import json
    import socket
    import torch.multiprocessing as tmp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    base = str(tmp_path / "rank")
    tmp.start_processes(_replica_rank, args=(2, port, base), nprocs=2, join=True,
                        start_method="spawn")
    outs = [json.load(open(f"{base}.{r}")) for r in range(2)]
    for out in outs:
        assert out["replicate_equal"] and out["upload_pull_equal"], outs
        assert out["violations"] == 0
