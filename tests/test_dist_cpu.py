"""The N > 1 host logic of the benchmark on CPU: two gloo ranks on 127.0.0.1.

Covers what bench.py does around the device execute when it runs one process per GPU:
- the balanced block-row partition (vbsr_partition_rows) seen identically by both ranks;
- the B replica broadcast from rank 0;
- the max-over-ranks reduction of step times;
- the verification gather (bench.gathered_parity): every rank's C block sent to rank 0,
  reassembled into the M x N column-major result and checked against the oracle for rows of
  every shard.
The per-shard C comes from the oracle here, standing in for the device execute, which needs a
GPU; the gather must reproduce the full-matrix oracle result exactly.
"""
import json
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist

    import bench
    import oracle
    import varblockspmm_b200 as vb
    from helpers import spec_case

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rhs = 16
    host = spec_case(300, 6, 2, False, bench.SEED)
    bounds = vb.partition_rows(host, world, rhs)
    # both ranks derive the same partition
    seen = [None] * world
    dist.all_gather_object(seen, [int(x) for x in bounds])
    assert all(s == seen[0] for s in seen)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])

    # B: generated on rank 0, replicated by broadcast
    K = host.scalar_cols()
    B = torch.zeros(K * rhs, dtype=torch.float32)
    if rank == 0:
        B.copy_(torch.from_numpy(vb.fill_uniform(bench.SEED, vb.STREAM_DENSE, 0, K * rhs)))
    dist.broadcast(B, src=0)
    B_np = B.numpy()

    # this rank's C block (stand-in for Plan.execute on its shard)
    C_r = torch.from_numpy(np.ascontiguousarray(oracle.spmm(host, B_np, rhs, r0, r1)))
    if C_r.numel() == 0:
        C_r = torch.zeros(1)

    # step time: max over ranks
    t = torch.tensor([1.0 + rank], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    assert t.item() == float(world)

    res = bench.gathered_parity(host, rhs, bounds, rank, world, C_r, B_np, per_shard=3)
    if rank == 0:
        with open(result_path, "w") as f:
            json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_partition_broadcast_gather(tmp_path):
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp

    result = tmp_path / "rank0.txt"
    mp.start_processes(_rank_main, args=(2, _free_port(), str(result)), nprocs=2, join=True,
                       start_method="spawn")
    res = json.loads(result.read_text())  # what rank 0 wrote
    assert res["violations"] == 0
    assert res["rows_checked"] >= 4  # rows of both shards
    assert res["max_err_over_bound"] == 0.0  # the oracle's own blocks, reassembled exactly
