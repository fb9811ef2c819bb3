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
