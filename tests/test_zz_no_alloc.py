"""The execute entry point that allocates nothing (vbsr_plan_execute_noalloc).

Some callers cannot let a library allocate device memory for them: hosts that own every device
allocation through their own pool, or code paths where cudaMalloc/cudaFree (which synchronise the
device) are forbidden. For them the kernel's scratch (status words, per-CTA timestamps) lives in a
fixed array compiled into the library. This test calls that entry point through the C ABI twice in
a row and checks both results against the regular vbsr_plan_execute, under the parity tests' bound
|C - C_ref| <= 1e-5 * sum|a||b| (and, since both run the same kernel, bit for bit).

The file is named so that pytest collects it last; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

import varblockspmm_b200 as vb
from helpers import assert_within_bound, spec_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("flags", [0, vb.PLAN_FUSED_PREPASS], ids=["two_launches", "fused"])
@pytest.mark.parametrize("rhs", [32, 64])
def test_noalloc_matches_execute_twice(cuda, rhs, flags):
    torch = cuda
    host = spec_case(1024, 8, 2, False, 21)
    B = vb.fill_uniform(21, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs), flags)
    dB = torch.from_numpy(B).cuda()
    n = host.scalar_rows() * rhs
    ref = torch.full((n,), float("nan"), device="cuda")
    p.execute(dB, ref)
    torch.cuda.synchronize()
    p.check_status()
    ref_h = ref.cpu().numpy()
    assert_within_bound(host, B, rhs, ref_h)
    stream = torch.cuda.Stream()
    for call in range(2):
        out = torch.full((n,), float("nan"), device="cuda")
        stream.wait_stream(torch.cuda.current_stream())  # the NaN fill lands before the kernel
        times = p.execute_noalloc(dB, out, stream, report=True)
        got = out.cpu().numpy()
        assert_within_bound(host, B, rhs, got)
        assert np.array_equal(got.view(np.uint32), ref_h.view(np.uint32)), f"call {call}"
        assert times.shape == (p.num_tasks(), 2)
        assert np.all(times[:, 1] >= times[:, 0]) and np.all(times[:, 0] > 0)
    # asynchronous form (no reporting) gives the same C as well
    out = torch.full((n,), float("nan"), device="cuda")
    stream.wait_stream(torch.cuda.current_stream())
    p.execute_noalloc(dB, out, stream)
    stream.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref_h.view(np.uint32))
