"""The reference's own GPU path (Matrix, Plan, row-owned CUDA kernels, compiled unchanged for
sm_100a into oracle/_ref/libvbsr_ref_gpu.so) on the same GPU and inputs as the engine.

Checks that the reference's kernels also meet the parity bound on this GPU, that the engine's C
agrees with theirs, and reports both device times. Each time is a median of CUDA-event
intervals over 30 launches with L2 flushed before each launch. The timings are printed, not
asserted: they are a side-by-side comparison on one B200, and the bench and the profiles hold
the measured numbers.
"""
import numpy as np
import pytest

import oracle
import varblockspmm_b200 as vb
from helpers import assert_within_bound, spec_case

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.ref_gpu_available(),
                                 reason="the reference's GPU library is not built")]

CASES = [
    # name, block rows, degree, distribution, local, rhs
    ("C1", 256, 4, 0, True, 8),
    ("C2", 1024, 16, 3, False, 64),
    ("C3-headline", 4096, 8, 2, False, 32),
    ("C4-like-rhs16", 1024, 8, 1, False, 16),
    ("C5-shape-16k", 16384, 16, 2, False, 64),
]


def _median_us(torch, fn, flush, n=30):
    times = []
    for i in range(n + 3):
        flush.fill_(float(i))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(a.elapsed_time(b) * 1e3)
    return float(np.median(times))


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0])
def test_reference_kernels_side_by_side(cuda, case):
    torch = cuda
    name, rows, degree, dist, local, rhs = case
    host = spec_case(rows, degree, dist, local, 1)
    K, M = host.scalar_cols(), host.scalar_rows()
    B = vb.fill_uniform(1, vb.STREAM_DENSE, 0, K * rhs)
    dB = torch.from_numpy(B).cuda()

    ref = oracle.RefGpuPlan(host, rhs)
    dC_ref = torch.full((M * rhs,), float("nan"), device="cuda")
    ref.execute(dB.data_ptr(), dC_ref.data_ptr())
    torch.cuda.synchronize()
    c_ref = dC_ref.cpu().numpy()
    assert_within_bound(host, B, rhs, c_ref)  # the reference's kernels meet the bar here too

    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    dC = torch.full((M * rhs,), float("nan"), device="cuda")
    p.execute(dB, dC)
    torch.cuda.synchronize()
    c = dC.cpu().numpy()
    assert_within_bound(host, B, rhs, c)
    scale = float(np.max(np.abs(c_ref))) or 1.0
    assert float(np.max(np.abs(c - c_ref))) <= 1e-4 * scale

    flush = torch.empty(64 << 20, device="cuda")  # 256 MB, twice the L2
    t_ref = _median_us(torch, lambda: ref.execute(dB.data_ptr(), dC_ref.data_ptr()), flush)
    t_eng = _median_us(torch, lambda: p.execute(dB, dC), flush)
    nbytes, _ = vb.compulsory_bytes(host, rhs)
    print(f"\n[reference-vs-engine] {name}: rows={rows} deg={degree} rhs={rhs} "
          f"reference {t_ref:.1f} us ({nbytes / t_ref / 1e3:.0f} GB/s, {ref.launch_count()} "
          f"launch(es)), engine {t_eng:.1f} us ({nbytes / t_eng / 1e3:.0f} GB/s), "
          f"speed-up {t_ref / t_eng:.2f}x")
    ref.close()
