"""Shared helpers for the test suite (inputs, device round trips, tolerance checks)."""
import numpy as np

import oracle
import varblockspmm_b200 as vb


def ref_case(rows, cols, degree, dist, local, seed):
    """Reference-profile matrix (bit-identical to the reference generator)."""
    return vb.generate(vb.GeneratorOptions(rows, cols, degree, 32, vb.Distribution(dist), local,
                                           seed, vb.Profile.Reference))


def spec_case(rows, degree, dist, local, seed, with_values=True):
    return vb.generate(vb.GeneratorOptions(rows, rows, degree, 32, vb.Distribution(dist), local,
                                           seed, vb.Profile.Spec), with_values=with_values)


def run_plan(torch, host, B, rhs, flags=0, stream=None, matrix=None, plan=None):
    """Uploads host + B, runs one Plan.execute on `stream`, returns C (numpy, col-major)."""
    m = matrix or vb.Matrix(host)
    p = plan or vb.Plan(m, vb.PlanOptions(rhs), flags)
    dB = torch.from_numpy(np.asarray(B, dtype=np.float32)).cuda()
    dC = torch.full((host.scalar_rows() * rhs,), float("nan"), device="cuda", dtype=torch.float32)
    p.execute(dB, dC, stream)
    if stream is not None:
        stream.synchronize()
    torch.cuda.synchronize()
    p.check_status(stream)
    return dC.cpu().numpy()


def reference_test_tolerance(ref, got):
    """The reference test's acceptance check (tests/test_main.cpp:14-40): finite, max|err| <= 5e-4,
    relative L2 <= 5e-5."""
    assert np.all(np.isfinite(got)), "NaN/Inf in result"
    err = got.astype(np.float64) - ref.astype(np.float64)
    max_err = float(np.max(np.abs(err))) if err.size else 0.0
    rel = float(np.sqrt(np.sum(err * err) / (np.sum(ref.astype(np.float64) ** 2) + 1e-30)))
    assert max_err <= 5e-4 and rel <= 5e-5, (max_err, rel)


def assert_within_bound(host, B, rhs, got, r0=0, r1=None):
    """|C - C_ref| <= 1e-5 * sum|a||b| per element (the engine's parity bar)."""
    ratio, max_abs, bad = oracle.compare(host, B, rhs, got, r0, r1)
    assert bad == 0, f"{bad} elements outside 1e-5*sum|a||b| (max ratio {ratio}, max abs {max_abs})"
    return ratio
