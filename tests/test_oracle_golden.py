"""Pins the CPU oracle (oracle/vbsr_oracle.c) and the engine's reference-profile generator against
fixtures produced by the reference itself (tests/golden/make_golden.py)."""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle
import varblockspmm_b200 as vb

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "golden_cases.json")))["cases"]
ARRAYS = ["row_ptr", "block_col", "row_size", "col_size", "row_scalar_off", "col_scalar_off",
          "value_off", "values"]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("idx", [0, 17, 49])
def test_oracle_bitwise_on_reference_arrays(idx):
    """Oracle C from the reference's own arrays is bit-identical to the reference's C."""
    z = np.load(os.path.join(HERE, "golden", "golden_arrays.npz"))
    rows, cols, rhs = (int(x) for x in z[f"c{idx}_dims"])
    host = vb.HostMatrix(rows, cols, *[z[f"c{idx}_{k}"] for k in ARRAYS])
    host.validate()
    got = oracle.spmm(host, z[f"c{idx}_B"], rhs)
    assert np.array_equal(got.view(np.uint32), z[f"c{idx}_C"].view(np.uint32))


@pytest.mark.parametrize("case", GOLDEN, ids=lambda c: f"s{c['seed']}d{c['degree']}r{c['rhs']}")
def test_generator_and_oracle_match_reference(case):
    host = vb.generate(vb.GeneratorOptions(case["rows"], case["cols"], case["degree"], case["rhs"],
                                           vb.Distribution(case["distribution"]), case["local"],
                                           case["seed"], vb.Profile.Reference))
    for k in ARRAYS:
        assert sha(getattr(host, k)) == case["sha"][k], k
    B = vb.fill_mt19937(case["seed"], host.scalar_cols() * case["rhs"])
    assert sha(B) == case["sha_B"]
    got = oracle.spmm(host, B, case["rhs"], threads=2)
    assert sha(got) == case["sha_C"]


@pytest.mark.skipif(not oracle.ref_available(), reason="reference not built here")
def test_oracle_vs_live_reference_threaded():
    """Against the reference compiled from its sources (when present): a bigger random case."""
    host = vb.generate(vb.GeneratorOptions(300, 300, 16, 64, vb.Distribution.Bimodal, False, 3))
    B = vb.fill_mt19937(3, host.scalar_cols() * 64)
    a = oracle.spmm(host, B, 64, threads=4)
    b = oracle.ref_cpu_reference(host, B, 64, threads=3)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("case", [(256, 256, 4, 0, True, 1), (1024, 1024, 16, 3, False, 1),
                                  (4096, 4096, 8, 2, False, 1), (1024, 1024, 8, 1, True, 7),
                                  (300, 40, 16, 2, False, 3)])
def test_workload_generator_matches_engine(case):
    """The oracle's own workload generator (used by the benchmark's reference arm, which must not
    load the engine) gives the engine generator's spec-profile matrices bit for bit."""
    rows, cols, degree, dist, local, seed = case
    w = oracle.WorkloadMatrix(rows, cols, degree, dist, local, seed, with_values=True)
    e = vb.generate(vb.GeneratorOptions(rows, cols, degree, 32, vb.Distribution(dist), local, seed,
                                        vb.Profile.Spec))
    for f in ("row_ptr", "block_col", "row_size", "col_size", "row_scalar_off",
              "col_scalar_off", "value_off"):
        assert np.array_equal(np.asarray(getattr(w, f), dtype=np.int64),
                              np.asarray(getattr(e, f), dtype=np.int64)), f
    assert np.array_equal(w.values.view(np.uint32), e.values.view(np.uint32))
    s = w.row_slice(rows // 3, rows // 2)
    t = e.row_slice(rows // 3, rows // 2)
    assert np.array_equal(s.values.view(np.uint32), t.values.view(np.uint32))
    assert np.array_equal(s.value_off, t.value_off)


def test_workload_dense_stream_matches_engine():
    a = oracle.fill_uniform(1, oracle.STREAM_DENSE, 12345, 200_000)
    b = vb.fill_uniform(1, vb.STREAM_DENSE, 12345, 200_000)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
def test_ref_timer_matches_oracle():
    """The prepared reference run (the benchmark's timed reference arm) computes the reference's
    C: bit-identical to the oracle restatement."""
    w = oracle.WorkloadMatrix(512, 512, 8, 2, False, 5, with_values=True)
    B = oracle.fill_uniform(5, oracle.STREAM_DENSE, 0, w.scalar_cols() * 32)
    t = oracle.RefTimer(w, B, 32, threads=3)
    C = np.empty(w.scalar_rows() * 32, dtype=np.float32)
    sec = t.run(C)
    assert sec > 0
    assert np.array_equal(C.view(np.uint32), oracle.spmm(w, B, 32).view(np.uint32))
