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
