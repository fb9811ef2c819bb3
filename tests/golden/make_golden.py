"""Generates tests/golden/ fixtures from the reference itself.

Runs the reference's own generate() and cpu_reference() (King-Clawthorne/VarBlockSpMM
src/format/generator.cpp, src/format/vbsr.cpp, compiled unchanged by oracle/Makefile into
oracle/_ref/libvbsr_ref.so) on
  * the reference test suite's 64-case parameter matrix (tests/test_main.cpp:61-73,145-161):
    9 x 17 block rows/columns, distributions x degrees {1,4,8,16} x RHS {8,16,32,64}, seeds
    11..74, local columns when the seed is odd, B = std::mt19937(seed) U[-1,1]
    (test_main.cpp:42-51);
  * two larger reference-generator cases (256 x 256 blocks),
and records SHA-256 digests of every generated array, of B and of the reference C, plus the full
arrays of three small cases (golden_arrays.npz). The reference checkout is needed only to
regenerate; the fixtures themselves are committed.

Usage: python tests/golden/make_golden.py
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
import varblockspmm_b200 as vb  # noqa: E402

ARRAYS = ["row_ptr", "block_col", "row_size", "col_size", "row_scalar_off", "col_scalar_off",
          "value_off", "values"]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def case_list():
    cases = []
    seed = 11
    for dist in range(4):
        for degree in (1, 4, 8, 16):
            for rhs in (8, 16, 32, 64):
                cases.append(dict(rows=9, cols=17, degree=degree, distribution=dist,
                                  local=bool(seed & 1), rhs=rhs, seed=seed))
                seed += 1
    cases.append(dict(rows=256, cols=256, degree=4, distribution=2, local=True, rhs=8, seed=1))
    cases.append(dict(rows=256, cols=256, degree=16, distribution=3, local=False, rhs=64, seed=7))
    return cases


def main():
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libvbsr_ref.so is missing: run `make -C oracle` with the reference")
    out, full = [], {}
    for i, c in enumerate(case_list()):
        r = oracle.ref_generate(c["rows"], c["cols"], c["degree"], c["distribution"], c["local"],
                                c["seed"])
        host = vb.HostMatrix(r["block_rows"], r["block_cols"], *[r[k] for k in ARRAYS])
        B = vb.fill_mt19937(c["seed"], host.scalar_cols() * c["rhs"])
        Cref = oracle.ref_cpu_reference(host, B, c["rhs"], threads=1)
        entry = dict(c)
        entry["sha"] = {k: sha(r[k]) for k in ARRAYS}
        entry["sha_B"] = sha(B)
        entry["sha_C"] = sha(Cref)
        entry["sum_C"] = float(np.sum(Cref, dtype=np.float64))
        entry["nnzb"] = int(host.nnzb)
        out.append(entry)
        if i in (0, 17, 49):
            for k in ARRAYS:
                full[f"c{i}_{k}"] = r[k]
            full[f"c{i}_B"] = B
            full[f"c{i}_C"] = Cref
            full[f"c{i}_dims"] = np.array([r["block_rows"], r["block_cols"], c["rhs"]])
    with open(os.path.join(HERE, "golden_cases.json"), "w") as f:
        json.dump({"generator": "reference generate() + cpu_reference(), compiled unchanged",
                   "cases": out}, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "golden_arrays.npz"), **full)
    print(f"wrote {len(out)} cases; full arrays for {sorted({k.split('_')[0] for k in full})}")


if __name__ == "__main__":
    main()
