"""Real matrices into the engine: scalar CSR -> VBSR for a block partition, Matrix Market files, and
the binary VBSR file (vbsr_io.cpp). CPU only; the GPU run of a converted matrix is in
tests/test_gpu_parity.py."""
import os

import numpy as np
import pytest
import scipy.io
import scipy.sparse as sp

import oracle
import varblockspmm_b200 as vb


def to_dense(m):
    """The scalar matrix a VBSR host matrix stands for."""
    A = np.zeros((m.scalar_rows(), m.scalar_cols()), dtype=np.float64)
    for i in range(m.block_rows):
        r0, h = int(m.row_scalar_off[i]), int(m.row_size[i])
        for b in range(int(m.row_ptr[i]), int(m.row_ptr[i + 1])):
            j = int(m.block_col[b])
            c0, w = int(m.col_scalar_off[j]), int(m.col_size[j])
            v = m.values[int(m.value_off[b]):int(m.value_off[b + 1])]
            A[r0:r0 + h, c0:c0 + w] = v.reshape(w, h).T
    return A


@pytest.mark.parametrize("shape,density,rb,cb", [((96, 160), 0.05, 32, 16), ((512, 256), 0.01, 64, 8),
                                                  ((64, 64), 0.3, 8, 64), ((40, 48), 0.0, 8, 8)])
def test_from_csr_reproduces_the_matrix(shape, density, rb, cb):
    a = sp.random(*shape, density=density, random_state=7, format="csr", dtype=np.float32)
    m = vb.from_csr(shape, a.indptr, a.indices, a.data, vb.block_sizes(shape[0], rb),
                    vb.block_sizes(shape[1], cb))
    m.validate()
    assert np.array_equal(to_dense(m), a.toarray().astype(np.float64))
    # only blocks that hold a nonzero are stored
    for b in range(m.nnzb):
        assert np.any(m.values[int(m.value_off[b]):int(m.value_off[b + 1])] != 0)
    # and the oracle's product is the dense product (within the tolerance the engine is held to)
    rhs = 16
    B = np.random.default_rng(1).uniform(-1, 1, shape[1] * rhs).astype(np.float32)
    C, S = oracle.spmm(m, B, rhs, bound=True)
    ref = a.toarray().astype(np.float64) @ B.reshape(rhs, shape[1]).T.astype(np.float64)
    assert np.all(np.abs(C.reshape(rhs, shape[0]).T - ref) <= 1e-5 * S.reshape(rhs, shape[0]).T + 1e-30)


def test_from_csr_sums_duplicates_and_rejects_bad_partitions():
    indptr = np.array([0, 2] + [2] * 7, dtype=np.int64)
    m = vb.from_csr((8, 8), indptr, [3, 3], [1.5, 2.0], [8], [8])
    assert to_dense(m)[0, 3] == 3.5
    with pytest.raises(vb.InvalidArgument, match="multiples of 8"):
        vb.from_csr((12, 8), np.zeros(13, dtype=np.int64), [], [], [12], [8])
    with pytest.raises(vb.InvalidArgument, match="do not sum"):
        vb.from_csr((16, 8), np.zeros(17, dtype=np.int64), [], [], [8], [8])
    with pytest.raises(vb.InvalidArgument, match="out of range"):
        vb.from_csr((8, 8), np.array([0, 1] + [1] * 7), [9], [1.0], [8], [8])


def test_matrix_market_and_vbsr_file_round_trip(tmp_path):
    a = sp.random(203, 130, density=0.03, random_state=3, format="coo", dtype=np.float32)
    mtx = os.path.join(tmp_path, "a.mtx")
    scipy.io.mmwrite(mtx, a)
    m, shape = vb.load_matrix_market(mtx, row_block=32, col_block=24)
    assert shape == (203, 130)
    assert (m.scalar_rows(), m.scalar_cols()) == (208, 136)  # padded to multiples of 8
    dense = to_dense(m)
    assert np.array_equal(dense[:203, :130], a.toarray().astype(np.float64))
    assert not dense[203:].any() and not dense[:, 130:].any()
    f = os.path.join(tmp_path, "a.vbsr")
    m.save(f)
    back = vb.load_matrix(f)
    for k in ("row_ptr", "block_col", "row_size", "col_size", "row_scalar_off", "col_scalar_off",
              "value_off", "values"):
        assert np.array_equal(getattr(back, k), getattr(m, k)), k
    raw = open(f, "rb").read()
    bad = os.path.join(tmp_path, "bad.vbsr")
    open(bad, "wb").write(b"NOTVBSR!" + raw[8:])
    with pytest.raises(vb.InvalidArgument, match="magic"):
        vb.load_matrix(bad)
    open(bad, "wb").write(raw[:len(raw) // 2])
    with pytest.raises(vb.InvalidArgument, match="truncated"):
        vb.load_matrix(bad)
    with pytest.raises(vb.InvalidArgument, match="cannot open"):
        vb.load_matrix(os.path.join(tmp_path, "missing.vbsr"))
