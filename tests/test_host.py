"""CPU tests of the host side: validation (against the reference's own validate()), the spec
generator, the counter-based generator, the partition and the byte model."""
import numpy as np
import pytest

import oracle
import varblockspmm_b200 as vb
from helpers import ref_case, spec_case


def test_negative_cases_of_reference_suite():
    """tests/test_main.cpp:116-130: row_ptr.back()++ and row_size[0]=7 must be rejected."""
    valid = ref_case(4, 4, 2, 2, True, 1)
    valid.validate()
    bad = valid.copy()
    bad.row_ptr[-1] += 1
    with pytest.raises(vb.InvalidArgument, match="bad row_ptr"):
        bad.validate()
    bad = valid.copy()
    bad.row_size[0] = 7
    with pytest.raises(vb.InvalidArgument, match="bad block row"):
        bad.validate()


def _mutations(m, rng):
    """Single-field corruptions of a valid matrix, one per validate() check."""
    out = []
    def mut(f):
        c = m.copy()
        f(c)
        out.append(c)
    mut(lambda c: setattr(c, "block_rows", 0))
    mut(lambda c: setattr(c, "row_size", c.row_size[:-1]))
    mut(lambda c: setattr(c, "col_scalar_off", c.col_scalar_off[:-1]))
    mut(lambda c: c.row_ptr.__setitem__(0, 1))
    mut(lambda c: setattr(c, "values", c.values[:-1]))
    mut(lambda c: c.value_off.__setitem__(0, 1))
    mut(lambda c: c.row_size.__setitem__(1, 72))
    mut(lambda c: c.row_size.__setitem__(2, 12))
    mut(lambda c: c.col_size.__setitem__(0, 0))
    mut(lambda c: c.col_scalar_off.__setitem__(1, c.col_scalar_off[1] + 8))
    mut(lambda c: c.block_col.__setitem__(0, c.block_cols))
    mut(lambda c: c.block_col.__setitem__(1, -1))
    mut(lambda c: c.value_off.__setitem__(1, c.value_off[1] + 8))
    def swap_rows(c):
        c.row_ptr[1], c.row_ptr[2] = c.row_ptr[2], c.row_ptr[1]
    mut(swap_rows)
    for _ in range(20):
        c = m.copy()
        arr = [c.row_ptr, c.block_col, c.row_size, c.col_size, c.row_scalar_off,
               c.col_scalar_off, c.value_off][rng.integers(7)]
        i = rng.integers(arr.size)
        arr[i] += rng.choice([-8, -1, 1, 8])
        out.append(c)
    return out


@pytest.mark.skipif(not oracle.ref_available(), reason="reference not built here")
def test_validation_agrees_with_reference():
    rng = np.random.default_rng(0)
    m = ref_case(6, 9, 3, 3, False, 5)
    for c in _mutations(m, rng):
        code, msg = oracle.ref_validate(c)
        try:
            c.validate()
            mine = (0, "")
        except vb.InvalidArgument as e:
            mine = (1, str(e))
        assert mine == (code, msg), (mine, code, msg)


def test_validation_messages_without_reference():
    rng = np.random.default_rng(1)
    m = ref_case(6, 9, 3, 3, False, 5)
    seen = set()
    for c in _mutations(m, rng)[:14]:  # the deterministic corruptions always invalidate
        with pytest.raises(vb.InvalidArgument) as e:
            c.validate()
        seen.add(str(e.value))
    assert {"bad row_ptr", "bad block row", "bad block column", "bad value offsets",
            "block column out of range", "block payload mismatch", "metadata size mismatch",
            "scalar offsets size mismatch", "positive block dimensions required"} <= seen


def test_generator_rejects_bad_dimensions():
    for kw in (dict(degree=0), dict(degree=17), dict(block_rows=0), dict(block_cols=3, degree=4)):
        o = vb.GeneratorOptions(block_rows=8, block_cols=8, degree=2)
        for k, v in kw.items():
            setattr(o, k, v)
        with pytest.raises(vb.InvalidArgument, match="invalid generator dimensions"):
            vb.generate(o)


def test_spec_distributions():
    """Block-size frequencies of the benchmark specification's four distributions."""
    n = 20000
    def sizes(dist):
        m = spec_case(n, 1, dist, False, 3, with_values=False)
        return np.concatenate([m.row_size, m.col_size])
    s = sizes(2)  # high variance
    for v, p in ((8, .3), (16, .2), (56, .2), (64, .3)):
        assert abs(np.mean(s == v) - p) < 0.01
    assert set(np.unique(s)) == {8, 16, 56, 64}
    s = sizes(3)
    assert set(np.unique(s)) == {8, 64} and abs(np.mean(s == 8) - .5) < .01
    s = sizes(1)
    assert abs(np.mean(s == 32) - .5) < .01 and abs(np.mean(s == 24) - .25) < .01
    assert set(np.unique(s)) == {24, 32, 40}
    s = sizes(0)
    assert set(np.unique(s)) == set(range(8, 65, 8))


def test_spec_local_window_clamped():
    m = spec_case(300, 16, 0, True, 9, with_values=False)
    for i in range(m.block_rows):
        cols = m.block_col[m.row_ptr[i]:m.row_ptr[i + 1]]
        lo = min(max(i - 8, 0), m.block_cols - 17)
        assert len(cols) == 16 and len(set(cols)) == 16 and np.all(np.diff(cols) > 0)
        assert cols.min() >= lo and cols.max() <= lo + 16


def test_spec_random_pattern_and_values():
    m = spec_case(64, 8, 2, False, 4)
    m.validate()
    for i in range(m.block_rows):
        cols = m.block_col[m.row_ptr[i]:m.row_ptr[i + 1]]
        assert len(cols) == 8 and np.all(np.diff(cols) > 0)
    # values are the counter-based stream at their packed index
    assert np.array_equal(m.values, vb.fill_uniform(4, vb.STREAM_VALUES, 0, m.values.size))
    s = spec_case(64, 8, 2, False, 4, with_values=False)
    assert s.values.size == 0 and np.array_equal(s.value_off, m.value_off)


def test_counter_rng_properties():
    a = vb.fill_uniform(1, vb.STREAM_DENSE, 0, 1 << 20, threads=4)
    b = vb.fill_uniform(1, vb.STREAM_DENSE, 12345, 1000, threads=1)
    assert np.array_equal(a[12345:13345], b)
    assert a.min() >= -1.0 and a.max() < 1.0
    assert abs(a.mean()) < 5e-3 and abs(a.var() - 1 / 3) < 5e-3
    # exact multiples of 2^-23
    assert np.all((a * 8388608.0) == np.round(a * 8388608.0))
    c = vb.fill_uniform(2, vb.STREAM_DENSE, 0, 1000)
    assert not np.array_equal(a[:1000], c)


def test_partition_balanced_and_monotone():
    m = spec_case(4096, 8, 2, False, 1, with_values=False)
    for parts in (1, 2, 4, 8):
        b = vb.partition_rows(m, parts, 64)
        assert b[0] == 0 and b[-1] == m.block_rows and np.all(np.diff(b) >= 0)
        w = m.col_size[m.block_col].astype(np.float64)
        h = np.repeat(m.row_size, np.diff(m.row_ptr)).astype(np.float64)
        per_block = 4 * h * w + 4 * 64 * w  # A bytes + staged B bytes
        pre = np.concatenate([[0], np.cumsum(per_block)])
        cost = [pre[m.row_ptr[b[k + 1]]] - pre[m.row_ptr[b[k]]] for k in range(parts)]
        assert max(cost) / (sum(cost) / parts) < 1.02


def test_compulsory_bytes_formula():
    m = spec_case(256, 4, 0, True, 1)
    N = 8
    R = S = 256
    nnzb = m.nnzb
    K, M = m.scalar_cols(), m.scalar_rows()
    expect = (4 * m.values.size + 4 * nnzb + 8 * (nnzb + 1) + 4 * (R + 1) + 4 * R + 8 * (R + 1)
              + 4 * S + 8 * (S + 1) + 4 * K * N + 4 * M * N)
    by, fl = vb.compulsory_bytes(m, N)
    assert by == expect and fl == 2 * m.values.size * N


@pytest.mark.parametrize("grid", [1, 2, 3, 7, 148])
def test_fused_prepass_arrival_word(grid):
    """The fused pre-pass's grid arrival (stack_arrive in vbsr_tc.cuh), restated on uint32: CTA 0
    adds 2^31 - (grid - 1), every other CTA adds 1, in any order. Over many launches from any
    starting low bits of 0, the top bit differs from the one each CTA saw at its own arrival
    exactly once every CTA has arrived, and the word's low bits return to 0 after each launch, so
    it needs no reset between executes."""
    rng = np.random.default_rng(grid)
    word = 0
    for launch in range(6):
        order = rng.permutation(grid)
        seen = {}
        for n, cta in enumerate(order):
            add = (0x80000000 - (grid - 1)) if cta == 0 else 1
            seen[cta] = word & 0x80000000
            word = (word + add) & 0xFFFFFFFF
            done = all(((word ^ seen[c]) & 0x80000000) != 0 for c in seen)
            # no waiter may pass before the last arrival; every waiter passes at it
            assert done == (n == grid - 1), (launch, n)
        assert word & 0x7FFFFFFF == 0
