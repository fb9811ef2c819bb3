"""Parity of the engine's CUDA path with the oracle, through the C ABI (Plan.execute).

Bar: every element within |C - C_ref| <= 1e-5 * sum_k |a_ik||b_kj| (C_ref = the reference's
double-accumulating CPU path, restated bit-exactly by the oracle), plus the reference test
suite's own acceptance check (finite, max abs error <= 5e-4, relative L2 <= 5e-5).
"""
import json
import os

import numpy as np
import pytest

import oracle
import varblockspmm_b200 as vb
from helpers import assert_within_bound, ref_case, reference_test_tolerance, run_plan, spec_case

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "golden_cases.json")))["cases"]


@pytest.mark.parametrize("case", GOLDEN, ids=lambda c: f"s{c['seed']}d{c['degree']}r{c['rhs']}")
def test_reference_parameter_matrix(cuda, case):
    """The reference suite's 64-case matrix (tests/test_main.cpp:145-161) and two 256-row cases,
    on a non-default stream, for the planned kernel and both raw launchers."""
    torch = cuda
    host = ref_case(case["rows"], case["cols"], case["degree"], case["distribution"],
                    case["local"], case["seed"])
    rhs = case["rhs"]
    B = vb.fill_mt19937(case["seed"], host.scalar_cols() * rhs)
    ref = oracle.spmm(host, B, rhs)
    stream = torch.cuda.Stream()
    got = run_plan(torch, host, B, rhs, stream=stream)
    reference_test_tolerance(ref, got)
    assert_within_bound(host, B, rhs, got)

    m = vb.Matrix(host)
    dB = torch.from_numpy(B).cuda()
    for launcher in (vb.launch_row_owned, vb.launch_row_owned_scalar):
        dC = torch.full((host.scalar_rows() * rhs,), float("nan"), device="cuda")
        launcher(m.device_view(), dB, dC, rhs, stream)
        stream.synchronize()
        out = dC.cpu().numpy()
        reference_test_tolerance(ref, out)
        assert_within_bound(host, B, rhs, out)


def test_plan_rejects_bad_options(cuda):
    """tests/test_main.cpp:132-142: RHS 7 and Kernel::SplitRow raise invalid_argument."""
    m = vb.Matrix(ref_case(4, 4, 2, 2, True, 1))
    with pytest.raises(vb.InvalidArgument, match="rhs_width must be 8,16,32,64"):
        vb.Plan(m, vb.PlanOptions(7, vb.Kernel.RowOwned))
    with pytest.raises(vb.InvalidArgument, match="split-row"):
        vb.Plan(m, vb.PlanOptions(8, vb.Kernel.SplitRow))
    p = vb.Plan(m, vb.PlanOptions(8, vb.Kernel.Auto))
    assert p.launch_count() == 2  # B pre-pass + SpMM kernel


def test_matrix_rejects_invalid_host(cuda):
    bad = ref_case(4, 4, 2, 2, True, 1)
    bad.row_ptr[-1] += 1
    with pytest.raises(vb.InvalidArgument, match="bad row_ptr"):
        vb.Matrix(bad)


@pytest.mark.parametrize("cfg", [
    ("C1", 256, 4, 0, True, 8),
    ("C2", 1024, 16, 3, False, 64),
    ("C3", 4096, 8, 2, False, 32),
], ids=lambda c: c[0])
def test_baseline_configs(cuda, cfg):
    """BASELINE configs 1-3 at full size (seed 1), spec generator, B from the counter stream."""
    _, rows, degree, dist, local, rhs = cfg
    host = spec_case(rows, degree, dist, local, 1)
    B = vb.fill_uniform(1, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    got = run_plan(cuda, host, B, rhs)
    ratio = assert_within_bound(host, B, rhs, got)
    assert ratio < 0.5, ratio  # comfortably inside the bound


GRID = [(rhs, dist, deg, local) for rhs in (8, 16, 32, 64) for dist in range(4)
        for deg in (1, 4, 8, 16) for local in (True, False)]


@pytest.mark.parametrize("k", range(0, 128, 1), ids=lambda k: "g%d" % k)
def test_regime_grid(cuda, k):
    """the 128-case 1024-row grid, seeds 1..128 in enumeration order."""
    rhs, dist, deg, local = GRID[k]
    host = spec_case(1024, deg, dist, local, k + 1)
    B = vb.fill_uniform(k + 1, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    got = run_plan(cuda, host, B, rhs)
    assert_within_bound(host, B, rhs, got)


@pytest.mark.parametrize("rhs", [8, 16, 32, 64])
def test_bounds_checked_build_and_no_split(cuda, rhs):
    host = spec_case(512, 16, 3, False, 77)
    B = vb.fill_uniform(77, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    a = run_plan(cuda, host, B, rhs)
    b = run_plan(cuda, host, B, rhs, flags=vb.PLAN_BOUNDS_CHECK)
    c = run_plan(cuda, host, B, rhs, flags=vb.PLAN_NO_SPLIT)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert_within_bound(host, B, rhs, c)


STACKS = [("raw", vb.PLAN_STACKS_RAW), ("presplit", vb.PLAN_STACKS_PRESPLIT),
          ("direct", vb.PLAN_B_DIRECT), ("direct_checked", vb.PLAN_B_DIRECT | vb.PLAN_BOUNDS_CHECK)]


@pytest.mark.parametrize("stacks", STACKS, ids=lambda s: s[0])
@pytest.mark.parametrize("case", [(1024, 16, 3, False, 1), (512, 4, 0, True, 9),
                                  (700, 8, 2, False, 4), (256, 1, 1, False, 13)],
                         ids=lambda c: "r%dd%d" % (c[0], c[1]))
def test_rhs64_stack_layouts(cuda, stacks, case):
    """RHS 64 with each operand-stack layout forced: raw-B stacks (lo rows formed in the kernel,
    three MMAs per group) from the pre-pass or read straight from B, and pre-split stacks (two
    MMAs per group). All meet the bound; the plan names the layout it uses."""
    rows, deg, dist, local, seed = case
    rhs = 64
    host = spec_case(rows, deg, dist, local, seed)
    B = vb.fill_uniform(seed, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs), stacks[1])
    assert ("raw-b" in p.describe()) == (stacks[0] == "raw")
    assert ("direct-b" in p.describe()) == stacks[0].startswith("direct")
    assert p.launch_count() == (1 if stacks[0].startswith("direct") else 2)
    got = run_plan(cuda, host, B, rhs, matrix=m, plan=p)
    assert_within_bound(host, B, rhs, got)
    # the bounds-checked build agrees bit for bit
    chk = run_plan(cuda, host, B, rhs, flags=stacks[1] | vb.PLAN_BOUNDS_CHECK)
    assert np.array_equal(got.view(np.uint32), chk.view(np.uint32))


FUSED_FORMS = [(8, 0), (16, 0), (32, 0), (64, vb.PLAN_STACKS_RAW), (64, vb.PLAN_STACKS_PRESPLIT),
               (32, vb.PLAN_CUDA_CORE_ROWS), (64, vb.PLAN_STACKS_RAW | vb.PLAN_BOUNDS_CHECK)]


@pytest.mark.parametrize("form", FUSED_FORMS, ids=lambda f: "r%d_%x" % f)
def test_fused_prepass(cuda, form):
    """VBSR_PLAN_FUSED_PREPASS: the SpMM's CTAs form the operand stacks themselves (one launch
    unless short rows run on the CUDA cores). C is bit-identical to the two-launch execute, also
    over repeated executes with changing B (the grid arrival word resets itself each launch)."""
    rhs, flags = form
    host = spec_case(700, 8, 3, False, 21)
    m = vb.Matrix(host)
    sep = vb.Plan(m, vb.PlanOptions(rhs), flags)
    fused = vb.Plan(m, vb.PlanOptions(rhs), flags | vb.PLAN_FUSED_PREPASS)
    assert fused.launch_count() == (2 if flags & vb.PLAN_CUDA_CORE_ROWS else 1)
    for it in range(3):
        B = vb.fill_uniform(21 + it, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
        a = run_plan(cuda, host, B, rhs, matrix=m, plan=sep)
        b = run_plan(cuda, host, B, rhs, matrix=m, plan=fused)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert_within_bound(host, B, rhs, b)


@pytest.mark.parametrize("flags", [0, vb.PLAN_FUSED_PREPASS], ids=["two_launches", "fused"])
@pytest.mark.parametrize("rhs", [16, 64])
def test_cuda_graph_capture(cuda, rhs, flags):
    """An execute captured into a CUDA graph and replayed with new B values in the same buffer
    gives, every replay, C bit-identical to an eager execute of that B (the capture records the
    pre-pass and SpMM launches with their programmatic dependency; the fused form's grid arrival
    word resets itself on every replay)."""
    torch = cuda
    host = spec_case(512, 8, 3, False, 5)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs), flags)
    eager = vb.Plan(m, vb.PlanOptions(rhs))
    dB = torch.zeros(host.scalar_cols() * rhs, device="cuda")
    dC = torch.full((host.scalar_rows() * rhs,), float("nan"), device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    p.execute(dB, dC, s)  # warm-up outside the capture
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        p.execute(dB, dC, s)
    for it in range(3):
        B = vb.fill_uniform(50 + it, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
        dB.copy_(torch.from_numpy(B))
        dC.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        p.check_status()
        ref = run_plan(cuda, host, B, rhs, matrix=m, plan=eager)
        assert np.array_equal(dC.cpu().numpy().view(np.uint32), ref.view(np.uint32)), it


def _handmade(heights, widths, rows_cols, seed=0):
    """A matrix from explicit per-row block column lists (possibly empty rows)."""
    rng = np.random.default_rng(seed)
    R, S = len(heights), len(widths)
    row_ptr, block_col, value_off = [0], [], [0]
    for i, cols in enumerate(rows_cols):
        for c in sorted(cols):
            block_col.append(c)
            value_off.append(value_off[-1] + heights[i] * widths[c])
        row_ptr.append(len(block_col))
    return vb.HostMatrix(R, S, row_ptr, block_col, heights, widths,
                         np.concatenate([[0], np.cumsum(heights)]),
                         np.concatenate([[0], np.cumsum(widths)]), value_off,
                         rng.uniform(-1, 1, value_off[-1]).astype(np.float32))


@pytest.mark.parametrize("rhs", [8, 16, 32, 64])
def test_edge_shapes(cuda, rhs):
    """Empty block rows (C must become exactly 0), one-block rows, extreme 8/64 blocks, a row
    with every column, and a matrix whose first and last rows are empty."""
    heights = [8, 64, 64, 8, 40, 64, 16]
    widths = [64, 8, 64, 8, 24, 56, 64, 8, 32]
    rows_cols = [[], [0], [2], list(range(9)), [], [1, 3, 7], []]
    host = _handmade(heights, widths, rows_cols, seed=rhs)
    host.validate()
    B = np.random.default_rng(1).uniform(-1, 1, host.scalar_cols() * rhs).astype(np.float32)
    got = run_plan(cuda, host, B, rhs)
    assert_within_bound(host, B, rhs, got)
    C = got.reshape(rhs, host.scalar_rows())
    for i in (0, 4, 6):
        r0, r1 = host.row_scalar_off[i], host.row_scalar_off[i + 1]
        assert np.all(C[:, r0:r1] == 0)


@pytest.mark.parametrize("rhs", [8, 16, 32, 64])
def test_heavy_rows(cuda, rhs):
    """A few very heavy block rows (64 blocks of 64 x 64) among many light ones: the planner cuts
    the heavy rows into row parts; with and without the cut C meets the bound, and the
    bounds-checked kernel on the cut schedule gives the same bits."""
    heights = [64] * 4 + [8] * 400
    widths = [64] * 64
    rows_cols = [list(range(64))] * 4 + [[i % 64] for i in range(400)]
    host = _handmade(heights, widths, rows_cols, seed=3)
    B = np.random.default_rng(2).uniform(-1, 1, host.scalar_cols() * rhs).astype(np.float32)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    assert "split_rows=4" in p.describe(), p.describe()
    got = run_plan(cuda, host, B, rhs, matrix=m, plan=p)
    assert_within_bound(host, B, rhs, got)
    q = vb.Plan(m, vb.PlanOptions(rhs), vb.PLAN_NO_SPLIT)
    assert "split_rows=0" in q.describe()
    whole = run_plan(cuda, host, B, rhs, matrix=m, plan=q)
    assert_within_bound(host, B, rhs, whole)
    chk = run_plan(cuda, host, B, rhs, flags=vb.PLAN_BOUNDS_CHECK, matrix=m)
    assert np.array_equal(chk.view(np.uint32), got.view(np.uint32))


def _power_law_case(light_rows, heavy_rows, heavy_degree, S, seed):
    """light_rows block rows of degree 8 and heavy_rows block rows of height 64 and degree
    heavy_degree (spread through the matrix), random distinct columns, high-variance sizes."""
    rng = np.random.default_rng(seed)
    sizes = np.array([8, 16, 56, 64])
    R = light_rows + heavy_rows
    heights = rng.choice(sizes, R, p=[.3, .2, .2, .3])
    heavy = np.linspace(R // (2 * heavy_rows), R - 1, heavy_rows).astype(int)
    heights[heavy] = 64
    widths = rng.choice(sizes, S, p=[.3, .2, .2, .3])
    rows_cols = []
    for i in range(R):
        d = heavy_degree if i in set(heavy.tolist()) else 8
        rows_cols.append(np.sort(rng.choice(S, d, replace=False)).tolist())
    return _handmade(heights.tolist(), widths.tolist(), rows_cols, seed=seed), heavy


def test_power_law_rows_split_and_balance(cuda):
    """Two block rows of degree 2048 among 16382 rows of degree 8 (RHS 8). Whole, each heavy row
    is several CTAs' fair share and sets the kernel's length; cut into row parts (each on its own
    CTA) the longest CTA is shorter. A part keeps all of the row's 8-column groups, so its
    pipeline-stage count does not shrink with its height: row parts bound the gain, which this
    test checks as a shorter longest CTA. Parity is checked for both schedules."""
    torch = cuda
    rhs = 8
    host, heavy = _power_law_case(16382, 2, 2048, 16384, seed=23)
    B = np.random.default_rng(4).uniform(-1, 1, host.scalar_cols() * rhs).astype(np.float32)
    m = vb.Matrix(host)
    spread = {}
    for name, flags in (("split", 0), ("whole", vb.PLAN_NO_SPLIT)):
        p = vb.Plan(m, vb.PlanOptions(rhs), flags)
        got = run_plan(cuda, host, B, rhs, matrix=m, plan=p)
        assert_within_bound(host, B, rhs, got)
        dB = torch.from_numpy(B).cuda()
        dC = torch.empty(host.scalar_rows() * rhs, device="cuda")
        for _ in range(3):
            p.execute(dB, dC)
        p.enable_cta_timing(True)
        p.execute(dB, dC)
        t = p.cta_timing().astype(np.int64)
        p.enable_cta_timing(False)
        dur = (t[:, 1] - t[:, 0]).astype(np.float64)
        spread[name] = (dur.max() / np.median(dur), dur.max(), p.describe())
    assert "split_rows=2" in spread["split"][2]
    # the cut shortens the longest CTA
    assert spread["split"][1] < 0.75 * spread["whole"][1], spread


def test_unaligned_and_offset_buffers(cuda):
    """B and C inside larger buffers at 16-byte and at 4-byte offsets."""
    torch = cuda
    host = spec_case(300, 8, 0, False, 5)
    rhs = 16
    B = vb.fill_uniform(5, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    for off in (4, 1):
        bigB = torch.zeros(B.size + 64, device="cuda")
        bigB[off:off + B.size] = torch.from_numpy(B).cuda()
        bigC = torch.full((host.scalar_rows() * rhs + 64,), 7.0, device="cuda")
        p.execute(bigB[off:].data_ptr(), bigC[off:].data_ptr())
        torch.cuda.synchronize()
        out = bigC.cpu().numpy()
        assert np.all(out[:off] == 7.0) and np.all(out[off + host.scalar_rows() * rhs:] == 7.0)
        assert_within_bound(host, B, rhs, out[off:off + host.scalar_rows() * rhs])


def test_deterministic_and_concurrent_streams(cuda):
    """Bitwise-identical results across runs, and two plans on two streams at once."""
    torch = cuda
    host = spec_case(2048, 8, 2, False, 11)
    rhs = 32
    B = torch.from_numpy(vb.fill_uniform(11, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)).cuda()
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = [torch.empty(host.scalar_rows() * rhs, device="cuda") for _ in range(4)]
    for i, o in enumerate(outs):
        p.execute(B, o, s1 if i % 2 == 0 else s2)
    torch.cuda.synchronize()
    ref = outs[0].cpu().numpy().view(np.uint32)
    for o in outs[1:]:
        assert np.array_equal(o.cpu().numpy().view(np.uint32), ref)


@pytest.mark.parametrize("rhs", [32, 64])
def test_one_plan_different_B_on_two_streams(cuda, rhs):
    """One const plan, two streams, a different B on each, issued back to back without host
    synchronisation (the reference allows concurrent execute calls on one Plan, plan.cpp:19-22).
    Both C match the oracle for their own B."""
    torch = cuda
    host = spec_case(2048, 8, 2, False, 17)
    K = host.scalar_cols()
    Bs = [vb.fill_uniform(100 + i, vb.STREAM_DENSE, 0, K * rhs) for i in range(2)]
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    dBs = [torch.from_numpy(b).cuda() for b in Bs]
    outs = [torch.full((host.scalar_rows() * rhs,), float("nan"), device="cuda") for _ in range(6)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    for i, o in enumerate(outs):
        p.execute(dBs[i % 2], o, streams[i % 2])
    torch.cuda.synchronize()
    p.check_status()
    for i, o in enumerate(outs):
        assert_within_bound(host, Bs[i % 2], rhs, o.cpu().numpy())


def test_one_plan_from_several_host_threads(cuda):
    """execute() from four host threads at once, each with its own stream, B and C."""
    import threading
    torch = cuda
    rhs = 16
    host = spec_case(1024, 8, 0, False, 19)
    K = host.scalar_cols()
    Bs = [vb.fill_uniform(200 + i, vb.STREAM_DENSE, 0, K * rhs) for i in range(4)]
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    dBs = [torch.from_numpy(b).cuda() for b in Bs]
    outs = [torch.full((host.scalar_rows() * rhs,), float("nan"), device="cuda") for _ in range(4)]
    streams = [torch.cuda.Stream() for _ in range(4)]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    errors = []

    def work(t):
        try:
            for _ in range(3):
                p.execute(dBs[t], outs[t], streams[t])
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=work, args=(t,)) for t in range(4)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    torch.cuda.synchronize()
    assert not errors
    p.check_status()
    for t in range(4):
        assert_within_bound(host, Bs[t], rhs, outs[t].cpu().numpy())


def test_stalled_pipeline_times_out_and_recovers(cuda):
    """The producer withholds one stage on purpose; every wait is bounded, so the kernel returns,
    the plan reports VBSR_TIMEOUT, and the same context keeps working afterwards."""
    torch = cuda
    host = spec_case(1024, 8, 2, False, 13)
    rhs = 32
    B = vb.fill_uniform(13, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    p.set_debug(drop_stage=3, wait_limit_cycles=2_000_000)  # ~1 ms per wait
    dB = torch.from_numpy(B).cuda()
    dC = torch.empty(host.scalar_rows() * rhs, device="cuda")
    p.execute(dB, dC)
    with pytest.raises(vb.TimeoutError_):
        p.check_status()
    p.set_debug(-1, 0)
    got = run_plan(cuda, host, B, rhs, matrix=m, plan=p)
    assert_within_bound(host, B, rhs, got)


def test_upload_across_slices_matches_device_generation(cuda):
    """A matrix of ~85 M values (more than one 64 M-value upload slice): built from host values
    through the pipelined upload + on-device relayout, it gives the same C, bit for bit, as the
    same matrix generated on the device, and that C meets the bound against the oracle."""
    torch = cuda
    rhs = 8
    host = spec_case(8192, 8, 2, False, 31)
    assert host.values.size > (1 << 26)
    B = vb.fill_uniform(31, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    up = run_plan(cuda, host, B, rhs)
    structure = spec_case(8192, 8, 2, False, 31, with_values=False)
    gen = vb.Matrix(structure, rows=(0, structure.block_rows), generated_seed=31)
    got = run_plan(cuda, host, B, rhs, matrix=gen)
    assert np.array_equal(up.view(np.uint32), got.view(np.uint32))
    assert_within_bound(host, B, rhs, up)


CC_CASES = [(1024, 8, 2, False, 41), (777, 16, 0, True, 42), (512, 4, 3, False, 43),
            (300, 1, 2, True, 44), (256, 16, 3, True, 45)]


@pytest.mark.parametrize("rhs", [8, 16, 32])
@pytest.mark.parametrize("case", CC_CASES, ids=lambda c: "r%dd%d" % (c[0], c[1]))
def test_cuda_core_rows(cuda, rhs, case):
    """Short block rows (h 8 and 16) on the CUDA-core path of the pre-pass launch, the other rows on
    the tensor cores: the result meets the bound, as does the all-tensor-core plan, and the work
    split covers every row and value."""
    rows, deg, dist, local, seed = case
    host = spec_case(rows, deg, dist, local, seed)
    B = vb.fill_uniform(seed, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs), vb.PLAN_CUDA_CORE_ROWS)
    w = p.work_info()
    short = int(np.count_nonzero(host.row_size <= 16))  # every short row here is light
    assert w["cc_rows"] == short
    assert w["cc_rows"] + w["tc_rows"] == host.block_rows
    assert w["cc_values"] + w["tc_values"] == host.values.size
    assert_within_bound(host, B, rhs, run_plan(cuda, host, B, rhs, matrix=m, plan=p))
    q = vb.Plan(m, vb.PlanOptions(rhs))  # default: every row on the tensor cores
    assert q.work_info()["cc_rows"] == 0
    assert_within_bound(host, B, rhs, run_plan(cuda, host, B, rhs, matrix=m, plan=q))


@pytest.mark.parametrize("rhs", [8, 32])
def test_all_rows_on_cuda_cores(cuda, rhs):
    """A matrix whose block rows are all short (and one empty): no tensor-core CTA is launched,
    every row is computed by the pre-pass launch, and C is complete (the empty row exactly 0)."""
    heights = [8, 16, 8, 16, 8] * 20 + [8]
    widths = [8, 16, 24, 32, 40, 48, 56, 64] * 4
    rng = np.random.default_rng(5)
    rows_cols = [sorted(rng.choice(32, 4, replace=False).tolist()) for _ in range(100)] + [[]]
    host = _handmade(heights, widths, rows_cols, seed=rhs)
    B = np.random.default_rng(6).uniform(-1, 1, host.scalar_cols() * rhs).astype(np.float32)
    m = vb.Matrix(host)
    p = vb.Plan(m, vb.PlanOptions(rhs), vb.PLAN_CUDA_CORE_ROWS)
    assert p.work_info()["cc_rows"] == host.block_rows
    assert p.num_tasks() == 0
    got = run_plan(cuda, host, B, rhs, matrix=m, plan=p)
    assert_within_bound(host, B, rhs, got)
    C = got.reshape(rhs, host.scalar_rows())
    assert np.all(C[:, host.row_scalar_off[100]:] == 0)


@pytest.mark.parametrize("rhs", [8, 32, 64])
def test_matrix_market_through_the_engine(cuda, rhs, tmp_path):
    """A scalar sparse matrix from a Matrix Market file, cut into 32 x 24 blocks (padded to
    multiples of 8), saved to and reloaded from a VBSR file, multiplied on the GPU: C meets the
    bound against the oracle, and its top-left block is the dense product of the file's matrix."""
    import scipy.io
    import scipy.sparse as sp
    a = sp.random(1003, 870, density=0.01, random_state=rhs, format="coo", dtype=np.float32)
    mtx = str(tmp_path / "a.mtx")
    scipy.io.mmwrite(mtx, a)
    m0, (rows, cols) = vb.load_matrix_market(mtx, row_block=32, col_block=24)
    m0.save(str(tmp_path / "a.vbsr"))
    host = vb.load_matrix(str(tmp_path / "a.vbsr"))
    B = np.random.default_rng(rhs).uniform(-1, 1, host.scalar_cols() * rhs).astype(np.float32)
    got = run_plan(cuda, host, B, rhs)
    assert_within_bound(host, B, rhs, got)
    Cm = got.reshape(rhs, host.scalar_rows()).T[:rows]
    ref = a.toarray().astype(np.float64) @ B.reshape(rhs, host.scalar_cols()).T[:cols]
    assert np.allclose(Cm, ref, rtol=0, atol=1e-4)
