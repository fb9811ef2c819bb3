"""bench.py — VBSR SpMM benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload large|headline|wide|small|large16k]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1, NCCL)
    python bench.py --impl reference ...                  (the reference's CPU path, rank 0 only;
                                                           loads the oracle library only)

Workload (default `large`): 262144 x 262144 block rows/columns, high-variance
block sizes {8,16,56,64} w.p. {.3,.2,.2,.3}, degree 16, random pattern, RHS 64, seed 1 (~22 GB of
A). Block rows are partitioned over the ranks by balanced cost (vbsr_partition_rows); each rank
builds its shard on its GPU (values generated on the device by the engine's counter-based
generator, identical to the host generator), receives its replica of B from rank 0 by peer copies
over NVLink between CUDA-IPC-mapped buffers (setup, timed as `replicate`; no NCCL) and runs
Plan.execute on its shard. No collective runs inside the timed region. After it, every block row of
every shard is checked against the oracle on its own rank.

Metric: effective HBM GB/s = compulsory bytes of the whole problem (reference VBSR format:
A values + indices + B + C) / device time per step, max over ranks. One JSON line on rank 0, with
the median/p95 step time, the roofline of the SpMM kernel, the end-to-end figure through the public
API with host buffers, the CPU baseline (N=1), clocks sampled during the timed region and, at N=1,
the headline workload measured in the same process.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (block_rows, degree, distribution, local, rhs, description)
    "large": (262144, 16, 2, False, 64,
              "BASELINE config 5: 262144 block rows/cols, high-variance {8,16,56,64}, degree 16, "
              "random, RHS 64, seed 1"),
    "headline": (4096, 8, 2, False, 32,
                 "BASELINE config 3 (headline): 4096 block rows/cols, high-variance {8,16,56,64}, "
                 "degree 8, random, RHS 32, seed 1"),
    "wide": (1024, 16, 3, False, 64,
             "BASELINE config 2: 1024 block rows/cols, bimodal 8/64, degree 16, random, RHS 64, "
             "seed 1"),
    "large16k": (16384, 16, 2, False, 64,
                 "profiling case: BASELINE config 5's generator settings (high-variance, degree 16, "
                 "random, RHS 64, seed 1) at 16384 block rows, A 1.4 GB, B 151 MB (above L2)"),
    "small": (256, 4, 0, True, 8,
              "BASELINE config 1: 256 block rows/cols, uniform {8..64}, degree 4, local, RHS 8, "
              "seed 1"),
}
SEED = 1
L2_BYTES = 126 * 1024 * 1024


def measured_hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_from_profiles(workload: str):
    """DRAM bytes per launch of the SpMM kernel from a committed ncu summary (or None)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            d = json.load(f)
        return d.get(workload, {}).get("dram_bytes_per_launch")
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clock/throttle samples every 20 ms while the timed region runs (the multi-GPU
    steps are a few ms each, so a 200 ms period could miss a short region). Entering waits for the
    sampler's first line, so the samples that count start before the timed work."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.QUERY,
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t = time.time()
            while not self.lines and time.time() - t < 3.0:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        self.first = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[max(0, getattr(self, "first", 1) - 1):]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def rank_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def make_structure(workload):
    import varblockspmm_b200 as vb
    rows, degree, dist, local, rhs, _ = WORKLOADS[workload]
    host = vb.generate(vb.GeneratorOptions(rows, rows, degree, rhs, vb.Distribution(dist), local,
                                           SEED, vb.Profile.Spec), with_values=False)
    return host, rhs


def make_workload(workload):
    """The workload's structure built by the oracle library alone (no engine library); its values
    are regenerated per row slice."""
    import oracle
    rows, degree, dist, local, rhs, _ = WORKLOADS[workload]
    return oracle.WorkloadMatrix(rows, rows, degree, dist, local, SEED), rhs


def problem_bytes(host, rhs, r0=0, r1=None):
    """Compulsory bytes of block rows [r0, r1) in the reference VBSR format (values, block_col,
    value_off, row_ptr, row_size, row_scalar_off, col_size, col_scalar_off, B, C) and the useful
    flops 2 * sum(h*w) * rhs; the same formula as vbsr_compulsory_bytes."""
    r1 = host.block_rows if r1 is None else r1
    b0, b1 = int(host.row_ptr[r0]), int(host.row_ptr[r1])
    hw = float(host.value_off[b1] - host.value_off[b0])
    nnzb, R, S = float(b1 - b0), float(r1 - r0), float(host.block_cols)
    M = float(host.row_scalar_off[r1] - host.row_scalar_off[r0])
    K = float(host.col_scalar_off[-1])
    return (4 * hw + 4 * nnzb + 8 * (nnzb + 1) + 4 * (R + 1) + 4 * R + 8 * (R + 1) + 4 * S
            + 8 * (S + 1) + 4 * K * rhs + 4 * M * rhs), 2 * hw * rhs


def flush_l2(rank_bytes):
    """Whether the timed steps flush L2 between launches (a rank's inputs smaller than 2 x L2)."""
    return rank_bytes < 2 * L2_BYTES


def workload_config(workload, host, rhs, pbytes, flops, gpus, rank_bytes):
    """The `config` object of both arms' JSON lines (identical for the same workload and N)."""
    return {"workload": WORKLOADS[workload][5], "block_rows": host.block_rows, "nnzb": host.nnzb,
            "rhs": rhs, "compulsory_bytes": pbytes, "useful_flops": flops,
            "parallelism": f"block-row partition over {gpus} GPU(s), B replicated",
            "l2": "L2 flushed before every launch" if flush_l2(rank_bytes)
                  else "inputs larger than L2 (no flush)"}


# ---- CPU reference path -----------------------------------------------------------------------

class _PortRunner:
    """The oracle's C restatement (bit-identical to the reference's cpu_reference), timed the way
    oracle.RefTimer times the reference itself: run() returns the computation's seconds."""

    def __init__(self, host, B, rhs, threads):
        self.host, self.B, self.rhs, self.threads = host, B, rhs, threads

    def run(self, C_out=None):
        import oracle
        t = time.perf_counter()
        oracle.spmm(self.host, self.B, self.rhs, threads=self.threads)
        return time.perf_counter() - t

    def close(self):
        pass


def cpu_reference_timing(host, rhs, B, warmup, repeats, min_frac=0.05, min_run_s=1.0):
    """The reference's own cpu_reference (oracle/_ref, compiled unchanged from the reference
    sources; the oracle's restatement when that is absent) on all host threads, on block rows
    [0, r) of the workload: at least `min_frac` of its flops and at least `min_run_s` per run. The
    sample's inputs (values, the per-thread row-slice HostMatrix parts and the std::vector copy of
    B the reference API takes) are built before timing; each timed run is only the cpu_reference
    calls. Returns (median seconds per sample, sample flops, details)."""
    import oracle
    threads = oracle.host_threads()
    use_ref = oracle.ref_available()
    rows = host.block_rows
    total = host.flops(rhs)

    def runner_for(r):
        sub = host.row_slice(0, r)
        return (oracle.RefTimer(sub, B, rhs, threads) if use_ref
                else _PortRunner(sub, B, rhs, threads))

    r = min(rows, max(threads, int(np.ceil(min_frac * rows))))
    while host.flops(rhs, 0, r) < min_frac * total and r < rows:
        r = min(rows, r + max(1, rows // 100))
    runner = runner_for(r)
    dt = runner.run()
    if dt < min_run_s and r < rows:
        r = min(rows, int(np.ceil(r * min_run_s / max(dt, 1e-6) * 1.1)))
        runner.close()
        runner = runner_for(r)
    for _ in range(warmup):
        runner.run()
    times = [runner.run() for _ in range(max(1, repeats))]
    runner.close()
    flops = host.flops(rhs, 0, r)
    med = statistics.median(times)
    return med, flops, {
        "kind": "reference" if use_ref else "port", "cores": threads, "rows": r,
        "flops_frac": flops / total, "runs": len(times), "run_s": times}


def run_reference_arm(args):
    """--impl reference: the reference's own cpu_reference (oracle/_ref, compiled unchanged from
    the reference sources) or, if that library is absent, the bit-identical C restatement, with all
    host threads, on samples of the same workload (every step one timed sample run, at least 5% of
    the workload's flops), extrapolated to the whole workload by flops. Rank 0 only. The inputs come
    from the oracle library's own generator: nothing of the engine is loaded in this arm."""
    rank, world, _ = rank_env()
    if rank != 0:
        return 0
    import oracle
    host, rhs = make_workload(args.workload)
    pbytes, total_flops = problem_bytes(host, rhs)
    B = oracle.fill_uniform(SEED, oracle.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    per_step = max(0.5, min(3.0, 75.0 / max(1, args.steps + args.warmup)))
    med, flops, info = cpu_reference_timing(host, rhs, B, args.warmup, args.steps,
                                            min_run_s=per_step)
    est_full_s = med * total_flops / flops
    value = pbytes / est_full_s / 1e9
    sample = (f"block rows [0,{info['rows']}) of the workload ({100 * info['flops_frac']:.1f}% of "
              f"its flops) per step, median of {info['runs']} timed runs {med:.3f} s on "
              f"{info['cores']} threads (cpu_reference calls only; inputs prepared before "
              f"timing), extrapolated to the whole workload by flops")
    # a step is one timed sample run; value is the sample's throughput (its share of the
    # workload's compulsory bytes, by flops, per second)
    line = {
        "metric": "spmm_effective_hbm_GBps", "impl": "reference", "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": med * 1e3, "full_workload_ms_extrapolated": est_full_s * 1e3,
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator)",
        "config": workload_config(args.workload, host, rhs, pbytes, total_flops, args.gpus,
                                  pbytes / max(1, args.gpus)),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": info["cores"],
                         "kind": info["kind"], "sample": sample,
                         "sample_seconds_median": med,
                         "sample_seconds_min": min(info["run_s"]),
                         "sample_seconds_max": max(info["run_s"])},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- GPU arm --------------------------------------------------------------------------------------

def full_parity(work, rhs, r0, r1, C_host, B_host, threads, slice_rows=4096):
    """Every block row of [r0, r1) against the oracle, after the timed region: the rows' values are
    regenerated by the oracle library's own generator slice by slice (host memory stays bounded)
    and each slice of C is compared under |C - C_ref| <= 1e-5 * sum|a||b| with all `threads`.
    C_host is the rank's C block, column-major with ld = its scalar row count."""
    import oracle
    t0 = time.perf_counter()
    off = work.row_scalar_off
    M_r = int(off[r1] - off[r0])
    Cv = np.asarray(C_host)[:M_r * rhs].reshape(rhs, M_r)
    worst, bad = 0.0, 0
    for a in range(r0, r1, slice_rows):
        b = min(r1, a + slice_rows)
        sub = work.row_slice(a, b)
        c0, c1 = int(off[a] - off[r0]), int(off[b] - off[r0])
        got = np.ascontiguousarray(Cv[:, c0:c1]).reshape(-1)
        ratio, _, nb = oracle.compare(sub, B_host, rhs, got, threads=threads)
        worst, bad = max(worst, ratio), bad + int(nb)
    return {"rows_checked": r1 - r0, "max_err_over_bound": worst, "violations": bad,
            "seconds": time.perf_counter() - t0, "threads": threads}


def gathered_parity(host, rhs, bounds, rank, world, dC, B_host, per_shard=4):
    """Verification only, outside the timed region: every rank's C block goes to rank 0 over NCCL
    (point-to-point sends acting as an allgatherv), rank 0 reassembles the column-major M x N
    result on the host, and checks block rows of every shard (its first and last rows and a few
    in between) against the oracle. Returns None on ranks > 0."""
    import oracle
    import torch
    import torch.distributed as dist
    M = int(host.scalar_rows())
    t0 = time.perf_counter()
    if rank != 0:
        dist.send(dC, dst=0)
        return None
    full = np.empty((rhs, M), dtype=np.float32)  # column-major M x rhs: row c holds column c
    for r in range(world):
        a, b = int(bounds[r]), int(bounds[r + 1])
        c0, c1 = int(host.row_scalar_off[a]), int(host.row_scalar_off[b])
        if r == 0:
            blk = dC
        else:
            blk = torch.empty(max(1, (c1 - c0) * rhs), device=dC.device)
            dist.recv(blk, src=r)
        if c1 > c0:
            full[:, c0:c1] = blk[:(c1 - c0) * rhs].view(rhs, c1 - c0).cpu().numpy()
    gather_ms = (time.perf_counter() - t0) * 1e3
    rng = np.random.default_rng(4321)
    worst, bad, rows = 0.0, 0, 0
    for r in range(world):
        a, b = int(bounds[r]), int(bounds[r + 1])
        if b <= a:
            continue
        picks = sorted(set([a, b - 1] + list(rng.integers(a, b, per_shard))))
        for i in picks:
            sub = host.row_slice(i, i + 1, values_seed=SEED)
            g0 = int(host.row_scalar_off[i])
            got = full[:, g0:g0 + int(host.row_size[i])].reshape(-1).copy()
            ratio, _, nb = oracle.compare(sub, B_host, rhs, got, threads=1)
            worst, bad, rows = max(worst, ratio), bad + nb, rows + 1
    return {"rows_checked": rows, "max_err_over_bound": worst, "violations": bad,
            "gather_ms": gather_ms,
            "how": "NCCL send/recv of every rank's C block to rank 0, host reassembly of the "
                   "M x N column-major result, oracle check of rows of every shard"}


def cta_time_stats(plan, B, C, stream):
    """One extra execution with per-CTA timing: spread of CTA durations (load-balance check)."""
    plan.enable_cta_timing(True)
    plan.execute(B, C, stream)
    t = plan.cta_timing(stream).astype(np.int64)
    plan.enable_cta_timing(False)
    dur = (t[:, 1] - t[:, 0]) / 1e3
    tw, cost = plan.task_stats()
    by_team = {}
    for w in sorted(set(tw.tolist())):
        d = dur[tw == w]
        by_team[f"team_warps_{w}"] = {"ctas": int(d.size), "median_us": float(np.median(d)),
                                      "max_us": float(d.max()),
                                      "us_per_model_unit": float(np.median(d / cost[tw == w]))}
    return {"ctas": int(t.shape[0]), "min_us": float(dur.min()), "median_us": float(np.median(dur)),
            "max_us": float(dur.max()), "span_us": float((t[:, 1].max() - t[:, 0].min()) / 1e3),
            "by_team_size": by_team}


def fp32_fma_tflops(torch, sm_max_mhz=None):
    """CUDA-core fp32 peak of one GPU: SMs x 128 FMA lanes x 2 flops x the maximum SM clock
    (nvidia-smi clocks.max.sm, else 1965 MHz)."""
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return sms * 128 * 2 * float(sm_max_mhz or 1965.0) * 1e6 / 1e12


def time_headline(vb, torch, stream, peak, steps=200, warmup=10):
    """BASELINE config 3 on this GPU: per-launch device time with L2 flushed between launches,
    every block row checked against the oracle afterwards."""
    import oracle
    host, rhs = make_structure("headline")
    work, _ = make_workload("headline")
    pbytes, flops = vb.compulsory_bytes(host, rhs)
    m = vb.Matrix(host, rows=(0, host.block_rows), generated_seed=SEED)
    p = vb.Plan(m, vb.PlanOptions(rhs))
    B = torch.empty(host.scalar_cols() * rhs, device="cuda")
    vb.fill_uniform_device(SEED, vb.STREAM_DENSE, 0, B.numel(), B, stream)
    Cd = torch.empty(host.scalar_rows() * rhs, device="cuda")
    flush = torch.empty(2 * L2_BYTES // 4, device="cuda")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            p.execute(B, Cd, stream)
        for i in range(steps):
            flush.fill_(float(i))
            ev[i][0].record(stream)
            p.execute(B, Cd, stream)
            ev[i][1].record(stream)
    stream.synchronize()
    p.check_status(stream)
    ts = sorted(a.elapsed_time(b) for a, b in ev)
    med = ts[len(ts) // 2]
    p95 = ts[min(len(ts) - 1, int(len(ts) * 0.95))]
    # the same executes back to back without the flush (B, its stacks and C stay in L2)
    with torch.cuda.stream(stream):
        for i in range(steps):
            ev[i][0].record(stream)
            p.execute(B, Cd, stream)
            ev[i][1].record(stream)
    stream.synchronize()
    uts = sorted(a.elapsed_time(b) for a, b in ev)
    umed = uts[len(uts) // 2]
    B_host = oracle.fill_uniform(SEED, oracle.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    parity = full_parity(work, rhs, 0, host.block_rows, Cd.cpu().numpy(), B_host,
                         oracle.host_threads())
    gbs = pbytes / (med * 1e-3) / 1e9
    # the tensor-core kernel alone (a plan that skips the pre-pass launch; timing only)
    kp = vb.Plan(m, vb.PlanOptions(rhs), vb.PLAN_DIAG_SKIP_PREPASS)
    kC = torch.empty_like(Cd)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            kp.execute(B, kC, stream)
        for i in range(steps):
            flush.fill_(float(i))
            kev[i][0].record(stream)
            kp.execute(B, kC, stream)
            kev[i][1].record(stream)
    stream.synchronize()
    kts = sorted(a.elapsed_time(b) for a, b in kev)
    kmed = kts[len(kts) // 2]
    work = p.work_info()
    kbytes = pbytes - 4.0 * work["cc_values"] - 4.0 * work["cc_scalar_rows"] * rhs
    return {"workload": WORKLOADS["headline"][5], "median_ms": med, "p95_ms": p95,
            "tc_kernel_median_ms": kmed, "tc_kernel_bytes": kbytes,
            "tc_kernel_frac_of_measured_hbm": kbytes / (kmed * 1e-3) / 1e9 / peak, "work": work,
            "GBps": gbs, "frac_of_measured_hbm": gbs / peak, "compulsory_bytes": pbytes,
            "useful_TFLOPs": flops / (med * 1e-3) / 1e12,
            "useful_frac_of_fp32_fma_peak": flops / (med * 1e-3) / 1e12 / fp32_fma_tflops(torch),
            "l2": "flushed before every launch", "median_ms_unflushed": umed,
            "plan": p.describe(), "parity": parity,
            "cta_time": cta_time_stats(p, B, Cd, stream)}


def run_gpu_arm(args):
    import torch
    import torch.distributed as dist
    import oracle
    import varblockspmm_b200 as vb
    from varblockspmm_b200.replica import PeerReplica, copy_async

    rank, world, local = rank_env()
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    if world != args.gpus:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local)
    hostgrp = None
    if world > 1:
        # NCCL only for the max-over-ranks reductions and the verification gather of C; the
        # data path (B replication) is peer copies ordered by barriers on a gloo group
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        hostgrp = dist.new_group(backend="gloo")
    stream = torch.cuda.Stream()
    peak, peak_kind = measured_hbm_peak()

    host, rhs = make_structure(args.workload)
    work, _ = make_workload(args.workload)
    assert np.array_equal(work.block_col, host.block_col) and \
        np.array_equal(work.value_off, host.value_off), "oracle and engine structures differ"
    pbytes, total_flops = vb.compulsory_bytes(host, rhs)
    bounds = vb.partition_rows(host, world, rhs)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    rank_bytes, rank_flops = vb.compulsory_bytes(host, rhs, r0, r1)
    M_r = int(host.row_scalar_off[r1] - host.row_scalar_off[r0])
    K = host.scalar_cols()
    nB = K * rhs

    def barrier():
        if world > 1:
            dist.barrier(group=hostgrp)
        torch.cuda.synchronize()

    def max_over_ranks(*vals):
        t = torch.tensor(list(vals), dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    t_setup = time.perf_counter()
    m = vb.Matrix(host, device=local, rows=(r0, r1), generated_seed=SEED)
    plan = vb.Plan(m, vb.PlanOptions(rhs))
    # two B buffers and two C buffers: buffer 0 for the device-timed steps, both for the pipelined
    # end-to-end steps
    rep = None
    if world > 1:
        rep = PeerReplica(nB, rank, world, local, hostgrp, buffers=2)
        bptr = [rep.ptr(0), rep.ptr(1)]
    else:
        dBs = [torch.empty(nB, device="cuda") for _ in range(2)]
        bptr = [t.data_ptr() for t in dBs]
    torch.cuda.synchronize()
    replicate = None
    if rank == 0:
        vb.fill_uniform_device(SEED, vb.STREAM_DENSE, 0, nB, bptr[0], stream)
        stream.synchronize()
    if world > 1:
        barrier()
        t_rep0 = time.perf_counter()
        got = rep.replicate_from(0, 0, stream)
        rep_ms = (time.perf_counter() - t_rep0) * 1e3
        rep_ms_max, = max_over_ranks(rep_ms)
        replicate = {"ms": rep_ms_max, "bytes_per_rank": 4 * nB,
                     "GBps_per_rank": 4 * nB / (rep_ms_max * 1e-3) / 1e9,
                     "how": "peer copies over NVLink between CUDA-IPC-mapped replicas (scatter "
                            "from rank 0, then every chunk from its owner), host barriers on a "
                            "gloo group; no NCCL; host-timed including two barriers"}
    dC = torch.empty(max(1, M_r * rhs), device="cuda")
    setup_s = time.perf_counter() - t_setup

    flush = None
    if flush_l2(rank_bytes):
        flush = torch.empty(2 * L2_BYTES // 4, device="cuda")

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            plan.execute(bptr[0], dC, stream)
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        with torch.cuda.stream(stream):
            t0.record(stream)
            for i in range(args.steps):
                if flush is not None:
                    flush.fill_(float(i))
                evs[i][0].record(stream)
                plan.execute(bptr[0], dC, stream)
                evs[i][1].record(stream)
            t1.record(stream)
        barrier()
    total_ms = t0.elapsed_time(t1)
    launch_ms = sorted(a.elapsed_time(b) for a, b in evs)
    med = launch_ms[len(launch_ms) // 2]
    p95 = launch_ms[min(len(launch_ms) - 1, int(len(launch_ms) * 0.95))]
    mean_launch = sum(launch_ms) / len(launch_ms)
    plan.check_status(stream)
    total_ms, med_max, p95_max = max_over_ranks(total_ms, med, p95)
    ms_per_step = total_ms / args.steps if flush is None else med_max

    cta_stats = cta_time_stats(plan, bptr[0], dC, stream)

    # ---- the SpMM kernel alone (roofline): a second plan that skips the B pre-pass ---------------
    kplan = vb.Plan(m, vb.PlanOptions(rhs), vb.PLAN_DIAG_SKIP_PREPASS)
    kC = torch.empty_like(dC)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            kplan.execute(bptr[0], kC, stream)
        for i in range(args.steps):
            if flush is not None:
                flush.fill_(float(i))
            kev[i][0].record(stream)
            kplan.execute(bptr[0], kC, stream)
            kev[i][1].record(stream)
    stream.synchronize()
    kernel_ms, = max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / args.steps)
    del kplan, kC

    # ---- end to end through the public API with host buffers ---------------------------------
    # Every step brings B from pinned host memory, executes, and brings this rank's C block back
    # to pinned host memory. At N = 1 the whole of B crosses PCIe; at N > 1 each rank uploads only
    # its own 1/N chunk of B and takes the other chunks from its peers over NVLink (peer copies,
    # ordered by a host barrier), so PCIe traffic per rank shrinks with N. Steps are pipelined:
    # B and C are double-buffered, uploads and downloads run on their own copy streams, and step
    # i+1's upload overlaps step i's execute and download. The timed region spans the first
    # upload to the last download on the device, max over ranks.
    B_host = oracle.fill_uniform(SEED, oracle.STREAM_DENSE, 0, nB)
    hB = torch.from_numpy(B_host).pin_memory()
    hC = [torch.empty(max(1, M_r * rhs), dtype=torch.float32).pin_memory() for _ in range(2)]
    dC2 = [dC, torch.empty_like(dC)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    e2e_steps = max(2, min(args.steps, 24))  # pipeline fill and drain amortised over the steps
    ev_up, ev_pull, ev_run, ev_down = ([torch.cuda.Event() for _ in range(e2e_steps)]
                                       for _ in range(4))
    h2d = d2h = nvl = 0
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(e2e_steps):
        b = i % 2
        if i >= 2:
            s_in.wait_event(ev_run[i - 2])  # the execute that read B buffer b is done
        if world > 1:
            h2d += rep.upload_own_chunk(hB.data_ptr(), b, s_in)
            ev_up[i].record(s_in)
            ev_up[i].synchronize()
            if i >= 1:
                ev_pull[i - 1].synchronize()  # this rank's pulls of step i-1 are done
            dist.barrier(group=hostgrp)  # every chunk of step i is in its owner's buffer
            nvl += rep.pull_peers(b, s_in)
        else:
            copy_async(bptr[b], hB.data_ptr(), 4 * nB, s_in)
            h2d += 4 * nB
        ev_pull[i].record(s_in)
        stream.wait_event(ev_pull[i])
        if i >= 2:
            stream.wait_event(ev_down[i - 2])  # C buffer b of step i-2 is downloaded
        plan.execute(bptr[b], dC2[b], stream)
        ev_run[i].record(stream)
        s_out.wait_event(ev_run[i])
        with torch.cuda.stream(s_out):
            hC[b].copy_(dC2[b], non_blocking=True)
        d2h += 4 * M_r * rhs
        ev_down[i].record(s_out)
    e1.record(s_out)
    e1.synchronize()
    torch.cuda.synchronize()
    e2e_ms, = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    if world > 1:
        barrier()
    plan.check_status(stream)

    # ---- parity: every block row of this rank's shard against the oracle ------------------------
    threads = max(1, oracle.host_threads() // max(1, local_world))
    parity = full_parity(work, rhs, r0, r1, dC.cpu().numpy(), B_host, threads)
    pr = torch.tensor([parity["max_err_over_bound"], parity["violations"],
                       parity["rows_checked"], parity["seconds"]], dtype=torch.float64,
                      device="cuda")
    gathered = None
    if world > 1:
        pr_max = pr.clone()
        dist.all_reduce(pr_max, op=dist.ReduceOp.MAX)
        dist.all_reduce(pr, op=dist.ReduceOp.SUM)
        pr[0], pr[3] = pr_max[0], pr_max[3]
        gathered = gathered_parity(host, rhs, bounds, rank, world, dC, B_host)
    parity = {"rows_checked": int(pr[2].item()), "block_rows": host.block_rows,
              "max_err_over_bound": pr[0].item(), "violations": int(pr[1].item()),
              "seconds": pr[3].item(),
              "how": "after the timed region, every block row of every rank's shard checked on "
                     "its own rank against the oracle (values regenerated by the oracle library "
                     "slice by slice), |C - C_ref| <= 1e-5 * sum|a||b| per element"}

    upload = None
    if args.host_upload:
        # Matrix construction from host values, the path a user with a host matrix takes
        t_g = time.perf_counter()
        hv = host.row_slice(r0, r1, values_seed=SEED)
        gen_s = time.perf_counter() - t_g
        torch.cuda.synchronize()
        t_u = time.perf_counter()
        mu = vb.Matrix(hv, device=local)
        up_s = time.perf_counter() - t_u
        upload = {"host_values_bytes": 4 * int(hv.values.size), "host_generate_s": gen_s,
                  "matrix_create_s": up_s,
                  "GBps": 4 * hv.values.size / up_s / 1e9,
                  "how": "vb.Matrix(host rows with values): pinned staging slices, H2D copy and "
                         "on-device relayout pipelined on private streams"}
        del mu, hv

    headline = None
    cpu = None
    if world == 1:
        if args.workload != "headline":
            headline = time_headline(vb, torch, stream, peak)
        if not args.no_cpu_baseline:
            med_s, flops_s, info = cpu_reference_timing(work, rhs, B_host, 1, 3, min_run_s=2.0)
            est_full = med_s * total_flops / flops_s
            cpu = {"value": pbytes / est_full / 1e9, "unit": "GB/s", "cores": info["cores"],
                   "kind": info["kind"],
                   "sample": f"block rows [0,{info['rows']}) of the workload "
                             f"({100 * info['flops_frac']:.1f}% of its flops), median of "
                             f"{info['runs']} timed runs {med_s:.2f} s on {info['cores']} threads "
                             f"(cpu_reference calls only), extrapolated by flops",
                   "sample_seconds_median": med_s}
    if rep is not None:
        rep.close()

    # the tensor-core kernel's own algorithmic bytes: the rank's compulsory bytes less the A values
    # and C rows of the short block rows the pre-pass launch computes on the CUDA cores
    work = plan.work_info()
    kernel_bytes = rank_bytes - 4.0 * work["cc_values"] - 4.0 * work["cc_scalar_rows"] * rhs
    if rank == 0:
        value = pbytes / (ms_per_step * 1e-3) / 1e9
        achieved = kernel_bytes / (kernel_ms * 1e-3) / 1e9
        traffic = traffic_from_profiles(args.workload) if world == 1 else None
        line = {
            "metric": "spmm_effective_hbm_GBps", "value": value, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "median_ms": med_max, "p95_ms": p95_max,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded spec generator; A values generated on device, bit-identical "
                    "to the host generator)",
            "config": workload_config(args.workload, host, rhs, pbytes, total_flops, world,
                                      rank_bytes),
            "plan": plan.describe(),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": kernel_bytes,
                         "kernel": "vbsr_b200::spmm_tc_kernel", "kernel_ms": kernel_ms,
                         "execute_ms": mean_launch,
                         "execute_frac": rank_bytes / (mean_launch * 1e-3) / 1e9 / peak,
                         "work": work,
                         "note": "achieved = the tensor-core kernel's compulsory bytes (the rank's, "
                                 "less the A values and C rows of the short rows computed on the "
                                 "CUDA cores in the pre-pass launch) / mean duration of that kernel "
                                 "alone (events around executes of a plan that skips the pre-pass "
                                 "launch); execute_frac = the rank's compulsory bytes / the whole "
                                 "execute (both launches)"},
            "useful_TFLOPs": total_flops / (ms_per_step * 1e-3) / 1e12,
            "useful_frac_of_fp32_fma_peak": total_flops / (ms_per_step * 1e-3) / 1e12 /
                (world * fp32_fma_tflops(torch, clocks.summary().get("sm_max_mhz"))),
            "e2e": {"value": pbytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d // e2e_steps,
                    "d2h_bytes_per_step": d2h // e2e_steps,
                    "nvlink_bytes_per_step": nvl // e2e_steps, "steps": e2e_steps,
                    "bytes_are": "per rank (rank 0)",
                    "path": "pinned host B -> device (at N>1 the rank's own 1/N chunk; the other "
                            "chunks by peer copies from the ranks that uploaded them), "
                            "Plan.execute (C ABI), device C block -> pinned host, every step; "
                            "steps pipelined (double-buffered B and C, separate copy streams)"},
            "gpu_launches": args.steps * plan.launch_count(),
            "clocks": clocks.summary(),
            "parity": parity,
            "setup_s": setup_s, "cta_time": cta_stats,
        }
        if replicate:
            line["replicate"] = replicate
        if upload:
            line["matrix_upload"] = upload
        if gathered:
            line["gathered_parity"] = gathered
        if headline:
            line["headline"] = headline
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="large")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--host-upload", action="store_true",
                    help="also time building the rank's Matrix from host values (generated on the "
                         "host, then uploaded and re-laid-out on the device)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
