"""bench.py — VBSR SpMM benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload large|headline|wide|small|large16k]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1, NCCL)
    python bench.py --impl reference ...                  (the reference's CPU path, rank 0 only)

Workload (default `large`): 262144 x 262144 block rows/columns, high-variance
block sizes {8,16,56,64} w.p. {.3,.2,.2,.3}, degree 16, random pattern, RHS 64, seed 1 (~22 GB of
A). Block rows are partitioned over the ranks by balanced cost (vbsr_partition_rows); each rank
builds its shard on its GPU (values generated on the device by the engine's counter-based
generator, identical to the host generator), receives one replica of B from rank 0 over NCCL
(setup, not timed) and runs Plan.execute on its shard. No collective runs inside the timed region.

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
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

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
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
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
        for ln in self.lines:
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


# ---- CPU baseline ---------------------------------------------------------------------------------

def cpu_sample_run(host, rhs, B, r1, threads, use_ref):
    """One run of the CPU path over block rows [0, r1); returns (seconds, flops of the sample)."""
    import oracle
    sub = host.row_slice(0, r1, values_seed=SEED)
    flops = 2.0 * sub.values.size * rhs
    t = time.perf_counter()
    if use_ref:
        oracle.ref_cpu_reference(sub, B, rhs, threads=threads)
    else:
        oracle.spmm(sub, B, rhs, threads=threads)
    return time.perf_counter() - t, flops


def calibrate_cpu_rows(host, rhs, B, threads, use_ref, target_s):
    """Block rows [0, r) whose CPU run takes about target_s seconds."""
    r = min(host.block_rows, max(threads * 4, 64))
    while True:
        dt, _ = cpu_sample_run(host, rhs, B, r, threads, use_ref)
        if dt >= 0.2 * target_s or r >= host.block_rows:
            break
        r = min(host.block_rows, r * 4)
    return max(1, min(host.block_rows, int(r * target_s / max(dt, 1e-6))))


def cpu_baseline(host, rhs, B, problem_bytes, total_flops, target_s=12.0):
    import oracle
    use_ref = oracle.ref_available()
    threads = os.cpu_count() or 1
    r = calibrate_cpu_rows(host, rhs, B, threads, use_ref, target_s)
    dt, flops = cpu_sample_run(host, rhs, B, r, threads, use_ref)
    est_full = dt * total_flops / flops
    return {"value": problem_bytes / est_full / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "reference" if use_ref else "port",
            "sample": f"block rows [0,{r}) of the workload ({100 * flops / total_flops:.2f}% of its "
                      f"flops) in {dt:.2f} s on {threads} threads, extrapolated to the full "
                      f"problem by flops",
            "sample_seconds": dt}


def run_reference_arm(args):
    """--impl reference: the reference's own cpu_reference (oracle/_ref, compiled unchanged from
    the reference sources) or, if that library is absent, the bit-identical C restatement, with all
    host threads, on bounded samples of the same workload. Rank 0 only."""
    rank, world, _ = rank_env()
    if rank != 0:
        return 0
    import oracle
    import varblockspmm_b200 as vb
    host, rhs = make_structure(args.workload)
    problem_bytes, total_flops = vb.compulsory_bytes(host, rhs)
    B = vb.fill_uniform(SEED, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    use_ref = oracle.ref_available()
    threads = os.cpu_count() or 1
    per_step = max(0.3, min(6.0, 150.0 / max(1, args.steps + args.warmup)))
    r = calibrate_cpu_rows(host, rhs, B, threads, use_ref, per_step)
    for _ in range(args.warmup):
        cpu_sample_run(host, rhs, B, r, threads, use_ref)
    times = []
    flops = 0.0
    for _ in range(args.steps):
        dt, flops = cpu_sample_run(host, rhs, B, r, threads, use_ref)
        times.append(dt)
    med = statistics.median(times)
    est_full_s = med * total_flops / flops
    value = problem_bytes / est_full_s / 1e9
    line = {
        "metric": "spmm_effective_hbm_GBps", "impl": "reference", "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": est_full_s * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator)",
        "config": {"workload": WORKLOADS[args.workload][5], "rhs": rhs,
                   "block_rows": host.block_rows, "compulsory_bytes": problem_bytes},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads,
                         "kind": "reference" if use_ref else "port",
                         "sample": f"block rows [0,{r}) per step "
                                   f"({100 * flops / total_flops:.2f}% of the flops), "
                                   f"median {med:.3f} s, extrapolated by flops"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- GPU arm --------------------------------------------------------------------------------------

def sampled_parity(host, rhs, row_range, dC, B_host, n_rows=12):
    """Size-independent parity at full size: a deterministic sample of this rank's block rows is
    recomputed by the oracle (values regenerated from the counter stream) and compared under
    |C - C_ref| <= 1e-5 * sum|a||b|. Returns (max error/limit ratio, violations)."""
    import oracle
    import torch
    r0, r1 = row_range
    if r1 <= r0:
        return 0.0, 0
    rng = np.random.default_rng(1234 + r0)
    picks = sorted(set([r0, r1 - 1] + list(rng.integers(r0, r1, n_rows))))
    M_r = int(host.row_scalar_off[r1] - host.row_scalar_off[r0])
    Cv = dC.view(rhs, M_r)
    worst, bad = 0.0, 0
    for i in picks:
        sub = host.row_slice(i, i + 1, values_seed=SEED)
        a = int(host.row_scalar_off[i] - host.row_scalar_off[r0])
        got = Cv[:, a:a + int(host.row_size[i])].contiguous().cpu().numpy().reshape(-1)
        ratio, _, nb = oracle.compare(sub, B_host, rhs, got, threads=1)
        worst, bad = max(worst, ratio), bad + nb
    return worst, bad


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


def time_headline(vb, torch, stream, peak, steps=200, warmup=10):
    """BASELINE config 3 on this GPU: per-launch device time with L2 flushed between launches."""
    host, rhs = make_structure("headline")
    problem_bytes, flops = vb.compulsory_bytes(host, rhs)
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
    ts = sorted(a.elapsed_time(b) for a, b in ev)
    med = ts[len(ts) // 2]
    p95 = ts[min(len(ts) - 1, int(len(ts) * 0.95))]
    B_host = vb.fill_uniform(SEED, vb.STREAM_DENSE, 0, host.scalar_cols() * rhs)
    ratio, bad = sampled_parity(host, rhs, (0, host.block_rows), Cd, B_host, n_rows=64)
    gbs = problem_bytes / (med * 1e-3) / 1e9
    return {"workload": WORKLOADS["headline"][5], "median_ms": med, "p95_ms": p95,
            "GBps": gbs, "frac_of_measured_hbm": gbs / peak, "compulsory_bytes": problem_bytes,
            "useful_TFLOPs": flops / (med * 1e-3) / 1e12, "l2": "flushed before every launch",
            "plan": p.describe(), "parity_max_ratio": ratio, "parity_violations": bad,
            "cta_time": cta_time_stats(p, B, Cd, stream)}


def run_gpu_arm(args):
    import torch
    import torch.distributed as dist
    import varblockspmm_b200 as vb

    rank, world, local = rank_env()
    if world != args.gpus:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    stream = torch.cuda.Stream()
    peak, peak_kind = measured_hbm_peak()

    host, rhs = make_structure(args.workload)
    problem_bytes, total_flops = vb.compulsory_bytes(host, rhs)
    bounds = vb.partition_rows(host, world, rhs)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    rank_bytes, rank_flops = vb.compulsory_bytes(host, rhs, r0, r1)
    M_r = int(host.row_scalar_off[r1] - host.row_scalar_off[r0])
    K = host.scalar_cols()

    t_setup = time.perf_counter()
    m = vb.Matrix(host, device=local, rows=(r0, r1), generated_seed=SEED)
    plan = vb.Plan(m, vb.PlanOptions(rhs))
    dB = torch.empty(K * rhs, device="cuda")
    torch.cuda.synchronize()
    t_rep0 = time.perf_counter()
    if rank == 0:
        vb.fill_uniform_device(SEED, vb.STREAM_DENSE, 0, dB.numel(), dB, stream)
        stream.synchronize()
    if world > 1:
        dist.broadcast(dB, src=0)  # B replica over NVLink (setup; not timed as SpMM)
    torch.cuda.synchronize()
    replicate_ms = (time.perf_counter() - t_rep0) * 1e3
    dC = torch.empty(max(1, M_r * rhs), device="cuda")
    setup_s = time.perf_counter() - t_setup

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    flush = None
    if rank_bytes < 2 * L2_BYTES:
        flush = torch.empty(2 * L2_BYTES // 4, device="cuda")

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            plan.execute(dB, dC, stream)
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
                plan.execute(dB, dC, stream)
                evs[i][1].record(stream)
            t1.record(stream)
        barrier()
    total_ms = t0.elapsed_time(t1)
    launch_ms = sorted(a.elapsed_time(b) for a, b in evs)
    med = launch_ms[len(launch_ms) // 2]
    p95 = launch_ms[min(len(launch_ms) - 1, int(len(launch_ms) * 0.95))]
    mean_launch = sum(launch_ms) / len(launch_ms)
    plan.check_status(stream)

    stats = torch.tensor([total_ms, med, p95, mean_launch], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    total_ms, med_max, p95_max, _ = stats.tolist()
    ms_per_step = total_ms / args.steps if flush is None else med_max

    cta_stats = cta_time_stats(plan, dB, dC, stream)

    # ---- the SpMM kernel alone (roofline): a second plan that skips the B pre-pass ---------------
    kplan = vb.Plan(m, vb.PlanOptions(rhs), vb.PLAN_DIAG_SKIP_PREPASS)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            kplan.execute(dB, dC, stream)
        for i in range(args.steps):
            if flush is not None:
                flush.fill_(float(i))
            kev[i][0].record(stream)
            kplan.execute(dB, dC, stream)
            kev[i][1].record(stream)
    stream.synchronize()
    kernel_ms = sum(a.elapsed_time(b) for a, b in kev) / args.steps
    kt = torch.tensor([kernel_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
    kernel_ms = float(kt.item())
    del kplan

    # ---- end to end through the public API with host buffers ---------------------------------
    # Every step uploads its B from pinned host memory, executes, and downloads its C. Steps are
    # pipelined the way a serving loop would run them: B and C are double-buffered on the device,
    # uploads run on one copy stream and downloads on another, so step i+1's upload overlaps step
    # i's download (the two PCIe directions) and execute. The timed region spans the first upload
    # to the last download.
    B_host = vb.fill_uniform(SEED, vb.STREAM_DENSE, 0, K * rhs)
    hB = torch.from_numpy(B_host).pin_memory()
    hC = [torch.empty(max(1, M_r * rhs), dtype=torch.float32).pin_memory() for _ in range(2)]
    dB2, dC2 = [dB, torch.empty_like(dB)], [dC, torch.empty_like(dC)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    e2e_steps = max(2, min(args.steps, 8))
    ev = [[torch.cuda.Event() for _ in range(e2e_steps)] for _ in range(3)]  # uploaded, run, down
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(e2e_steps):
        b = i % 2
        if i >= 2:
            s_in.wait_event(ev[1][i - 2])  # the execute that read dB[b] is done
        with torch.cuda.stream(s_in):
            dB2[b].copy_(hB, non_blocking=True)
        ev[0][i].record(s_in)
        stream.wait_event(ev[0][i])
        if i >= 2:
            stream.wait_event(ev[2][i - 2])  # dC[b] of step i-2 is downloaded
        plan.execute(dB2[b], dC2[b], stream)
        ev[1][i].record(stream)
        s_out.wait_event(ev[1][i])
        with torch.cuda.stream(s_out):
            hC[b].copy_(dC2[b], non_blocking=True)
        ev[2][i].record(s_out)
    e1.record(s_out)
    e1.synchronize()
    torch.cuda.synchronize()
    del dB2, dC2
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    # ---- parity at full size on a sample of rows -------------------------------------------------
    ratio, bad = sampled_parity(host, rhs, (r0, r1), dC, B_host)
    pr = torch.tensor([ratio, float(bad)], dtype=torch.float64, device="cuda")
    gathered = None
    if world > 1:
        dist.all_reduce(pr, op=dist.ReduceOp.MAX)
        gathered = gathered_parity(host, rhs, bounds, rank, world, dC, B_host)

    headline = None
    cpu = None
    if world == 1:
        if args.workload != "headline":
            headline = time_headline(vb, torch, stream, peak)
        if not args.no_cpu_baseline:
            cpu = cpu_baseline(host, rhs, B_host, problem_bytes, total_flops)

    if rank == 0:
        value = problem_bytes / (ms_per_step * 1e-3) / 1e9
        achieved = rank_bytes / (kernel_ms * 1e-3) / 1e9
        traffic = traffic_from_profiles(args.workload) if world == 1 else None
        line = {
            "metric": "spmm_effective_hbm_GBps", "value": value, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "median_ms": med_max, "p95_ms": p95_max,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded spec generator; A values generated on device, bit-identical "
                    "to the host generator)",
            "config": {"workload": WORKLOADS[args.workload][5], "block_rows": host.block_rows,
                       "nnzb": host.nnzb, "rhs": rhs, "compulsory_bytes": problem_bytes,
                       "useful_flops": total_flops,
                       "parallelism": f"block-row partition over {world} GPU(s), B replicated",
                       "l2": ("inputs larger than L2 (A is %.1f GB)" % (rank_bytes / 1e9))
                       if flush is None else "L2 flushed before every launch",
                       "plan": plan.describe()},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": rank_bytes,
                         "kernel": "vbsr_b200::spmm_tc_kernel", "kernel_ms": kernel_ms,
                         "execute_ms": mean_launch,
                         "execute_frac": rank_bytes / (mean_launch * 1e-3) / 1e9 / peak,
                         "note": "achieved = compulsory bytes of the rank / mean duration of the "
                                 "SpMM kernel alone (events around executes of a plan that skips "
                                 "the B pre-pass); execute_frac covers pre-pass + kernel"},
            "useful_TFLOPs": total_flops / (ms_per_step * 1e-3) / 1e12,
            "e2e": {"value": problem_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": K * rhs * 4,
                    "d2h_bytes_per_step": M_r * rhs * 4, "steps": e2e_steps,
                    "path": "pinned host B -> device, Plan.execute (C ABI), device C -> pinned "
                            "host, every step; steps pipelined (double-buffered B and C, upload "
                            "and download on separate copy streams)"},
            "gpu_launches": args.steps * plan.launch_count(),
            "clocks": clocks.summary(),
            "parity": {"sampled_rows_max_err_over_bound": pr[0].item(),
                       "violations": int(pr[1].item())},
            "setup_s": setup_s, "replicate_ms": replicate_ms, "cta_time": cta_stats,
        }
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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
