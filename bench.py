#!/usr/bin/env python
"""bench.py — emulated MAC/s of the policy sweep on B200.

Workload (the reference's large policy sweep): GEMMs of M = N = K = 8192 on
N(0,1) x lognormal(0,1) inputs held as fp32 values in doubles; the 12
accumulator x order x cast policies of RealDotSweep
(java/src/main/java/io/drift/tools/RealDotSweep.java:97-108) plus the FP64
exact GEMM they are scored against. One step on one rank is one seed: cast,
contract and score all 12 policies and run the exact GEMM. Each rank takes its
own seed (rank + world * step), so per-GPU work is fixed as GPUs are added
(weak scaling); at 8 GPUs one step is the whole 12 x 8 sweep. Error and clamp
statistics are summed across ranks with NCCL all-reduce.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--size 8192]
    python bench.py --impl reference ...   # the oracle, timed on the host cores

`value` counts every emulated multiply-accumulate (13 GEMMs per step per
rank) over the max-over-ranks device time of the K timed steps. `e2e` runs the
same step through the C ABI's one-call sweep (drift_real_dot_sweep) on pinned
host buffers: both operands copied in and the statistics read back inside the
timed region, every step.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "bit-exact emulated MAC/s per policy at 1/2/4/8 B200 vs Java host; mismatches=0"

# DRAM bytes per emulated MAC of the contraction, from one ncu capture of the
# same kernels at 4096^3 (dram__bytes_read.sum + dram__bytes_write.sum per
# launch over its MACs); a launch's traffic scales with its MAC count because
# every operand tile is re-read once per 64-wide output tile.
DRAM_BYTES_PER_MAC = {"pairwise": 0.144, "other": 0.0583}
UNIT = "emulated MAC/s"
# The sweep's policies by name, in order (sweep_policies builds them for the
# engine; the reference arm, which loads no engine code, names them here).
SWEEP_NAMES = ["fp32 sequential", "fp32 pairwise", "fp32 blocked", "fp16 sequential",
               "fp16 pairwise", "fp16 blocked", "bf16 sequential", "bf16 pairwise",
               "bf16 blocked", "bf16 cast", "e4m3 per-tensor cast", "e4m3 mx32 cast"]


def sweep_policies(d):
    """RealDotSweep's policy list (RealDotSweep.java:97-108)."""
    from drift_b200 import sweeps

    return sweeps.policy_sweep_policies()


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while a region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.device),
                                      f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=6)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in self.rows for k in range(4)
                          if len(r) > 5 + k and r[5 + k].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


# ------------------------------------------------------------------ distributed

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------ CPU baseline

# The fixed CPU sample, the same in the engine arm's cpu_baseline leg and in
# the reference arm: for each of the 13 GEMMs, SAMPLE_ROWS rows of A against
# SAMPLE_COLS rows of B with the full K terms.
SAMPLE_ROWS, SAMPLE_COLS = 64, 512


class CpuSample:
    """The sweep's 13 GEMMs on the oracle (the C restatement of the Java
    path) over one fixed row sample of the same workload: SAMPLE_ROWS x
    SAMPLE_COLS outputs each, full K = size terms. Per-tensor scales come from
    the full tensors, as in the real job; the casts run once, before any
    timing (over the whole job they are about 1e-4 of the contraction work)."""

    def __init__(self, size: int, threads: int | None = None):
        import numpy as np
        from oracle import oracle as O

        self.O = O
        self.threads = threads or os.cpu_count() or 1
        self.K = K = size
        self.rows = min(size, SAMPLE_ROWS)
        self.cols = min(size, SAMPLE_COLS)
        rs = np.random.default_rng(0)
        full_a = rs.standard_normal(size * K) * np.exp(rs.standard_normal(size * K))
        full_b = rs.standard_normal(size * K) * np.exp(rs.standard_normal(size * K))
        amax_a, amax_b = O.amax(full_a), O.amax(full_b)
        pols = [O.policy(acc=O.ACC_FP64)]
        for acc in (O.ACC_FP32, O.ACC_FP16, O.ACC_BF16):
            for order in (O.SEQUENTIAL, O.PAIRWISE, O.BLOCKED):
                pols.append(O.policy(acc=acc, order=order))
        pols.append(O.policy(input_format=O.BF16))
        pols.append(O.policy(input_format=O.E4M3, scaling=O.PER_TENSOR))
        pols.append(O.policy(input_format=O.E4M3, scaling=O.MX_BLOCK))
        A = full_a[:self.rows * K].copy()
        B = full_b[:self.cols * K].copy()
        del full_a, full_b
        self.work = []
        for p in pols:
            if p.input_format < 0:
                self.work.append((p, A, B))
                continue
            f = p.input_format
            sa = O.per_tensor_scale(f, amax_a) if p.scaling == O.PER_TENSOR else 1.0
            sb = O.per_tensor_scale(f, amax_b) if p.scaling == O.PER_TENSOR else 1.0
            self.work.append((p, O.quantize(p, f, 0, A, sa)[0], O.quantize(p, f, 0, B, sb)[0]))
        self.macs = len(pols) * self.rows * self.cols * K

    def run(self) -> float:
        """One pass over the sample; returns its wall time in seconds."""
        t0 = time.perf_counter()
        for p, qa, qb in self.work:
            self.O.gemm(p, self.rows, self.cols, self.K, qa, 0, self.K, 1, qb, 0, self.K, 1,
                        threads=self.threads)
        return time.perf_counter() - t0

    def describe(self, seconds: float) -> str:
        return (f"oracle (C restatement of the Java path, -O2, no FMA) on {self.threads} host "
                f"threads: {len(self.work)} GEMMs of {self.rows} x {self.cols} outputs with "
                f"K={self.K} (the first rows of A and B of the seed-0 workload); "
                f"{self.macs:.3e} MACs in {seconds:.2f} s")


def cpu_baseline(size: int, repeats: int = 3):
    """The engine arm's cpu_baseline leg: the fixed sample, timed `repeats`
    times after one untimed pass; the median pass. Returns (MAC/s, threads,
    description)."""
    smp = CpuSample(size)
    smp.run()
    times = sorted(smp.run() for _ in range(max(1, repeats)))
    t = statistics.median(times)
    return smp.macs / t, smp.threads, smp.describe(t)


# ------------------------------------------------------------------ engine arm

def run_engine(args):
    import numpy as np
    import torch
    import drift_b200 as d

    from drift_b200 import dist as ddist
    from drift_b200 import stats as dstats

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    d.Context.use_device(local)
    ctx = d.Context.current()
    pg = None
    if world > 1:
        pg = ddist.init("nccl", timeout_s=600, device=torch.device("cuda", local))
    stream = torch.cuda.current_stream()
    S = args.size
    M = N = K = S
    pols = sweep_policies(d)
    exact_p = d.NumericPolicy.exact()
    dev = torch.device("cuda", local)

    def make_inputs(seed):
        from drift_b200 import sweeps

        return sweeps.policy_sweep_inputs(S, seed, dev)

    seed = ddist.seeds_for(rank, world, 0)[0]  # this rank's seed, the same every step
    A, B = make_inputs(seed)
    qA = torch.empty_like(A)
    qB = torch.empty_like(B)
    C = torch.empty((M, N), dtype=torch.float64, device=dev)
    Cx = torch.empty((M, N), dtype=torch.float64, device=dev)
    n_pol = len(pols)
    sums = torch.zeros((n_pol, 2), dtype=torch.float64, device=dev)
    med_state = torch.zeros((n_pol, 2), dtype=torch.int64, device=dev)
    med_hist = torch.empty(dstats.RADIX_BINS, dtype=torch.int64, device=dev)
    clamps = torch.zeros((n_pol, 2), dtype=torch.int64, device=dev)  # clamps in A, in B
    scal = torch.zeros((4,), dtype=torch.float64, device=dev)  # amax A, amax B, scale A, scale B
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n_pol + 1)]
    gemm_ms = [0.0] * (n_pol + 1)
    launches = [0]
    # Each contraction's route (drift_gemm_route), read in the first warm-up
    # step. The kernels each GEMM call queued (operand scans, decisions and
    # both builds of a scanned route, one of which stands down at once) come
    # from drift_gemm_launches, a host-side count read after every call.
    routes = [None] * (n_pol + 1)

    def gemm_launches():
        return d.gemm_launches(ctx=ctx)

    # The cast pass's own device time (the quantize launch of each cast policy's
    # A operand, last step), for its HBM roofline.
    cast_ev = {k: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for k, p in enumerate(pols) if p.input_format is not None}

    def cast(p, src, dst, slot, counter, k=None):
        f = p.input_format
        if f is None:
            return src
        timed = k in cast_ev and slot == 0
        if p.scaling == d.Scaling.PER_TENSOR:
            d.amax_dev(src, scal[slot:slot + 1], ctx=ctx)
            d.per_tensor_scale_dev(f, scal[slot:slot + 1], scal[2 + slot:3 + slot], ctx=ctx)
            if timed:
                cast_ev[k][0].record(stream)
            d.quantize_dev(p, f, p.input_rounding, src, dst, d_scale=scal[2 + slot:3 + slot],
                           d_clamped=counter, ctx=ctx)
            launches[0] += 3
        else:
            if timed:
                cast_ev[k][0].record(stream)
            d.quantize_dev(p, f, p.input_rounding, src, dst, d_clamped=counter, ctx=ctx)
            launches[0] += 1
        if timed:
            cast_ev[k][1].record(stream)
        return dst

    def step(read_routes: bool):
        ev[0][0].record(stream)
        d.gemm_dev(exact_p, A, B, Cx, ctx=ctx)
        ev[0][1].record(stream)
        if read_routes:
            routes[0] = d.gemm_route(ctx=ctx)
        launches[0] += gemm_launches()
        for k, p in enumerate(pols):
            a = cast(p, A, qA, 0, clamps[k, 0:1], k)
            b = cast(p, B, qB, 1, clamps[k, 1:2])
            ev[k + 1][0].record(stream)
            d.gemm_dev(p, a, b, C, ctx=ctx)
            ev[k + 1][1].record(stream)
            if read_routes:
                routes[k + 1] = d.gemm_route(ctx=ctx)
            launches[0] += gemm_launches() - 1
            d.error_sums_dev(C, Cx, sums[k], ctx=ctx)
            # DotSweep's summary statistic over every rank's outputs: the upper
            # median of the relative errors (DotSweep.java:152-153).
            dstats.select_rel_error_dev(C, Cx, (world * M * N) // 2, med_state[k], med_hist,
                                        dist=pg, ctx=ctx)
            launches[0] += 2 + 2 * dstats.RADIX_PASSES
        ddist.reduce_stats(sums, clamps, pg)

    def barrier():
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
            torch.cuda.synchronize()

    for w in range(args.warmup):
        step(w == 0)
    d.check_dev(ctx=ctx)
    barrier()
    sums.zero_()
    clamps.zero_()
    launches[0] = 0
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        t_start.record(stream)
        for _ in range(args.steps):
            step(True)
        t_end.record(stream)
        barrier()
    # Per-GEMM device times of the last step (events on the launching stream).
    for k in range(n_pol + 1):
        gemm_ms[k] = ev[k][0].elapsed_time(ev[k][1])
    d.check_dev(ctx=ctx)
    ms_max = ddist.max_over_ranks(t_start.elapsed_time(t_end), pg, dev)
    macs_per_step_rank = (n_pol + 1) * M * N * K
    value = macs_per_step_rank * world * args.steps / (ms_max * 1e-3)
    # The 12 policies alone: their MACs over the step time less the exact
    # GEMM's device time (last step's events, max over ranks).
    exact_ms = ddist.max_over_ranks(gemm_ms[0], pg, dev)
    value_excl = n_pol * M * N * K * world / ((ms_max / args.steps - exact_ms) * 1e-3)

    # Roofline of the dominant kernel, the double-precision contraction
    # (gemm_kernel, every contraction not on the FP32 pipe): FP64-pipe work is
    # 2 operations (DMUL + DADD) per emulated MAC; the peak is this GPU's
    # measured DMUL+DADD rate. The FP32-pipe contractions (gemm_f32_kernel)
    # get their own line: one FFMA per MAC against the measured FFMA rate.
    fp64_peak = d.probe_fp64(ctx)
    fp32_peak = d.probe_fp32(ctx)
    on_fp32 = [k for k in range(n_pol + 1) if routes[k] == d.ROUTE_FP32]
    on_fp64 = [k for k in range(n_pol + 1) if routes[k] != d.ROUTE_FP32]
    gemm_total_ms = sum(gemm_ms[k] for k in on_fp64)
    achieved = 2.0 * len(on_fp64) * M * N * K / (gemm_total_ms * 1e-3)
    fp32_ms = sum(gemm_ms[k] for k in on_fp32)
    fp32_achieved = len(on_fp32) * M * N * K / (fp32_ms * 1e-3) if on_fp32 else 0.0
    all_pols = [exact_p] + list(pols)
    names = ["exact fp64"] + [p.name for p in pols]
    n_pair = sum(1 for k in on_fp64 if all_pols[k].order == d.Order.PAIRWISE)
    traffic_per_launch = M * N * K * (n_pair * DRAM_BYTES_PER_MAC["pairwise"] +
                                      (len(on_fp64) - n_pair) * DRAM_BYTES_PER_MAC["other"]) \
        / len(on_fp64)
    # The HBM view of the same launches: their DRAM traffic over their time,
    # against the measured copy bandwidth of this pool's B200s.
    hbm_peak, hbm_src = 6650.0, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"
    try:
        hbm_peak = float(json.load(open(REPO / "MEASURED_PEAKS.json"))["hbm_gbs"])
        hbm_src = "MEASURED_PEAKS.json hbm_gbs"
    except (OSError, KeyError, ValueError):
        pass
    hbm_gbs = traffic_per_launch * len(on_fp64) / (gemm_total_ms * 1e-3) / 1e9
    # The cast pass (cast_vec_kernel): 8 bytes read and 8 written per element.
    cast_bytes = 16 * M * K
    cast_line = {}
    for k, (e0, e1) in cast_ev.items():
        ms = e0.elapsed_time(e1)
        cast_line[pols[k].name] = {"ms": ms, "achieved": cast_bytes / (ms * 1e-3) / 1e9,
                                   "frac": cast_bytes / (ms * 1e-3) / 1e9 / hbm_peak}
    per_policy = {"exact fp64": M * N * K / (gemm_ms[0] * 1e-3)}
    for k, p in enumerate(pols):
        per_policy[p.name] = M * N * K / (gemm_ms[k + 1] * 1e-3)

    # Statistics (summed over ranks): RMS ratio and clamps per pair.
    s = sums.cpu().numpy()
    c = clamps.cpu().numpy()
    med = med_state.cpu().numpy()
    stats = {p.name: {"median_rel_error": dstats.bits_to_double(med[k, 0]),
                      "rms_error_ratio": ddist.rms_ratio(float(s[k, 0]), float(s[k, 1])),
                      # DotSweep's clamps per pair (DotSweep.java:119-120): clamps in
                      # row i of A plus clamps in row j of B, averaged over all pairs.
                      "clamped_per_pair": (float(c[k, 0]) / M + float(c[k, 1]) / N)
                      / (args.steps * world)}
             for k, p in enumerate(pols)}

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(d, args, A, B, pols, exact_p, world, rank, pg)

    # The host-core baseline is timed at N = 1 only (rank 0); at N > 1 the
    # line carries none, so no rank waits on it.
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, desc = cpu_baseline(S)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc}

    ddist.finish(pg)
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "value_excluding_exact": value_excl,
        "value_excluding_exact_note": "the 12 policies' MACs over the step time less the exact "
                                      "FP64 GEMM's device time",
        "data": "synthetic: N(0,1) x lognormal(0,1) doubles (53-bit, like Java's nextGaussian), "
                "seeded per rank",
        "config": {"workload": f"policy sweep GEMM M=N=K={S}, 12 policies + exact FP64, "
                               f"1 seed per rank per step", "M": M, "N": N, "K": K,
                   "policies": [p.name for p in pols], "seeds_per_step": world, "seed_of_rank_0": 0,
                   "l2": "inputs (2 x 512 MiB at 8192) are larger than L2",
                   "parallelism": f"shard by seed x{world}"},
        "roofline": {"bound": "fp64", "achieved": achieved / 1e12, "peak": fp64_peak / 1e12,
                     "unit": "TFLOP/s", "frac": achieved / fp64_peak,
                     "traffic": traffic_per_launch,
                     "traffic_unit": "bytes per double-precision contraction launch, averaged "
                                     "over the step's launches of it",
                     "kernel": "gemm_kernel",
                     "contractions": [names[k] for k in on_fp64],
                     "hbm_view": {"achieved": hbm_gbs, "peak": hbm_peak, "unit": "GB/s",
                                  "frac": hbm_gbs / hbm_peak, "peak_source": hbm_src,
                                  "note": "DRAM traffic of the contraction launches (per-MAC "
                                          "bytes from the ncu capture) over their time"},
                     "peak_source": "measured DMUL+DADD probe (drift_probe_fp64) on this GPU",
                     "fp32_pipe": {"kernel": "gemm_f32_kernel",
                                   "contractions": [names[k] for k in on_fp32],
                                   "achieved": fp32_achieved / 1e12, "peak": fp32_peak / 1e12,
                                   "unit": "TFMA/s", "frac": fp32_achieved / fp32_peak,
                                   "peak_source": "measured FFMA probe (drift_probe_fp32) on "
                                                  "this GPU",
                                   "note": "one FFMA per emulated MAC; the time includes the "
                                           "operand scans and the decision"},
                     "cast_pass": {"kernel": "cast_vec_kernel", "bound": "hbm", "unit": "GB/s",
                                   "peak": hbm_peak, "peak_source": hbm_src,
                                   "bytes_per_element": 16, "per_policy": cast_line,
                                   "note": "the quantize launch of one 8192 x 8192 operand, "
                                           "CUDA events on the launching stream, last step"}},
        "per_policy_mac_per_s": per_policy,
        "stats": stats,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": launches[0],
    }
    print(json.dumps(line), flush=True)
    return 0


def run_e2e(d, args, A, B, pols, exact_p, world, rank, pg):
    """The same step through the reference-facing host entry point: one
    drift_real_dot_sweep call per step on pinned host copies of this rank's
    A and B (RealDotSweep's loop, RealDotSweep.java:119-142). Inside the timed
    region, every step copies both operands in, runs the exact GEMM and the 12
    policies' casts, contractions and statistics, and reads the statistics
    back; only statistics cross back, as in the reference, which keeps the
    outputs in the loop that scores them."""
    import torch

    from drift_b200 import dist as ddist
    from drift_b200 import sweeps

    S = args.size
    hA = torch.empty((S, S), dtype=torch.float64, pin_memory=True)
    hB = torch.empty((S, S), dtype=torch.float64, pin_memory=True)
    hA.copy_(A)
    hB.copy_(B)
    a, b = hA.numpy(), hB.numpy()
    P = len(pols)
    # Per step: both operands and the radix selections' start states in; the
    # sums, clamp counts, selected medians and the error word out.
    h2d = a.nbytes + b.nbytes + 4 * 8 * P
    d2h = (2 + 2 + 4) * 8 * P + 4

    def one_step():
        return sweeps.real_dot_sweep(a, b, pols)

    one_step()  # warm-up
    steps = max(1, args.e2e_steps)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        out = one_step()
    dt = time.perf_counter() - t0
    dt = ddist.max_over_ranks(dt, pg, torch.device("cuda", torch.cuda.current_device()))
    macs = (P + 1) * S ** 3 * world * steps
    return {"value": macs / dt, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps,
            "path": "drift_real_dot_sweep on pinned host buffers (one C-ABI call per step; "
                    "statistics per rank)",
            "stats_rank0": {k: {"median_rel_error": v["median_rel_error"],
                                "rms_error_ratio": v["rms_error_ratio"]}
                            for k, v in out.items()} if rank == 0 else None}


# ------------------------------------------------------------------ reference arm

def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    smp = CpuSample(args.size)
    for _ in range(args.warmup):
        smp.run()
    times = [smp.run() for _ in range(args.steps)]
    t = statistics.median(times)
    value = smp.macs / t
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup,
        # Each step is one pass over the fixed sample; this is its measured time.
        "ms_per_step": t * 1e3, "higher_is_better": True,
        "full_step_ms_extrapolated": 13 * float(args.size) ** 3 / value * 1e3,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "impl": "reference",
        "data": "synthetic: N(0,1) x lognormal(0,1) doubles (53-bit, like Java's nextGaussian)",
        "config": {"workload": f"policy sweep GEMM M=N=K={args.size}, 12 policies + exact FP64, "
                               f"1 seed per rank per step", "M": args.size, "N": args.size,
                   "K": args.size, "policies": SWEEP_NAMES,
                   "seeds_per_step": 1, "parallelism": "host threads of rank 0"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": smp.threads, "kind": "port",
                         "sample": smp.describe(t)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "no JVM on this image: the reference's Java path is timed through its C "
                "restatement (the oracle), with all host threads. A step is one pass over a "
                "fixed row sample of the workload (the same sample as the engine arm's "
                "cpu_baseline); ms_per_step is that pass's median time, and "
                "full_step_ms_extrapolated is a whole step at the measured rate",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_kernels(args):
    """Per-policy contraction timing at one size (also the command ncu profiles):
    each selected policy's GEMM runs once to warm up, then `--steps` times under
    CUDA events on the launching stream."""
    import torch
    import drift_b200 as d

    S = args.size
    M, N, K = (int(x) for x in args.mnk.split(",")) if args.mnk else (S, S, S)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    f64 = torch.float64
    A = (torch.randn(M, K, device=dev, generator=g, dtype=f64) *
         torch.exp(torch.randn(M, K, device=dev, generator=g, dtype=f64)))
    B = (torch.randn(N, K, device=dev, generator=g, dtype=f64) *
         torch.exp(torch.randn(N, K, device=dev, generator=g, dtype=f64)))
    C = torch.empty((M, N), dtype=f64, device=dev)
    qA, qB = torch.empty_like(A), torch.empty_like(B)
    scal = torch.zeros((4,), dtype=torch.float64, device=dev)
    pols = [d.NumericPolicy.exact()] + sweep_policies(d)
    if args.policies:
        keep = [x.strip() for x in args.policies.split(",")]
        pols = [p for p in pols if p.name in keep]
    stream = torch.cuda.current_stream()
    out, routes = {}, {}
    for p in pols:
        # The policy's input cast, as in the sweep step, outside the timing.
        a, b = A, B
        if p.input_format is not None:
            a, b = qA, qB
            for k, (src, dst) in enumerate(((A, qA), (B, qB))):
                if p.scaling == d.Scaling.PER_TENSOR:
                    d.amax_dev(src, scal[k:k + 1])
                    d.per_tensor_scale_dev(p.input_format, scal[k:k + 1], scal[2 + k:3 + k])
                    d.quantize_dev(p, p.input_format, p.input_rounding, src, dst,
                                   d_scale=scal[2 + k:3 + k])
                else:
                    d.quantize_dev(p, p.input_format, p.input_rounding, src, dst)
        d.gemm_dev(p, a, b, C)
        routes[p.name] = d.gemm_route()
        if args.steps > 0:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                d.gemm_dev(p, a, b, C)
            e1.record(stream)
            torch.cuda.synchronize()
            out[p.name] = args.steps * M * N * K / (e0.elapsed_time(e1) * 1e-3)
    d.check_dev()
    print(json.dumps({"mode": "kernels", "M": M, "N": N, "K": K, "mac_per_s": out,
                      "routes": routes}), flush=True)
    return 0


def run_train(args):
    """The training-step configuration (vocab 96, ctx 32, emb 64, hidden 2048,
    batch 64) under fp8 delayed scaling with stochastic gradient rounding:
    steps per second and emulated MAC/s of the device-resident step, and of
    the same step through the host-buffer entry points. A step is one policy
    pass and the Adam update; measurement steps (exact recompute) are moved
    out of the timed window."""
    import numpy as np
    import torch
    import drift_b200 as d
    from drift_b200 import mlp, mlp_dev

    p = (d.policies.by_name("fp8-delayed").to_builder("fp8-delayed-sr-grads")
         .grad_rounding(d.Rounding.STOCHASTIC).build())
    far = 10 ** 9   # no measurement step inside the timed window
    tr = mlp_dev.DeviceTrainer(p, 0, measure_every=far)
    for _ in range(args.warmup):
        tr.step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tr.step()
    torch.cuda.synchronize()
    dev_s = (time.perf_counter() - t0) / args.steps
    tr.result()
    macs = tr.macs_per_step()

    net = mlp.Net(96, 32, 64, 2048, 1000)
    net.round_to_fp32()
    pas = mlp.Pass(p, net, 64, 0xC0FFEE)
    rs = np.random.default_rng(0)
    ctx, tgt = rs.integers(0, 96, 64 * 32), rs.integers(0, 96, 64)
    pas.loss_and_grads(ctx, tgt)
    t0 = time.perf_counter()
    n_host = max(1, min(args.steps, 3))
    for _ in range(n_host):
        pas.loss_and_grads(ctx, tgt)
    host_s = (time.perf_counter() - t0) / n_host
    # The four attention contractions of AttnPass (scores, context, dProb, dv)
    # at batch 64, t 256, d 64, device-resident; MACs count the dots actually
    # taken (the causal half of scores and dProb, the ragged windows).
    Bt, T, D = 64, 256, 64
    W = d.Window
    ops = {
        "scores": (d.contraction(batch=Bt, rows=T, cols=T, depth=D, a_batch=T * D, a_row=D, a_k=1,
                                 b_batch=T * D, b_col=D, b_k=1, c_batch=T * T, c_row=T,
                                 alpha=0.125, causal=True), T * D, T * D, T * T,
                   T * (T + 1) // 2 * D),
        "context": (d.contraction(batch=Bt, rows=T, cols=D, depth=T, a_batch=T * T, a_row=T, a_k=1,
                                  b_batch=T * D, b_col=1, b_k=D, c_batch=T * D, c_row=D,
                                  window=W.PREFIX), T * T, T * D, T * D, T * (T + 1) // 2 * D),
        "dv": (d.contraction(batch=Bt, rows=T, cols=D, depth=T, a_batch=T * T, a_row=1, a_k=T,
                             b_batch=T * D, b_col=1, b_k=D, c_batch=T * D, c_row=D,
                             window=W.SUFFIX), T * T, T * D, T * D, T * (T + 1) // 2 * D),
    }
    attn = {}
    dev = torch.device("cuda", 0)
    for pname in ("exact", "fp8-acc-bf16", "acc-bf16-pairwise"):
        pol = d.policies.by_name(pname)
        row = {}
        for name, (op, na, nb, nc, macs_b) in ops.items():
            A = torch.randn(Bt * na, dtype=torch.float64, device=dev)
            Bm = torch.randn(Bt * nb, dtype=torch.float64, device=dev)
            C = torch.empty(Bt * nc, dtype=torch.float64, device=dev)
            d.contract_dev(pol, op, A, Bm, C)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                d.contract_dev(pol, op, A, Bm, C)
            e1.record()
            torch.cuda.synchronize()
            row[name] = Bt * macs_b * args.steps / (e0.elapsed_time(e1) * 1e-3)
        attn[pname] = row
    d.check_dev()

    # The stochastically rounded BF16 accumulator (fp8-acc-bf16-sr's contraction):
    # the training step's forward shape and a square one, device-resident, the
    # Rng state advancing on the device.
    sr_pol = d.policies.by_name("fp8-acc-bf16-sr")
    sr = {}
    for (Ms, Ns, Ks) in ((64, 2048, 2048), (2048, 2048, 2048)):
        A = torch.randn(Ms, Ks, dtype=torch.float64, device=dev)
        Bm = torch.randn(Ns, Ks, dtype=torch.float64, device=dev)
        C = torch.empty(Ms, Ns, dtype=torch.float64, device=dev)
        st = torch.tensor([1], dtype=torch.int64, device=dev)
        d.gemm_dev(sr_pol, A, Bm, C, d_rng_state=st)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            d.gemm_dev(sr_pol, A, Bm, C, d_rng_state=st)
        torch.cuda.synchronize()
        sr[f"{Ms}x{Ns}x{Ks}"] = Ms * Ns * Ks * args.steps / (time.perf_counter() - t0)

    print(json.dumps({"mode": "train", "policy": p.name, "macs_per_step": macs,
                      "attention_mac_per_s": attn, "sr_accumulator_mac_per_s": sr,
                      "config": {"vocab": 96, "ctx": 32, "emb": 64, "hidden": 2048, "batch": 64},
                      "device_resident": {"s_per_step": dev_s, "mac_per_s": macs / dev_s,
                                          "steps": args.steps},
                      "host_buffers": {"s_per_step": host_s, "mac_per_s": macs / host_s,
                                       "steps": n_host, "note": "no Adam step"}}), flush=True)
    return 0


def _cpu_dot_sweep(inputs, policies, threads):
    """The dot sweep on the oracle (the C restatement of DotSweep.run,
    DotSweep.java:112-122) over the given vectors: (policy, length) groups in
    parallel on `threads` host threads. Returns seconds."""
    import concurrent.futures as cf
    from oracle import oracle as O

    def opol(p):
        c = p.to_c()
        return O.OraclePolicy(*[getattr(c, f) for f, _ in c._fields_])

    exact = O.policy(acc=O.ACC_FP64)

    def group(p, n):
        op = opol(p)
        f = p.input_format
        fid = f.id if f is not None else -1
        A, B = inputs[n]
        for seed in range(A.shape[0]):
            a, b = A[seed], B[seed]
            rng = 0xD1F7 + seed
            if f is not None:
                sa = O.per_tensor_scale(fid, O.amax(a))
                sb = O.per_tensor_scale(fid, O.amax(b))
                a, _, rng = O.quantize(op, fid, int(p.input_rounding), a, sa, rng)
                b, _, rng = O.quantize(op, fid, int(p.input_rounding), b, sb, rng)
            O.dot(a, 0, 1, b, 0, 1, n, op, rng)
            O.dot(A[seed], 0, 1, B[seed], 0, 1, n, exact)

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda pn: group(*pn), [(p, n) for p in policies for n in inputs]))
    return time.perf_counter() - t0


def _cpu_real_dot(X, W, policies, threads):
    """The real-shape batch on the oracle with `threads` host threads: casts,
    every contraction, the medians and RMS sums. Returns seconds."""
    import numpy as np
    from oracle import oracle as O

    def opol(p):
        c = p.to_c()
        return O.OraclePolicy(*[getattr(c, f) for f, _ in c._fields_])

    t0 = time.perf_counter()
    M, K = X.shape
    N = W.shape[0]
    xf, wf = X.reshape(-1), W.reshape(-1)
    exact, _ = O.gemm(O.policy(acc=O.ACC_FP64), M, N, K, xf, 0, K, 1, wf, 0, K, 1,
                      threads=threads)
    for p in policies:
        f = p.input_format
        qx, qw, rng = xf, wf, 7
        if f is not None:
            qx, _, rng = O.quantize(opol(p), f.id, 0, xf, O.per_tensor_scale(f.id, O.amax(xf)),
                                    rng)
            qw, _, rng = O.quantize(opol(p), f.id, 0, wf, O.per_tensor_scale(f.id, O.amax(wf)),
                                    rng)
        got, _ = O.gemm(opol(p), M, N, K, qx, 0, K, 1, qw, 0, K, 1, threads=threads)
        err = np.abs(got - exact).reshape(-1) / np.abs(exact).reshape(-1)
        np.partition(err, [err.size // 2 - 1, err.size // 2])
        np.sqrt(np.sum((got - exact) ** 2) / np.sum(exact ** 2))
    return time.perf_counter() - t0


def run_configs(args):
    """The other study configurations, timed end to end on one GPU (inputs
    generated or copied in, results read back), each beside the oracle on
    the host's threads over the same work: the dot sweep (200 seeds x lengths
    16..4096, 10 policies + exact, inputs generated on the device), the
    real-shape batch (4096 x 64 x 2048, 7 policies + exact, the host tensors
    copied in once) and the block-scaled GEMM (4096^3, 6 policies + exact; the
    CPU leg is a 16-row sample, scaled to the whole study)."""
    import statistics as stt

    import numpy as np
    import torch
    from drift_b200 import sweeps
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    out = {"cpu_threads": threads}
    reps = max(1, args.steps)

    def timed(fn):
        fn()   # warm-up, the same call
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            r = fn()
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        return stt.median(ts), r

    lengths = tuple(2 ** k for k in range(4, 13))
    dt, ds = timed(lambda: sweeps.dot_sweep_dev(lengths=lengths, seeds=200))
    macs = 11 * 200 * sum(lengths)
    inputs = sweeps.dot_sweep_dev(lengths=lengths, seeds=200, keep_inputs=True)["inputs"]
    cpu = _cpu_dot_sweep(inputs, sweeps.dot_sweep_policies(), threads)
    out["dot_sweep"] = {"seconds": dt, "macs": macs, "mac_per_s": macs / dt,
                        "cpu_port_seconds": cpu, "vs_cpu_port": cpu / dt,
                        "path": "device: inputs generated on the GPU, one read-back",
                        "median_rel_error_at_4096": {k: v[4096]["median_rel_error"]
                                                      for k, v in ds["table"].items()}}
    X, W = sweeps.real_dot_inputs()
    dt, rd = timed(lambda: sweeps.real_dot_batch_dev(X, W))
    macs = 8 * X.shape[0] * W.shape[0] * X.shape[1]
    cpu = _cpu_real_dot(X, W, sweeps.real_dot_policies(), threads)
    out["real_dot_batch"] = {"seconds": dt, "macs": macs, "mac_per_s": macs / dt,
                             "cpu_port_seconds": cpu, "vs_cpu_port": cpu / dt,
                             "path": "device: host X and W copied in once, one read-back",
                             "stats": rd}
    dt, mx = timed(lambda: sweeps.mx_gemm(4096))
    macs = 7 * 4096 ** 3
    A, Wm = (t.cpu().numpy() for t in sweeps.mx_gemm_inputs(4096))
    rows = 16
    t0 = time.perf_counter()
    for p in [sweeps.NumericPolicy.exact()] + sweeps.mx_policies():
        c = p.to_c()
        op = O.OraclePolicy(*[getattr(c, f) for f, _ in c._fields_])
        a, w = A[:rows].reshape(-1), Wm.reshape(-1)
        if p.input_format is not None:
            fid = p.input_format.id
            sa = O.per_tensor_scale(fid, O.amax(A)) if p.scaling == 1 else 1.0
            sw = O.per_tensor_scale(fid, O.amax(Wm)) if p.scaling == 1 else 1.0
            a = O.quantize(op, fid, 0, a, sa)[0]
            w = O.quantize(op, fid, 0, w, sw)[0]
        O.gemm(op, rows, 4096, 4096, a, 0, 4096, 1, w, 0, 4096, 1, threads=threads)
    cpu = (time.perf_counter() - t0) * 4096 / rows
    out["mx_gemm"] = {"seconds": dt, "macs": macs, "mac_per_s": macs / dt,
                      "cpu_port_seconds_extrapolated": cpu, "vs_cpu_port": cpu / dt,
                      "path": "device-resident", "stats": mx}
    print(json.dumps({"mode": "configs", **out}), flush=True)
    return 0


def run_mx(args):
    """The block-scaled GEMM study (M = N = K = size, e4m3/e2m1 x per-tensor /
    MX spec / MX +1, FP32 sequential, plus the exact GEMM) as one job over N
    ranks, each GEMM sharded by N-tile: per-GPU work shrinks as ranks are added
    (strong scaling). Device time of the whole study (casts, contractions,
    statistics) per step, max over ranks."""
    import torch
    import drift_b200 as d
    from drift_b200 import dist as ddist
    from drift_b200 import sweeps

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    d.Context.use_device(local)
    pg = None
    if world > 1:
        pg = ddist.init("nccl", timeout_s=600, device=torch.device("cuda", local))
    S = args.size
    inputs = sweeps.mx_gemm_inputs(S, 0, local)
    for _ in range(args.warmup):
        res = sweeps.mx_gemm(S, dist=pg, inputs=inputs, device=local)
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        res = sweeps.mx_gemm(S, dist=pg, inputs=inputs, device=local)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = ddist.max_over_ranks(e0.elapsed_time(e1), pg, torch.device("cuda", local))
    n_gemm = 1 + len(sweeps.mx_policies())
    macs = n_gemm * S ** 3 * args.steps
    ddist.finish(pg)
    if rank == 0:
        print(json.dumps({"mode": "mx", "metric": UNIT, "value": macs / (ms * 1e-3), "unit": UNIT,
                          "n_gpus": world, "steps": args.steps, "ms_per_step": ms / args.steps,
                          "scaling": "strong",
                          "config": {"workload": f"block-scaled GEMM study M=N=K={S}, "
                                                 f"{n_gemm - 1} policies + exact, one study per "
                                                 f"step sharded by N-tile over {world} ranks"},
                          "stats": res}), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", choices=["sweep", "kernels", "train", "configs", "mx"], default="sweep",
                    help="kernels: time each policy's contraction alone (for profiling)")
    ap.add_argument("--policies", default="", help="kernels mode: comma-separated policy names")
    ap.add_argument("--mnk", default="", help="kernels mode: M,N,K instead of size^3")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "engine":
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args)
    if args.mode == "kernels":
        return run_kernels(args)
    if args.mode == "train":
        return run_train(args)
    if args.mode == "configs":
        return run_configs(args)
    if args.mode == "mx":
        return run_mx(args)
    return run_engine(args)


if __name__ == "__main__":
    sys.exit(main())
