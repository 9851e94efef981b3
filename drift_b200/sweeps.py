"""Drivers of the reference's dot-product studies on the engine.

dot_sweep       DotSweep (java/src/main/java/io/drift/tools/DotSweep.java): many
                seeds x lengths x policies, the median relative error per
                (policy, length) and the clamps per vector pair.
real_dot_batch  RealDotSweep (java/src/main/java/io/drift/tools/RealDotSweep.java):
                4096 windows x 64 units of 2048 terms on synthetic tensors, the
                true median relative error and the RMS ratio per policy.
mx_gemm         The block-scaled GEMM study: e4m3 / e2m1 operands under per-tensor
                and MX (spec and +1) scaling, FP32 sequential accumulation, with
                clamps per vector pair and per block pair and the relative error.
policy_sweep_*  The large policy sweep: square GEMMs under RealDotSweep's 12
                accumulator x order x cast policies plus the FP64 exact GEMM.

Inputs are synthetic (seeded): N(0,1) x lognormal(0, sigma) vectors, windows
of an N(0,1) embedding table, and Kaiming-normal weights. Every cast and dot
runs in the engine; the statistics are order statistics and sums of the
bit-exact outputs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np

from .fmt import Formats, Rng, Rounding
from .kernel import Acc, NumericPolicy, Order, Quant, Scaling, gemm


def heavy_tailed(rs: np.random.Generator, n: int, sigma: float = 1.0, fp32: bool = True):
    """N(0,1) x lognormal(0, sigma); held as fp32 values when fp32 is set."""
    x = rs.standard_normal(n) * np.exp(rs.standard_normal(n) * sigma)
    return x.astype(np.float32).astype(np.float64) if fp32 else x


def dot_sweep_policies() -> List[NumericPolicy]:
    """The dot-sweep configuration: FP32/FP16/BF16 accumulators x sequential /
    pairwise / blocked-32 on uncast inputs, plus an e4m3 per-tensor cast with
    FP32 sequential accumulation (a subset of DotSweep.cases, DotSweep.java:66-106)."""
    b = NumericPolicy.builder
    ps = []
    for acc in (Acc.FP32, Acc.FP16, Acc.BF16):
        for o in (Order.SEQUENTIAL, Order.PAIRWISE, Order.BLOCKED):
            ps.append(b(f"{acc.name.lower()} {o.name.lower()}").acc(acc).order(o).acc_block(32).build())
    ps.append(b("e4m3 per-tensor").input(Formats.E4M3).scaling(Scaling.PER_TENSOR).build())
    return ps


@dataclass
class DotResult:
    value: float
    clamped: int


def dot_run(p: NumericPolicy, a: np.ndarray, b: np.ndarray, seed: int) -> DotResult:
    """DotSweep.run (DotSweep.java:112-122): its own Rng, per-tensor scales of
    each vector, cast a then b on the shared Rng, one dot."""
    n = a.size
    rng = Rng(0xD1F7 + seed)
    f = p.input_format
    sa = 1.0 if f is None else Quant.per_tensor_scale(f, Quant.amax(a))
    sb = 1.0 if f is None else Quant.per_tensor_scale(f, Quant.amax(b))
    qa, qb = np.empty(n), np.empty(n)
    clamped = Quant.quantize(a, 0, qa, 0, n, f, p, sa, rng)
    clamped += Quant.quantize(b, 0, qb, 0, n, f, p, sb, rng)
    out = np.empty((1, 1))
    gemm(p, 1, 1, n, qa, 0, 0, 1, qb, 0, 0, 1, out=out, rng=rng)
    return DotResult(float(out[0, 0]), clamped)


def dot_sweep(lengths: Sequence[int] = tuple(2 ** k for k in range(4, 13)), seeds: int = 200,
              policies: Optional[List[NumericPolicy]] = None, sigma: float = 1.0,
              fill=None) -> Dict:
    """The dot sweep. Returns, per policy and length, the upper median of the
    relative errors (DotSweep.java:152-153) and the mean clamps per pair.
    `fill(n, seed)` may supply the vectors (for instance the reference's own
    fill); by default they are N(0,1) x lognormal(0, sigma)."""
    policies = policies or dot_sweep_policies()
    exact_p = NumericPolicy.exact()
    table: Dict[str, Dict[int, Dict[str, float]]] = {p.name: {} for p in policies}
    rows = []
    for n in lengths:
        errs = {p.name: [] for p in policies}
        clamps = {p.name: 0 for p in policies}
        for seed in range(seeds):
            if fill is not None:
                a, b = fill(n, seed)
            else:
                rs = np.random.default_rng(seed * 7919 + n)
                a, b = heavy_tailed(rs, n, sigma), heavy_tailed(rs, n, sigma)
            ex = np.empty((1, 1))
            gemm(exact_p, 1, 1, n, a, 0, 0, 1, b, 0, 0, 1, out=ex)
            exact = float(ex[0, 0])
            for p in policies:
                r = dot_run(p, a, b, seed)
                errs[p.name].append(abs(r.value - exact) / abs(exact))
                clamps[p.name] += r.clamped
                rows.append((p.name, n, seed, r.value, exact, r.clamped))
        for p in policies:
            e = sorted(errs[p.name])
            table[p.name][n] = {"median_rel_error": e[len(e) // 2],
                                "clamped_per_pair": clamps[p.name] / seeds}
    return {"table": table, "rows": rows}


def dot_sweep_inputs_dev(lengths: Sequence[int], seeds: int, sigma: float = 1.0,
                         device: int = 0) -> Dict[int, tuple]:
    """The dot sweep's vectors for every length and seed, generated on the
    device in one seeded draw per operand: for each n, two seeds x n tensors
    of fp32 N(0,1) x lognormal(0, sigma) values held as doubles (row s is
    seed s's vector), each a contiguous block of one buffer."""
    import torch

    dev = torch.device("cuda", device)
    g = torch.Generator(device=dev)
    g.manual_seed(7919)
    total = seeds * sum(lengths)
    out = []
    for _ in range(2):
        x = torch.randn(total, device=dev, generator=g)
        x *= torch.exp(torch.randn(total, device=dev, generator=g) * sigma)
        out.append(x.double())
    blocks, off = {}, 0
    for n in lengths:
        blocks[n] = tuple(t[off:off + seeds * n].view(seeds, n) for t in out)
        off += seeds * n
    return blocks


def dot_sweep_dev(lengths: Sequence[int] = tuple(2 ** k for k in range(4, 13)),
                  seeds: int = 200, policies: Optional[List[NumericPolicy]] = None,
                  sigma: float = 1.0, device: int = 0, host_inputs: bool = False,
                  keep_inputs: bool = False) -> Dict:
    """The dot sweep on the device. The seeds' vectors are the rows of two
    seeds x n tensors and each (policy, length) is one batched contraction of
    1 x 1 dots. The casts follow DotSweep.run (DotSweep.java:112-122) per
    seed: the vector's own per-tensor scale, a then b on the seed's
    Rng(0xD1F7 + seed). Every value and clamp count lands in one device
    array, the per-(policy, length) upper medians (DotSweep.java:152-153)
    come from one launch, and everything is read back once at the end.

    Inputs are generated on the device (dot_sweep_inputs_dev), or with
    host_inputs on the host exactly as dot_sweep draws them (the same rows as
    dot_sweep then). keep_inputs returns the vectors too, for checking."""
    import torch

    from .kernel import (amax_dev, check_dev, contract_dev, contraction, per_tensor_scale_dev,
                         quantize_dev, quantize_rows_dev)
    from .stats import group_kth_rel_error_dev

    policies = policies or dot_sweep_policies()
    dev = torch.device("cuda", device)
    exact_p = NumericPolicy.exact()
    P, L = len(policies), len(lengths)
    vals = torch.empty((P + 1, L, seeds), dtype=torch.float64, device=dev)  # [0]: exact
    clamps = torch.zeros((P, L, seeds), dtype=torch.int64, device=dev)
    scal = torch.zeros(2, dtype=torch.float64, device=dev)
    kept = {}
    generated = None if host_inputs else dot_sweep_inputs_dev(lengths, seeds, sigma, device)
    for li, n in enumerate(lengths):
        if host_inputs:
            ab = []
            for seed in range(seeds):
                rs = np.random.default_rng(seed * 7919 + n)
                ab.append((heavy_tailed(rs, n, sigma), heavy_tailed(rs, n, sigma)))
            A = torch.from_numpy(np.stack([a for a, _ in ab])).to(dev)
            B = torch.from_numpy(np.stack([b for _, b in ab])).to(dev)
        else:
            A, B = generated[n]
        if keep_inputs:
            kept[n] = (A, B)
        op = contraction(batch=seeds, rows=1, cols=1, depth=n, a_batch=n, a_row=0, a_k=1,
                         b_batch=n, b_col=0, b_k=1, c_batch=1, c_row=1)
        contract_dev(exact_p, op, A, B, vals[0, li])
        qa, qb = torch.empty_like(A), torch.empty_like(B)
        for pi, p in enumerate(policies):
            f = p.input_format
            cl = clamps[pi, li]
            a, b = A, B
            if f is not None and p.input_rounding != Rounding.STOCHASTIC \
                    and p.scaling != Scaling.MX_BLOCK:
                # Every vector its own tensor: one launch per operand.
                quantize_rows_dev(p, f, p.input_rounding, A, qa, d_clamped=cl)
                quantize_rows_dev(p, f, p.input_rounding, B, qb, d_clamped=cl)
                a, b = qa, qb
            elif f is not None:
                for seed in range(seeds):
                    st = torch.tensor([0xD1F7 + seed], dtype=torch.int64, device=dev)
                    for src, dst in ((A[seed], qa[seed]), (B[seed], qb[seed])):
                        sc = None
                        if p.scaling == Scaling.PER_TENSOR:
                            amax_dev(src, scal[0:1])
                            per_tensor_scale_dev(f, scal[0:1], scal[1:2])
                            sc = scal[1:2]
                        quantize_dev(p, f, p.input_rounding, src, dst, d_scale=sc,
                                     d_rng_state=st, d_clamped=cl[seed:seed + 1])
                a, b = qa, qb
            contract_dev(p, op, a, b, vals[pi + 1, li])
    med = torch.empty((P, L), dtype=torch.float64, device=dev)
    exact_rep = vals[0:1].expand(P, L, seeds).contiguous()
    group_kth_rel_error_dev(vals[1:], exact_rep, P * L, seeds, seeds // 2, med)
    check_dev()
    v, c, m = vals.cpu().tolist(), clamps.cpu().tolist(), med.cpu().tolist()
    table: Dict[str, Dict[int, Dict[str, float]]] = {p.name: {} for p in policies}
    for pi, p in enumerate(policies):
        for li, n in enumerate(lengths):
            table[p.name][n] = {"median_rel_error": m[pi][li],
                                "clamped_per_pair": float(sum(c[pi][li])) / seeds}
    rows = [(p.name, n, seed, v[pi + 1][li][seed], v[0][li][seed], c[pi][li][seed])
            for pi, p in enumerate(policies) for li, n in enumerate(lengths)
            for seed in range(seeds)]
    out = {"table": table, "rows": rows}
    if keep_inputs:
        out["inputs"] = {n: (a.cpu().numpy(), b.cpu().numpy()) for n, (a, b) in kept.items()}
    return out


def real_dot_policies() -> List[NumericPolicy]:
    """The real-shape batch's 7 policies: FP32/FP16/BF16 sequential, FP16/BF16
    pairwise, the e4m3 per-tensor cast and the bf16 cast (from
    RealDotSweep.java:97-108)."""
    b = NumericPolicy.builder
    return [b("fp32 sequential").build(),
            b("fp16 sequential").acc(Acc.FP16).build(),
            b("bf16 sequential").acc(Acc.BF16).build(),
            b("fp16 pairwise").acc(Acc.FP16).order(Order.PAIRWISE).build(),
            b("bf16 pairwise").acc(Acc.BF16).order(Order.PAIRWISE).build(),
            b("e4m3 per-tensor cast").input(Formats.E4M3).scaling(Scaling.PER_TENSOR).build(),
            b("bf16 cast").input(Formats.BF16).build()]


def real_dot_inputs(seed: int = 424242, windows: int = 4096, units: int = 64, ctx: int = 32,
                    emb: int = 64, vocab: int = 96):
    """Synthetic stand-ins for RealDotSweep's tensors (RealDotSweep.java:78-86):
    X = windows of an N(0,1) embedding table picked by uniform tokens (64 groups
    of 64 windows); W = Kaiming-normal rows, std sqrt(2 / fan_in)."""
    rs = np.random.default_rng(seed)
    table = rs.standard_normal((vocab, emb))
    tokens = rs.integers(0, vocab, size=(windows, ctx))
    X = table[tokens].reshape(windows, ctx * emb).copy()
    W = rs.standard_normal((units, ctx * emb)) * np.sqrt(2.0 / (ctx * emb))
    return X, W


def true_median(v: np.ndarray) -> float:
    """RealDotSweep's median: the mean of the two middle values (:255-256)."""
    s = np.sort(v)
    k = s.size
    return 0.5 * (s[k // 2 - 1] + s[k // 2])


def rms(v: np.ndarray) -> float:
    """RealDotSweep.rms (:264-270)."""
    s = 0.0
    for x in v:
        s += x * x
    return float(np.sqrt(s / v.size))


def policy_outputs(p: NumericPolicy, X: np.ndarray, W: np.ndarray, rng_seed: int = 7):
    """RealDotSweep's per-policy flow (:235-254): Rng(7), per-tensor scales of
    the whole X and W, cast X then W, every (window, unit) dot."""
    f = p.input_format
    rng = Rng(rng_seed)
    qx, qw = X, W
    clamped = 0
    if f is not None:
        sx = Quant.per_tensor_scale(f, Quant.amax(X))
        sw = Quant.per_tensor_scale(f, Quant.amax(W))
        qx, qw = np.empty_like(X), np.empty_like(W)
        clamped += Quant.quantize(X, 0, qx, 0, X.size, f, p, sx, rng)
        clamped += Quant.quantize(W, 0, qw, 0, W.size, f, p, sw, rng)
    M, K = X.shape
    N = W.shape[0]
    C = gemm(p, M, N, K, qx, 0, K, 1, qw, 0, K, 1, rng=rng)
    return C, clamped


def real_dot_batch(X=None, W=None, policies=None) -> Dict[str, Dict[str, float]]:
    """The real-shape batch: per policy, the true median relative error and the
    RMS ratio over all windows x units (RealDotSweep.java:130-142)."""
    if X is None:
        X, W = real_dot_inputs()
    policies = policies or real_dot_policies()
    M, K = X.shape
    N = W.shape[0]
    exact = gemm(NumericPolicy.exact(), M, N, K, X, 0, K, 1, W, 0, K, 1).reshape(-1)
    out = {}
    for p in policies:
        C, _ = policy_outputs(p, X, W)
        got = C.reshape(-1)
        err = got - exact
        out[p.name] = {"median_rel_error": true_median(np.abs(err) / np.abs(exact)),
                       "rms_error_ratio": rms(err) / rms(exact)}
    return out


def real_dot_batch_dev(X=None, W=None, policies=None, device: int = 0) -> Dict:
    """real_dot_batch on the device: X and W cross to the GPU once; per policy
    the whole-tensor per-tensor scales, the casts of X then W on the policy's
    Rng(7) (RealDotSweep.java:119-128), the contraction, the true median of
    the relative errors (two radix selections) and the RMS sums, all on the
    device; one read-back at the end. The medians are exact order statistics
    of bit-exact outputs; the RMS ratio comes from a parallel sum, so it
    agrees with the sequential Java sum to rounding."""
    import torch

    from .kernel import (amax_dev, check_dev, error_sums_dev, gemm_dev, per_tensor_scale_dev,
                         quantize_dev)
    from .stats import RADIX_BINS, select_rel_error_dev

    if X is None:
        X, W = real_dot_inputs()
    policies = policies or real_dot_policies()
    dev = torch.device("cuda", device)
    Xd = torch.from_numpy(np.ascontiguousarray(X)).to(dev)
    Wd = torch.from_numpy(np.ascontiguousarray(W)).to(dev)
    M, K = Xd.shape
    N = Wd.shape[0]
    total = M * N
    exact = torch.empty((M, N), dtype=torch.float64, device=dev)
    gemm_dev(NumericPolicy.exact(), Xd, Wd, exact)
    C = torch.empty_like(exact)
    qx, qw = torch.empty_like(Xd), torch.empty_like(Wd)
    scal = torch.zeros(2, dtype=torch.float64, device=dev)
    P = len(policies)
    sums = torch.zeros((P, 2), dtype=torch.float64, device=dev)
    med = torch.zeros((P, 2, 2), dtype=torch.int64, device=dev)
    hist = torch.empty(RADIX_BINS, dtype=torch.int64, device=dev)
    for k, p in enumerate(policies):
        f = p.input_format
        st = torch.tensor([7], dtype=torch.int64, device=dev)
        a, b = Xd, Wd
        if f is not None:
            for src, dst in ((Xd, qx), (Wd, qw)):
                amax_dev(src, scal[0:1])
                per_tensor_scale_dev(f, scal[0:1], scal[1:2])
                quantize_dev(p, f, p.input_rounding, src, dst, d_scale=scal[1:2], d_rng_state=st)
            a, b = qx, qw
        gemm_dev(p, a, b, C, d_rng_state=st)
        error_sums_dev(C, exact, sums[k])
        select_rel_error_dev(C, exact, total // 2 - 1, med[k, 0], hist)
        select_rel_error_dev(C, exact, total // 2, med[k, 1], hist)
    check_dev()
    s, m = sums.cpu().numpy(), med[:, :, 0].cpu().numpy()
    out = {}
    for k, p in enumerate(policies):
        lo, hi = (float(np.int64(x).view(np.float64)) for x in m[k])
        out[p.name] = {"median_rel_error": 0.5 * (lo + hi),
                       "rms_error_ratio": float(np.sqrt(s[k, 0] / s[k, 1]))}
    return out


def real_dot_sweep(X=None, W=None, policies=None, rng_seed: int = 7) -> Dict:
    """RealDotSweep's whole policy loop (:235-257) in one host-buffer C-ABI
    call: X and W cross to the device once, every policy's casts, contraction,
    median and RMS sums run there, and only four numbers per policy come back:
    the true median relative error, the RMS ratio and the clamp counts of the
    casts of X and of W."""
    import ctypes

    from . import _lib

    if X is None:
        X, W = real_dot_inputs()
    policies = policies or real_dot_policies()
    X = np.ascontiguousarray(X, dtype=np.float64)
    W = np.ascontiguousarray(W, dtype=np.float64)
    M, K = X.shape
    N, K2 = W.shape
    if K2 != K:
        raise ValueError(f"X is {M}x{K} but W is {N}x{K2}")
    P = len(policies)
    pols = (_lib.DriftPolicy * max(P, 1))(*[p.to_c() for p in policies])
    stats = np.zeros((max(P, 1), 4), dtype=np.float64)
    _lib.check(_lib.load().drift_real_dot_sweep(
        _lib.Context.current().handle, ctypes.cast(pols, ctypes.c_void_p), P, M, N, K,
        X.ctypes.data, W.ctypes.data, ctypes.c_uint64(rng_seed), stats.ctypes.data))
    return {p.name: {"median_rel_error": float(stats[k, 0]),
                     "rms_error_ratio": float(stats[k, 1]),
                     "clamped_x": int(stats[k, 2]), "clamped_w": int(stats[k, 3])}
            for k, p in enumerate(policies)}


def mx_policies() -> List[NumericPolicy]:
    """The block-scaled study: e4m3 and e2m1 under per-tensor, MX spec and MX +1
    scaling, FP32 sequential accumulation (DotSweep.java:71-82's scaling group)."""
    b = NumericPolicy.builder
    ps = []
    for f in (Formats.E4M3, Formats.E2M1):
        ps.append(b(f"{f.name} per-tensor").input(f).scaling(Scaling.PER_TENSOR).build())
        ps.append(b(f"{f.name} mx32 spec").input(f).scaling(Scaling.MX_BLOCK).build())
        ps.append(b(f"{f.name} mx32 +1").input(f).scaling(Scaling.MX_BLOCK).mx_headroom(1).build())
    return ps


def mx_gemm_inputs(size: int = 4096, seed: int = 0, device: int = 0):
    """The block-scaled study's operands: A and W of size x size, fp32
    N(0,1) x lognormal(0,1) values held as doubles, the same on every rank."""
    import torch

    dev = torch.device("cuda", device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    A = (torch.randn(size, size, device=dev, generator=g) *
         torch.exp(torch.randn(size, size, device=dev, generator=g))).double()
    W = (torch.randn(size, size, device=dev, generator=g) *
         torch.exp(torch.randn(size, size, device=dev, generator=g))).double()
    return A, W


def mx_gemm(size: int = 4096, seed: int = 0, policies=None, device: int = 0, dist=None,
            inputs=None) -> Dict:
    """The block-scaled GEMM at size^3 on device-resident tensors. Per policy:
    median relative error (upper), RMS ratio, clamps per vector pair (clamps in
    row i of A plus row j of W, averaged over pairs, as DotSweep.java:119-120
    counts them) and per pair of 32-blocks.

    With a process group `dist`, the GEMMs are sharded by N-tile
    (drift_b200.dist.ntile_gemm): every rank casts all of A and its block of
    W's rows (a per-tensor scale of W from the all-reduced amax), contracts
    its block of C's columns, and only statistics cross ranks (error sums and
    W's clamp counts summed, the median's radix histograms all-reduced). The
    results are those of one GPU."""
    import torch

    from . import dist as ddist
    from .kernel import (amax_dev, check_dev, error_sums_dev, gemm_dev, per_tensor_scale_dev,
                         quantize_dev)
    from .stats import upper_median_rel_error

    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    A, W = inputs if inputs is not None else mx_gemm_inputs(size, seed, device)
    dev = A.device
    lo, hi = ddist.ntile_bounds(size, world, rank)
    Wc = W[lo:hi]
    exact = torch.empty((size, hi - lo), dtype=torch.float64, device=dev)
    ddist.ntile_gemm(NumericPolicy.exact(), A, Wc, exact)
    qa, qw = torch.empty_like(A), torch.empty_like(Wc)
    C = torch.empty_like(exact)
    scal = torch.zeros(4, dtype=torch.float64, device=dev)
    res = {}
    for p in (policies or mx_policies()):
        f = p.input_format
        cl = torch.zeros(2, dtype=torch.int64, device=dev)
        if p.scaling == Scaling.PER_TENSOR:
            amax_dev(A, scal[0:1])
            per_tensor_scale_dev(f, scal[0:1], scal[2:3])
            quantize_dev(p, f, Rounding.NEAREST_EVEN, A, qa, d_scale=scal[2:3], d_clamped=cl[0:1])
            ddist.sharded_scale(f, Wc, scal[1:2], scal[3:4], dist)
            quantize_dev(p, f, Rounding.NEAREST_EVEN, Wc, qw, d_scale=scal[3:4],
                         d_clamped=cl[1:2])
        else:
            quantize_dev(p, f, Rounding.NEAREST_EVEN, A, qa, d_clamped=cl[0:1])
            quantize_dev(p, f, Rounding.NEAREST_EVEN, Wc, qw, d_clamped=cl[1:2])
        ddist.ntile_gemm(p, qa, qw, C)
        check_dev()
        # Statistics on the engine's own kernels: the upper median by radix
        # selection, the RMS ratio from two device sums.
        sums = torch.zeros(2, dtype=torch.float64, device=dev)
        error_sums_dev(C, exact, sums)
        wcl = cl[1:2].clone()
        if dist is not None:
            dist.all_reduce(sums)
            dist.all_reduce(wcl)
        err_sq, ex_sq = (float(x) for x in sums.cpu())
        ca, cw = int(cl[0].item()), int(wcl.item())
        per_pair = ca / size + cw / size
        res[p.name] = {"median_rel_error": upper_median_rel_error(C, exact, size * size, dist),
                       "rms_error_ratio": float(np.sqrt(err_sq / ex_sq)),
                       "clamped_per_pair": per_pair,
                       "clamped_per_block_pair": per_pair / (size // 32)}
    return res


# ------------------------------------------------------------------ policy sweep

def policy_sweep_policies() -> List[NumericPolicy]:
    """RealDotSweep's policy list (RealDotSweep.java:97-108): the 9
    accumulator x order policies (blocked in chunks of 32), the bf16 cast,
    e4m3 per-tensor and e4m3 MX32, each with its cast of both operands."""
    b = NumericPolicy.builder
    ps = []
    for acc in (Acc.FP32, Acc.FP16, Acc.BF16):
        for o in (Order.SEQUENTIAL, Order.PAIRWISE, Order.BLOCKED):
            ps.append(b(f"{acc.name.lower()} {o.name.lower()}").acc(acc).order(o).acc_block(32).build())
    ps.append(b("bf16 cast").input(Formats.BF16).build())
    ps.append(b("e4m3 per-tensor cast").input(Formats.E4M3).scaling(Scaling.PER_TENSOR).build())
    ps.append(b("e4m3 mx32 cast").input(Formats.E4M3).scaling(Scaling.MX_BLOCK).build())
    return ps


def policy_sweep_inputs(size: int, seed: int, device, rows: Optional[int] = None):
    """The sweep's operands for one seed, generated on the device: A and B of
    `rows` (default `size`) x `size` doubles, each element N(0,1) x
    lognormal(0,1) with a full 53-bit significand, as Java's nextGaussian
    gives (the reference's weights and embeddings start from it). Row r of a
    larger draw equals row r of a smaller one only for the same `rows`."""
    import torch

    rows = size if rows is None else rows
    g = torch.Generator(device=device)
    g.manual_seed(1000 + seed)
    x = torch.randn(rows, size, device=device, generator=g, dtype=torch.float64)
    x *= torch.exp(torch.randn(rows, size, device=device, generator=g, dtype=torch.float64))
    y = torch.randn(rows, size, device=device, generator=g, dtype=torch.float64)
    y *= torch.exp(torch.randn(rows, size, device=device, generator=g, dtype=torch.float64))
    return x, y
