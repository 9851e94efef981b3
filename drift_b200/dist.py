"""Multi-GPU sharding of the policy sweep and of single tensors.

The sweep's units are independent (policy, seed) GEMMs, so ranks never
exchange operands: each rank takes its own seeds and only the statistics are
combined, with one all-reduce of the error sums and one of the clamp counts
(NCCL on GPUs, gloo in the CPU tests). Every rank makes the same collective
calls in the same order.

One tensor can also be cast across ranks, each holding a contiguous shard in
element order. Its per-tensor scale takes one all-reduce (MAX) of the shards'
amax. A stochastic cast draws from one Rng stream in element order, so rank
r starts after the draws of shards 0..r-1: each rank counts its shard's
draws, one all-gather shares the counts, and each rank casts from the state
advanced by the earlier shards' total (k draws advance splitmix64's state by
k * golden). Every rank ends with the state the whole cast leaves, and the
shards together equal the one-GPU cast bit for bit.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import List, Optional


@dataclass(frozen=True)
class RankInfo:
    world: int
    rank: int
    local_rank: int


def rank_info() -> RankInfo:
    """RANK / LOCAL_RANK / WORLD_SIZE as torchrun sets them (1 rank if unset)."""
    return RankInfo(int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def seeds_for(rank: int, world: int, step: int, seeds_per_rank: int = 1) -> List[int]:
    """The seeds one rank owns in one step: disjoint across ranks and steps,
    so per-GPU work is fixed as ranks are added (weak scaling) and the whole
    job over `world` ranks covers seeds 0 .. world*seeds_per_rank-1 per step."""
    base = (step * world + rank) * seeds_per_rank
    return list(range(base, base + seeds_per_rank))


def init(backend: str, timeout_s: float = 600.0, device=None):
    """Joins the process group torchrun describes, with a bounded timeout so
    that ranks waiting on a lost peer fail instead of hanging."""
    import torch.distributed as dist

    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist


def reduce_stats(sums, clamps, dist) -> None:
    """Sums per-policy error sums (float64 [P, 2]) and clamp counts (int64 [P])
    over all ranks, in place."""
    if dist is None:
        return
    dist.all_reduce(sums)
    dist.all_reduce(clamps)


def max_over_ranks(value: float, dist, device=None) -> float:
    """The largest of one float across ranks (device time of the timed region)."""
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def finish(dist) -> None:
    if dist is None:
        return
    dist.barrier()
    dist.destroy_process_group()


def rms_ratio(err_sq: float, exact_sq: float) -> Optional[float]:
    """RealDotSweep's RMS ratio (RealDotSweep.java:142, :149-155) from sums."""
    import math

    if exact_sq <= 0.0:
        return None
    return math.sqrt(err_sq / exact_sq)


# ------------------------------------------------------------------ sharded casts

GOLDEN = 0x9E3779B97F4A7C15
_MASK64 = (1 << 64) - 1


def advance(state: int, draws: int) -> int:
    """The Rng state after `draws` nextLong calls (Rng.java:17-22)."""
    return (state + draws * GOLDEN) & _MASK64


def shard_bounds(n: int, world: int, rank: int, unit: int = 1):
    """Element range [lo, hi) of `rank`'s shard of n elements: contiguous, in
    element order, balanced, with boundaries on multiples of `unit` (the MX
    block length, so no block is split)."""
    units = (n + unit - 1) // unit
    per, extra = divmod(units, world)
    lo_u = rank * per + min(rank, extra)
    hi_u = lo_u + per + (1 if rank < extra else 0)
    return min(n, lo_u * unit), min(n, hi_u * unit)


def shard_unit(p) -> int:
    """Shard boundaries a cast under policy p needs (an MX block never spans two ranks)."""
    from .kernel import Scaling
    return p.scale_block if p.scaling == Scaling.MX_BLOCK else 1


def count_draws(p, f, rm, src, *, d_scale=None, scale: float = 1.0, stream=None, ctx=None) -> int:
    """The Rng draws a stochastic cast of this shard takes (0 for other roundings)."""
    import torch
    from . import _lib
    from .kernel import _stream_ptr, _tptr

    ctx = ctx or _lib.Context.current()
    out = torch.zeros(1, dtype=torch.int64, device=src.device)
    pc = p.to_c()
    import ctypes
    _lib.check(_lib.load().drift_quantize_draws_dev(
        ctx.handle, ctypes.byref(pc), f.id if f is not None else -1, int(rm), _tptr(src),
        src.numel(), _tptr(d_scale), float(scale), _tptr(out), _stream_ptr(stream)))
    return int(out.item())


def cast_shard(p, f, rm, src, dst, state: int, draws_before: int, *, d_scale=None,
               scale: float = 1.0, d_clamped=None, stream=None):
    """Casts one shard from the stream position after `draws_before` draws."""
    import torch
    from .kernel import quantize_dev

    s = advance(state, draws_before)
    d_state = torch.tensor([s - (1 << 64) if s >> 63 else s], dtype=torch.int64,
                           device=src.device)
    quantize_dev(p, f, rm, src, dst, scale=scale, d_scale=d_scale, d_rng_state=d_state,
                 d_clamped=d_clamped, stream=stream)


def sharded_scale(f, src, d_amax, d_scale, dist=None) -> None:
    """Quant.perTensorScale of the whole tensor from this rank's shard: the
    local amax, all-reduced with MAX across ranks (amax ignores NaN and is
    order-free, so this is the one-GPU amax), then the scale, on the device."""
    from .kernel import amax_dev, per_tensor_scale_dev

    amax_dev(src, d_amax)
    if dist is not None:
        dist.all_reduce(d_amax, op=dist.ReduceOp.MAX)
    per_tensor_scale_dev(f, d_amax, d_scale)


def gather_counts(mine: int, dist=None, device=None):
    """Every rank's draw count, in rank order, and this rank's index: one
    all-gather of an int64."""
    import torch

    if dist is None:
        return [mine], 0
    t = torch.tensor([mine], dtype=torch.int64, device=device)
    parts = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return [int(x.item()) for x in parts], dist.get_rank()


def sharded_quantize(p, f, rm, src, dst, state: int, dist=None, *, d_scale=None,
                     scale: float = 1.0, d_clamped=None) -> int:
    """Quant.quantize of a tensor held as one shard per rank (this rank's
    `src`, element order across ranks by rank). Returns the Rng state after
    the whole cast, the same on every rank. One all-gather of an int64."""
    mine = count_draws(p, f, rm, src, d_scale=d_scale, scale=scale)
    counts, rank = gather_counts(mine, dist, src.device)
    cast_shard(p, f, rm, src, dst, state, sum(counts[:rank]), d_scale=d_scale, scale=scale,
               d_clamped=d_clamped)
    return advance(state, sum(counts))


# ------------------------------------------------------------------ sharded GEMM

_GOLDEN_INV = pow(GOLDEN, -1, 1 << 64)  # golden is odd, so k draws are recoverable

# Rounds the last sharded_gemm on this process took (1 when the first guess
# held; max_rounds + world when it fell back to computing in turn).
last_gemm_rounds = 0


def draws_between(before: int, after: int) -> int:
    """How many draws took the Rng state from `before` to `after`."""
    return ((after - before) * _GOLDEN_INV) & _MASK64


def _signed(x: int) -> int:
    return x - (1 << 64) if x >> 63 else x


def predicted_draws(p, K: int) -> int:
    """Draws of one dot when every sum is inexact: one per rounding its order
    performs (K adds, plus the combines of Dot.pairwise's tree)."""
    from .kernel import Order

    if K <= 0:
        return 0
    if p.order != Order.PAIRWISE:
        return K

    def leaves(n):
        return 1 if n <= 8 else leaves(n >> 1) + leaves(n - (n >> 1))
    return K + leaves(K) - 1


def gemm_rows_from(p, A_rows, B, C_rows, state: int, draws_before: int, *, bias=None) -> int:
    """C_rows = the dots of A_rows against B's rows, the accumulator drawing
    from the stream position after `draws_before` draws; returns the draws
    those dots took (0 unless the accumulator is stochastic)."""
    import torch
    from .kernel import gemm_dev

    s0 = advance(state, draws_before)
    d_state = torch.tensor([_signed(s0)], dtype=torch.int64, device=A_rows.device)
    gemm_dev(p, A_rows, B, C_rows, bias=bias, d_rng_state=d_state)
    return draws_between(s0, int(d_state.item()) & _MASK64)


def stochastic_acc(p) -> bool:
    from .fmt import Rounding
    from .kernel import Acc

    return p.acc_rounding == Rounding.STOCHASTIC and p.acc in (Acc.FP16, Acc.BF16)


def sharded_gemm(p, A_rows, B, C_rows, state: int, dist=None, *, bias=None,
                 max_rounds: int = 4) -> int:
    """A GEMM sharded by row blocks: this rank holds rows [lo, hi) of A (and
    of C) in rank order, and all of B. Returns the Rng state after the whole
    GEMM, the same on every rank.

    The dots run in (i, o) order, so a rank's dots draw after every earlier
    rank's; how many draws those take depends on the draws themselves. The
    ranks therefore settle the offsets as a fixed point: each computes its
    rows from a guessed offset and recovers its true count from the state
    change, one all-gather shares the counts, and the round repeats until the
    offsets come back unchanged (then every rank used its true offset, by
    induction from rank 0's, which is always 0). The first guess — every sum
    inexact — is right unless some sum is exactly representable. After
    `max_rounds` the ranks compute in turn, each from its predecessors' true
    counts, which is right for any data."""
    global last_gemm_rounds
    if not stochastic_acc(p):
        from .kernel import gemm_dev
        gemm_dev(p, A_rows, B, C_rows, bias=bias)
        last_gemm_rounds = 1
        return state
    K, rows, N = A_rows.shape[1], A_rows.shape[0], B.shape[0]
    mine_guess = rows * N * predicted_draws(p, K)
    guesses, rank = gather_counts(mine_guess, dist, A_rows.device)
    offset = sum(guesses[:rank])
    for rnd in range(max_rounds):
        true = gemm_rows_from(p, A_rows, B, C_rows, state, offset, bias=bias)
        counts, _ = gather_counts(true, dist, A_rows.device)
        prefix = sum(counts[:rank])
        stable = all(sum(counts[:r]) == sum(guesses[:r]) for r in range(len(counts)))
        if stable:
            last_gemm_rounds = rnd + 1
            return advance(state, sum(counts))
        guesses, offset = counts, prefix
    # In turn: rank r computes once ranks 0..r-1 have published their true counts.
    world = len(guesses)
    settled = []
    for r in range(world):
        mine = gemm_rows_from(p, A_rows, B, C_rows, state, sum(settled), bias=bias) \
            if r == rank else 0
        counts, _ = gather_counts(mine, dist, A_rows.device)
        settled.append(counts[r])
    last_gemm_rounds = max_rounds + world
    return advance(state, sum(settled))


# ------------------------------------------------------------------ N-tile sharded GEMM

def ntile_bounds(N: int, world: int, rank: int, tile: int = 64):
    """Output columns [lo, hi) of `rank`'s N-tile shard: contiguous, balanced,
    on the contraction's 64-wide tile boundaries."""
    return shard_bounds(N, world, rank, tile)


def ntile_gemm(p, A, B_cols, C_cols, *, bias_cols=None) -> None:
    """One GEMM sharded by N-tile: every rank holds all of A and the rows
    [lo, hi) of B (ntile_bounds; B's rows are C's columns) and writes
    C[:, lo:hi], which `C_cols` may view inside a full C (any row stride).
    Each output is its own dot over A's row and B's row, so no operand
    crosses ranks and the contraction needs no collective; the callers reduce
    only statistics. A stochastic accumulator draws in (i, o) order, which
    interleaves the ranks' columns row by row, so it is refused here:
    sharded_gemm splits by rows and settles the draw offsets."""
    from .kernel import gemm_dev

    if stochastic_acc(p):
        raise ValueError("ntile_gemm: a stochastic accumulator draws in (i, o) order across "
                         "the column shards; use sharded_gemm (row blocks)")
    gemm_dev(p, A, B_cols, C_cols, c_rs=C_cols.stride(0), bias=bias_cols)
