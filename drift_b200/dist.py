"""Multi-GPU sharding of the policy sweep and the reduction of its statistics.

The sweep's units are independent (policy, seed) GEMMs, so ranks never
exchange operands: each rank takes its own seeds and only the statistics are
combined, with one all-reduce of the error sums and one of the clamp counts
(NCCL on GPUs, gloo in the CPU tests). Every rank makes the same collective
calls in the same order.
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
    """RealDotSweep's RMS ratio (RealDotSweep.java:257, :264-270) from sums."""
    import math

    if exact_sq <= 0.0:
        return None
    return math.sqrt(err_sq / exact_sq)
