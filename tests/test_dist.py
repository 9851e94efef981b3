"""The multi-rank host logic of the sweep on CPU: two gloo ranks reduce their
statistics exactly as the NCCL ranks of bench.py do, and seeds never overlap."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from drift_b200 import dist as ddist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    info = ddist.rank_info()
    assert (info.rank, info.world) == (rank, world)
    pg = ddist.init("gloo", timeout_s=60)
    P = 12
    sums = torch.full((P, 2), float(rank + 1), dtype=torch.float64)
    clamps = torch.arange(P, dtype=torch.int64) * (rank + 1)
    ddist.reduce_stats(sums, clamps, pg)
    mx = ddist.max_over_ranks(10.0 * (rank + 1), pg)
    out[rank] = (sums.tolist(), clamps.tolist(), mx)
    ddist.finish(pg)


def test_two_gloo_ranks_reduce_statistics():
    world = 2
    with mp.get_context("spawn").Manager() as m:  # no fork after CUDA use
        out = m.dict()
        mp.spawn(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    for rank in range(world):
        sums, clamps, mx = res[rank]
        assert all(v == [3.0, 3.0] for v in sums)          # 1 + 2 on every policy
        assert clamps == [3 * k for k in range(12)]
        assert mx == 20.0


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_seeds_are_disjoint_and_cover_the_sweep(world):
    seen = set()
    for step in range(3):
        for rank in range(world):
            s = ddist.seeds_for(rank, world, step, seeds_per_rank=2)
            assert not (seen & set(s))
            seen |= set(s)
    assert seen == set(range(3 * world * 2))


def test_rms_ratio():
    assert ddist.rms_ratio(4.0, 16.0) == 0.5
    assert ddist.rms_ratio(1.0, 0.0) is None
