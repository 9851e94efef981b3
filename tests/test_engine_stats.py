"""Order statistics of the relative error on the device (radix selection),
against numpy's sort; and across two ranks, where the histograms are summed
between passes so the selection runs over the union of both ranks' outputs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def java_sorted_rel(got, exact):
    with np.errstate(all="ignore"):
        rel = np.abs(got - exact) / np.abs(exact)
    # Java's Arrays.sort(double[]) puts NaN after +Inf.
    return np.concatenate([np.sort(rel[~np.isnan(rel)]), rel[np.isnan(rel)]])


def make(n, seed):
    rs = np.random.default_rng(seed)
    exact = rs.standard_normal(n) * np.exp(rs.standard_normal(n) * 2)
    got = exact * (1 + rs.standard_normal(n) * 1e-3)
    got[::97] = exact[::97]             # zero error
    exact[5::1009] = 0.0                # x / 0 = inf
    got[5::2018] = 0.0                  # 0 / 0 = nan
    return got, exact


def test_kth_relative_error_matches_sort():
    import torch
    from drift_b200 import stats

    got, exact = make(200_003, 1)
    want = java_sorted_rel(got, exact)
    g, e = torch.from_numpy(got).cuda(), torch.from_numpy(exact).cuda()
    for k in [0, 1, 17, 1000, want.size // 2 - 1, want.size // 2, want.size - 3, want.size - 1]:
        v = stats.kth_rel_error(g, e, k)
        assert (np.isnan(v) and np.isnan(want[k])) or v == want[k], k
    n = want.size
    assert stats.true_median_rel_error(g, e, n) == 0.5 * (want[n // 2 - 1] + want[n // 2])
    # Errors that nearly all share their top digits (and many exactly equal):
    # whole warps add to one histogram bin at once.
    rs = np.random.default_rng(2)
    exact = rs.standard_normal(300_001)
    got = exact * (1 + 2.0 ** -10)
    got[::3] = exact[::3] * (1 + 2.0 ** -11)
    want = java_sorted_rel(got, exact)
    g, e = torch.from_numpy(got).cuda(), torch.from_numpy(exact).cuda()
    for k in [0, 99_999, 100_000, 100_001, 150_000, want.size - 1]:
        assert stats.kth_rel_error(g, e, k) == want[k], k


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch
    from drift_b200 import dist as ddist, stats

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK="0")
    pg = ddist.init("gloo", timeout_s=120)
    got, exact = make(50_001 + 1000 * rank, 10 + rank)
    g, e = torch.from_numpy(got).cuda(), torch.from_numpy(exact).cuda()
    total = 50_001 * world + 1000 * (world * (world - 1) // 2)
    out[rank] = stats.upper_median_rel_error(g, e, total, dist=pg)
    ddist.finish(pg)


def test_union_median_over_two_ranks():
    import torch.multiprocessing as mp

    world = 2
    with mp.get_context("spawn").Manager() as m:  # no fork after CUDA use
        out = m.dict()
        mp.spawn(_rank, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    parts = [make(50_001 + 1000 * r, 10 + r) for r in range(world)]
    want = java_sorted_rel(np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts]))
    assert res[0] == res[1] == want[want.size // 2]
