"""One tensor cast across ranks (drift_b200.dist): contiguous shards in
element order, a per-tensor scale from the all-reduced amax, and a stochastic
cast whose ranks continue one Rng stream after one all-gather of the shards'
draw counts. The shards together must equal the one-GPU cast bit for bit,
and every rank must end with the Rng state the whole cast leaves."""
import os
import socket

import numpy as np
import pytest

from helpers import heavy_tailed, opolicy
from oracle import oracle as O


@pytest.mark.parametrize("n,world,unit", [(10, 3, 1), (1000, 4, 32), (7, 5, 1), (96, 2, 37),
                                          (0, 2, 1), (65, 8, 32)])
def test_shard_bounds_cover_in_order(n, world, unit):
    from drift_b200 import dist

    b = [dist.shard_bounds(n, world, r, unit) for r in range(world)]
    assert b[0][0] == 0 and b[-1][1] == n
    for (lo, hi), (lo2, _) in zip(b, b[1:]):
        assert hi == lo2 and lo <= hi
    assert all(lo % unit == 0 or lo == n for lo, _ in b)   # empty trailing shards start at n


def test_advance_is_k_draws_of_the_stream():
    from drift_b200 import dist

    s = 0xC0FFEE
    for k in range(25):
        assert dist.advance(0xC0FFEE, k) == s
        _, s = O.rng_next_double(s)


def _gloo_rank(rank, world, port, q):
    import torch.distributed as td
    from drift_b200 import dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    td.init_process_group("gloo", rank=rank, world_size=world)
    counts, r = dist.gather_counts(10 * rank + 3, td, "cpu")
    q.put((r, counts))
    td.destroy_process_group()


def test_two_gloo_ranks_gather_counts():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got == [(0, [3, 13]), (1, [3, 13])]


def _policies(d):
    sr = d.Rounding.STOCHASTIC
    return [d.policies.by_name("mxfp4-sr"),
            d.policies.by_name("fp8").to_builder("fp8-sr").input_rounding(sr).build(),
            d.policies.by_name("fp8-mx").to_builder("mx37-sr").scale_block(37)
             .input_rounding(sr).build(),
            d.policies.by_name("fp8")]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 3, 5])
def test_shards_on_one_gpu_equal_the_whole_cast(world):
    """The protocol driven shard by shard on one GPU: count every shard, then
    cast each after the earlier shards' draws."""
    import torch
    import drift_b200 as d
    from drift_b200 import dist

    rs = np.random.default_rng(world)
    n = 300_007
    x = heavy_tailed(rs, n)
    x[::97] = 0.0
    for p in _policies(d):
        f, rm = p.input_format, p.input_rounding
        dx = torch.from_numpy(x).cuda()
        scale = 1.0
        amax = torch.zeros(1, dtype=torch.float64, device="cuda")
        d_scale = torch.zeros(1, dtype=torch.float64, device="cuda")
        if p.scaling == d.Scaling.PER_TENSOR:
            # The all-reduced amax of the shards: their maximum.
            lo_hi = [dist.shard_bounds(n, world, r, dist.shard_unit(p)) for r in range(world)]
            parts = []
            for lo, hi in lo_hi:
                d.amax_dev(dx[lo:hi], amax)
                parts.append(float(amax.item()))
            amax.fill_(max(parts))
            d.per_tensor_scale_dev(f, amax, d_scale)
            scale = float(d_scale.item())
        bounds = [dist.shard_bounds(n, world, r, dist.shard_unit(p)) for r in range(world)]
        counts = [dist.count_draws(p, f, rm, dx[lo:hi], d_scale=d_scale if scale != 1.0 else None,
                                   scale=scale) for lo, hi in bounds]
        out = torch.empty_like(dx)
        state = 0x5EED
        for r, (lo, hi) in enumerate(bounds):
            dist.cast_shard(p, f, rm, dx[lo:hi], out[lo:hi], state, sum(counts[:r]),
                            d_scale=d_scale if scale != 1.0 else None, scale=scale)
        want, _, st = O.quantize(opolicy(p), f.id, int(rm), x, scale, state)
        got = out.cpu().numpy()
        nan = np.isnan(want)
        assert (np.isnan(got) == nan).all()
        assert (got[~nan].view(np.int64) == want[~nan].view(np.int64)).all(), p.name
        assert dist.advance(state, sum(counts)) == st, p.name


def _nccl_rank(rank, world, port, q):
    import torch
    import torch.distributed as td
    import drift_b200 as d
    from drift_b200 import dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    d.Context.use_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        x = heavy_tailed(np.random.default_rng(11), 500_000)
        res = []
        for p in _policies(d):
            f, rm = p.input_format, p.input_rounding
            lo, hi = dist.shard_bounds(x.size, world, rank, dist.shard_unit(p))
            src = torch.from_numpy(x[lo:hi].copy()).cuda()
            dst = torch.empty_like(src)
            d_scale = None
            if p.scaling == d.Scaling.PER_TENSOR:
                amax = torch.zeros(1, dtype=torch.float64, device="cuda")
                d_scale = torch.zeros(1, dtype=torch.float64, device="cuda")
                dist.sharded_scale(f, src, amax, d_scale, td)
            st = dist.sharded_quantize(p, f, rm, src, dst, 0x1234, td, d_scale=d_scale)
            res.append((lo, dst.cpu().numpy(), st,
                        float(d_scale.item()) if d_scale is not None else 1.0))
        q.put((rank, res))
    finally:
        td.destroy_process_group()


@pytest.mark.gpu
def test_two_gpus_nccl():
    import torch
    import torch.multiprocessing as mp
    import drift_b200 as d

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    x = heavy_tailed(np.random.default_rng(11), 500_000)
    for k, p in enumerate(_policies(d)):
        scale = got[0][k][3]
        assert got[1][k][3] == scale
        want, _, st = O.quantize(opolicy(p), p.input_format.id, int(p.input_rounding), x, scale,
                                 0x1234)
        out = np.concatenate([got[0][k][1], got[1][k][1]])
        assert (out.view(np.int64) == want.view(np.int64)).all(), p.name
        assert got[0][k][2] == st and got[1][k][2] == st


class ThreadRanks:
    """W ranks as threads of one process: get_rank/get_world_size and an
    all_gather that waits for every rank (enough for drift_b200.dist)."""

    def __init__(self, world):
        import threading

        self.world = world
        self.local = threading.local()
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots = [None] * world

    def get_world_size(self):
        return self.world

    def get_rank(self):
        return self.local.rank

    def all_gather(self, parts, t):
        self.barrier.wait()
        self.slots[self.local.rank] = t.clone()
        self.barrier.wait()
        for i in range(self.world):
            parts[i].copy_(self.slots[i])
        self.barrier.wait()


def _run_thread_ranks(world, fn):
    import threading

    group = ThreadRanks(world)
    out, errs = [None] * world, []

    def body(r):
        group.local.rank = r
        try:
            out[r] = fn(r, group)
        except Exception as e:  # surfaced below
            errs.append(e)
            group.barrier.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    if errs:
        raise errs[0]
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("data", ["general", "exact-sums"])
@pytest.mark.parametrize("order", [0, 2, 3])
def test_sharded_gemm_with_stochastic_accumulator(data, order):
    """sharded_gemm over 3 thread-ranks on one GPU against the oracle's one
    GEMM: outputs and the final Rng state. Small integers make many sums exact,
    so the offsets take several rounds or the in-turn fallback."""
    import torch
    import drift_b200 as d
    from drift_b200 import dist

    rs = np.random.default_rng(order + 10 * (data == "general"))
    M, N, K, world = 37, 29, 41, 3
    if data == "general":
        A, B = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
    else:
        A = rs.integers(-3, 4, M * K).astype(np.float64)
        B = rs.integers(-2, 3, N * K).astype(np.float64)
    p = (d.NumericPolicy.builder("sr").acc(d.Acc.BF16).order(d.Order(order))
         .acc_rounding(d.Rounding.STOCHASTIC).build())
    want, st = O.gemm(opolicy(p), M, N, K, A, 0, K, 1, B, 0, K, 1, rng_state=777)

    def rank_fn(r, group):
        lo, hi = dist.shard_bounds(M, world, r)
        a = torch.from_numpy(A.reshape(M, K)[lo:hi].copy()).cuda()
        b = torch.from_numpy(B.reshape(N, K)).cuda()
        c = torch.empty((hi - lo, N), dtype=torch.float64, device="cuda")
        s = dist.sharded_gemm(p, a, b, c, 777, group)
        return lo, c.cpu().numpy(), s

    res = _run_thread_ranks(world, rank_fn)
    got = np.concatenate([c for _, c, _ in sorted(res, key=lambda x: x[0])])
    assert (got.view(np.int64) == want.view(np.int64)).all()
    assert all(s == st for _, _, s in res)
    if data == "exact-sums":   # exact sums draw nothing: the first guess cannot hold
        assert dist.last_gemm_rounds > 1

    # Rows in turn from the true offsets, the fallback's order, on its own.
    a_all = torch.from_numpy(A.reshape(M, K)).cuda()
    b = torch.from_numpy(B.reshape(N, K)).cuda()
    c = torch.empty((M, N), dtype=torch.float64, device="cuda")
    before = 0
    for r in range(world):
        lo, hi = dist.shard_bounds(M, world, r)
        before += dist.gemm_rows_from(p, a_all[lo:hi], b, c[lo:hi], 777, before)
    assert (c.cpu().numpy().view(np.int64) == want.view(np.int64)).all()
    assert dist.advance(777, before) == st


def _nccl_gemm_rank(rank, world, port, q):
    import torch
    import torch.distributed as td
    import drift_b200 as d
    from drift_b200 import dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    d.Context.use_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        rs = np.random.default_rng(5)
        M, N, K = 130, 70, 257
        A, B = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
        p = (d.NumericPolicy.builder("sr").acc(d.Acc.FP16).order(d.Order.PAIRWISE)
             .acc_rounding(d.Rounding.STOCHASTIC).build())
        lo, hi = dist.shard_bounds(M, world, rank)
        a = torch.from_numpy(A.reshape(M, K)[lo:hi].copy()).cuda()
        c = torch.empty((hi - lo, N), dtype=torch.float64, device="cuda")
        s = dist.sharded_gemm(p, a, torch.from_numpy(B.reshape(N, K)).cuda(), c, 99, td)
        q.put((rank, lo, c.cpu().numpy(), s))
    finally:
        td.destroy_process_group()


@pytest.mark.gpu
def test_sharded_gemm_two_gpus_nccl():
    import torch
    import torch.multiprocessing as mp
    import drift_b200 as d

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_gemm_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in procs), key=lambda x: x[1])
    for p in procs:
        p.join(timeout=120)
    rs = np.random.default_rng(5)
    M, N, K = 130, 70, 257
    A, B = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
    p = (d.NumericPolicy.builder("sr").acc(d.Acc.FP16).order(d.Order.PAIRWISE)
         .acc_rounding(d.Rounding.STOCHASTIC).build())
    want, st = O.gemm(opolicy(p), M, N, K, A, 0, K, 1, B, 0, K, 1, rng_state=99)
    got = np.concatenate([r[2] for r in res])
    assert (got.view(np.int64) == want.view(np.int64)).all()
    assert res[0][3] == st and res[1][3] == st
