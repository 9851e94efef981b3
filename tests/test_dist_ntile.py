"""One GEMM sharded by N-tile (drift_b200.dist.ntile_gemm): each rank holds
all of A and a block of B's rows (C's columns on 64-wide tile boundaries);
nothing but statistics crosses ranks. The column blocks together must equal
the oracle's one GEMM bit for bit, and the block-scaled study run over ranks
(sweeps.mx_gemm with a process group) must give the one-GPU statistics."""
import os
import socket

import numpy as np
import pytest

from helpers import heavy_tailed, opolicy
from oracle import oracle as O
from test_dist_shards import ThreadRanks


@pytest.mark.parametrize("N,world", [(4096, 8), (130, 3), (64, 2), (1000, 4), (5, 3)])
def test_ntile_bounds_on_tile_edges(N, world):
    from drift_b200 import dist

    b = [dist.ntile_bounds(N, world, r) for r in range(world)]
    assert b[0][0] == 0 and b[-1][1] == N
    for (lo, hi), (lo2, _) in zip(b, b[1:]):
        assert hi == lo2 and lo <= hi
    assert all(lo % 64 == 0 or lo == N for lo, _ in b)


def test_ntile_gemm_refuses_a_stochastic_accumulator():
    import drift_b200 as d
    from drift_b200 import dist

    p = (d.NumericPolicy.builder("sr").acc(d.Acc.BF16)
         .acc_rounding(d.Rounding.STOCHASTIC).build())
    with pytest.raises(ValueError, match="sharded_gemm"):
        dist.ntile_gemm(p, None, None, None)


class ReducingThreadRanks(ThreadRanks):
    """ThreadRanks with the all-reduce (SUM, MAX) and barrier the sharded
    study uses."""

    class ReduceOp:
        SUM = "sum"
        MAX = "max"

    def all_reduce(self, t, op="sum"):
        self.barrier.wait()
        self.slots[self.local.rank] = t.clone()
        self.barrier.wait()
        acc = self.slots[0].clone()
        for x in self.slots[1:]:
            acc = acc + x if op == "sum" else acc.maximum(x)
        self.barrier.wait()
        t.copy_(acc)

    def barrier_all(self):
        self.barrier.wait()


def _run(world, fn):
    """Runs fn(rank, group) on `world` threads sharing one ReducingThreadRanks."""
    import threading

    group = ReducingThreadRanks(world)
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


def _same_study(got, want):
    """Medians and clamp counts bit for bit; the RMS ratio is a sum whose
    order follows the shards, so it agrees to rounding."""
    assert got.keys() == want.keys()
    for name in want:
        g, w = got[name], want[name]
        assert g["median_rel_error"] == w["median_rel_error"], name
        assert g["clamped_per_pair"] == w["clamped_per_pair"], name
        assert g["clamped_per_block_pair"] == w["clamped_per_block_pair"], name
        assert g["rms_error_ratio"] == pytest.approx(w["rms_error_ratio"], rel=1e-12), name


def _policies(d):
    b = d.NumericPolicy.builder
    A, O_ = d.Acc, d.Order
    return [d.NumericPolicy.exact(), b("fp32").build(),
            b("fp16 pairwise").acc(A.FP16).order(O_.PAIRWISE).build(),
            b("bf16 blocked").acc(A.BF16).order(O_.BLOCKED).acc_block(32).build(),
            b("fp16 trunc").acc(A.FP16).acc_rounding(d.Rounding.TRUNCATE).build()]


@pytest.mark.gpu
def test_ntile_gemm_over_thread_ranks_matches_oracle():
    """Three thread-ranks on one GPU, each writing its column block into a
    view of one C; the assembled C against the oracle's GEMM."""
    import torch
    import drift_b200 as d
    from drift_b200 import dist

    rs = np.random.default_rng(21)
    M, N, K, world = 150, 200, 300, 3
    A, B = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
    a = torch.from_numpy(A.reshape(M, K)).cuda()
    b = torch.from_numpy(B.reshape(N, K)).cuda()
    for p in _policies(d):
        want, _ = O.gemm(opolicy(p), M, N, K, A, 0, K, 1, B, 0, K, 1, threads=8)
        C = torch.full((M, N), np.nan, dtype=torch.float64, device="cuda")

        def rank_fn(r, group):
            lo, hi = dist.ntile_bounds(N, world, r)
            dist.ntile_gemm(p, a, b[lo:hi], C[:, lo:hi])
            torch.cuda.synchronize()

        _run(world, rank_fn)
        got = C.cpu().numpy()
        assert (got.view(np.int64) == want.view(np.int64)).all(), p.name


@pytest.mark.gpu
def test_block_scaled_study_over_thread_ranks_equals_one_gpu():
    import torch
    from drift_b200 import sweeps

    size, world = 512, 3
    inputs = sweeps.mx_gemm_inputs(size, 4, 0)
    one = sweeps.mx_gemm(size, inputs=inputs)

    def rank_fn(r, group):
        return sweeps.mx_gemm(size, inputs=inputs, dist=group)

    res = _run(world, rank_fn)
    for r in res:
        _same_study(r, one)


def _nccl_rank(rank, world, port, q):
    import torch
    import torch.distributed as td
    import drift_b200 as d
    from drift_b200 import dist, sweeps

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    d.Context.use_device(rank)
    td.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        rs = np.random.default_rng(22)
        M, N, K = 190, 300, 257
        A, B = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
        a = torch.from_numpy(A.reshape(M, K)).cuda()
        b = torch.from_numpy(B.reshape(N, K)).cuda()
        lo, hi = dist.ntile_bounds(N, world, rank)
        out = []
        for p in _policies(d):
            c = torch.empty((M, hi - lo), dtype=torch.float64, device="cuda")
            dist.ntile_gemm(p, a, b[lo:hi], c)
            out.append(c.cpu().numpy())
        study = sweeps.mx_gemm(512, inputs=sweeps.mx_gemm_inputs(512, 4, rank), dist=td,
                               device=rank)
        q.put((rank, lo, out, study))
    finally:
        td.destroy_process_group()


@pytest.mark.gpu
def test_ntile_two_gpus_nccl():
    import torch
    import torch.multiprocessing as mp
    import drift_b200 as d
    from drift_b200 import sweeps

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
    res = sorted((q.get(timeout=300) for _ in procs), key=lambda x: x[1])
    for p in procs:
        p.join(timeout=120)
    rs = np.random.default_rng(22)
    M, N, K = 190, 300, 257
    A, B = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
    for k, p in enumerate(_policies(d)):
        want, _ = O.gemm(opolicy(p), M, N, K, A, 0, K, 1, B, 0, K, 1, threads=8)
        got = np.concatenate([r[2][k] for r in res], axis=1)
        assert (got.view(np.int64) == want.view(np.int64)).all(), p.name
    one = sweeps.mx_gemm(512, inputs=sweeps.mx_gemm_inputs(512, 4, 0))
    _same_study(res[0][3], one)
    _same_study(res[1][3], one)
