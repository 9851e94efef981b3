"""The batched, ragged and causal contractions (drift_contract): the four
attention matmul loops of AttnPass.java:245-290 and :373-427, with the score
scale and dInput's accumulation, for every accumulator, order and
accumulator rounding (stochastic included). Outputs and the Rng state are
bit-exact against the oracle's loops."""
import numpy as np
import pytest

from helpers import assert_bits, heavy_tailed, opolicy
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def d():
    import drift_b200
    return drift_b200


def attention_ops(d, B, t, dim, scale):
    """(name, op, A size, B size, C size) of the AttnPass loops."""
    W = d.Window
    return [
        ("scores", d.contraction(batch=B, rows=t, cols=t, depth=dim, a_batch=t * dim, a_row=dim,
                                 a_k=1, b_batch=t * dim, b_col=dim, b_k=1, c_batch=t * t,
                                 c_row=t, alpha=scale, causal=True),
         B * t * dim, B * t * dim, B * t * t),
        ("context", d.contraction(batch=B, rows=t, cols=dim, depth=t, a_batch=t * t, a_row=t,
                                  a_k=1, b_batch=t * dim, b_col=1, b_k=dim, c_batch=t * dim,
                                  c_row=dim, window=W.PREFIX),
         B * t * t, B * t * dim, B * t * dim),
        ("dprob", d.contraction(batch=B, rows=t, cols=t, depth=dim, a_batch=t * dim, a_row=dim,
                                a_k=1, b_batch=t * dim, b_col=dim, b_k=1, c_batch=t * t,
                                c_row=t, causal=True),
         B * t * dim, B * t * dim, B * t * t),
        ("dv", d.contraction(batch=B, rows=t, cols=dim, depth=t, a_batch=t * t, a_row=1, a_k=t,
                             b_batch=t * dim, b_col=1, b_k=dim, c_batch=t * dim, c_row=dim,
                             window=W.SUFFIX),
         B * t * t, B * t * dim, B * t * dim),
    ]


def run(d, p, op, A, B, C0, seed=None):
    rng = d.Rng(seed) if seed is not None else None
    got = d.contract(p, op, A, B, C0.copy(), rng=rng)
    want = C0.copy()
    st = O.contract(opolicy(p), op, A, B, want, seed)
    return got, want, (rng.state() if rng else None), st


POLICIES = [(a, o, r) for a in range(4) for o in range(4)
            for r in ([0, 1, 2] if a >= 2 else [0])]


@pytest.mark.parametrize("acc,order,rm", POLICIES)
def test_attention_loops(d, acc, order, rm):
    rs = np.random.default_rng(acc * 100 + order * 10 + rm)
    p = (d.NumericPolicy.builder("c").acc(d.Acc(acc)).order(d.Order(order))
         .acc_rounding(d.Rounding(rm)).acc_block(5).build())
    for B, t, dim in [(3, 11, 13), (1, 1, 1), (2, 20, 3)]:
        for name, op, na, nb, nc in attention_ops(d, B, t, dim, 1.0 / np.sqrt(dim)):
            A, Bm = heavy_tailed(rs, na), heavy_tailed(rs, nb)
            got, want, s1, s2 = run(d, p, op, A, Bm, np.full(nc, 7.0), seed=12345)
            assert_bits(got, want, f"{name} B={B} t={t} d={dim}")
            assert s1 == s2


@pytest.mark.parametrize("order,blk", [(0, 32), (1, 32), (2, 32), (3, 32), (3, 48), (3, 64)])
@pytest.mark.parametrize("acc,rm", [(0, 0), (1, 0), (2, 0), (3, 0), (2, 2), (3, 2)])
def test_long_ragged_windows(d, acc, rm, order, blk):
    """Windows up to 150 terms: deep, uneven pairwise trees per row, and the
    staged chunk walk's windows that start and end inside 32-term chunks."""
    rs = np.random.default_rng(acc + 7 * order + 13 * rm + blk)
    p = (d.NumericPolicy.builder("c").acc(d.Acc(acc)).order(d.Order(order)).acc_block(blk)
         .acc_rounding(d.Rounding(rm)).build())
    for name, op, na, nb, nc in attention_ops(d, 2, 150, 4, 0.5):
        if name in ("context", "dv"):
            got, want, _, _ = run(d, p, op, heavy_tailed(rs, na), heavy_tailed(rs, nb),
                                  np.zeros(nc))
            assert_bits(got, want, name)


@pytest.mark.parametrize("acc", [2, 3])
def test_stochastic_with_many_exact_sums(d, acc):
    """Small integers make sums exact, so offsets need extra passes."""
    rs = np.random.default_rng(acc)
    p = (d.NumericPolicy.builder("c").acc(d.Acc(acc)).acc_rounding(d.Rounding.STOCHASTIC)
         .order(d.Order.PAIRWISE).build())
    for name, op, na, nb, nc in attention_ops(d, 4, 17, 9, 0.25):
        A = rs.integers(-3, 4, na).astype(np.float64)
        Bm = rs.integers(-2, 3, nb).astype(np.float64) * 0.37
        got, want, s1, s2 = run(d, p, op, A, Bm, np.zeros(nc), seed=99)
        assert_bits(got, want, name)
        assert s1 == s2


@pytest.mark.parametrize("rm", [0, 1])
def test_accumulate_into_c(d, rm):
    """dInput's dx += dot (AttnPass.java:478-484), with a strided C."""
    rs = np.random.default_rng(4)
    p = (d.NumericPolicy.builder("c").acc(d.Acc.BF16).acc_rounding(d.Rounding(rm)).build())
    op = d.contraction(rows=9, cols=6, depth=40, a_row=40, a_k=1, b_col=1, b_k=6, c_row=8,
                       c_off=3, accumulate=True)
    A, Bm = heavy_tailed(rs, 360), heavy_tailed(rs, 240)
    C0 = heavy_tailed(rs, 3 + 8 * 9)
    got, want, s1, s2 = run(d, p, op, A, Bm, C0, seed=5 if rm else None)
    assert_bits(got, want)
    assert s1 == s2


def test_device_entry_point(d):
    import torch

    rs = np.random.default_rng(8)
    p = (d.NumericPolicy.builder("c").acc(d.Acc.FP16).acc_rounding(d.Rounding.STOCHASTIC)
         .build())
    name, op, na, nb, nc = attention_ops(d, 5, 12, 7, 0.3)[3]
    A, Bm = heavy_tailed(rs, na), heavy_tailed(rs, nb)
    state = torch.tensor([77], dtype=torch.int64, device="cuda")
    dC = torch.zeros(nc, dtype=torch.float64, device="cuda")
    d.contract_dev(p, op, torch.from_numpy(A).cuda(), torch.from_numpy(Bm).cuda(), dC,
                   d_rng_state=state)
    want = np.zeros(nc)
    st = O.contract(opolicy(p), op, A, Bm, want, 77)
    assert_bits(dC.cpu().numpy(), want)
    assert (int(state.item()) & 0xFFFFFFFFFFFFFFFF) == st


def test_bad_contractions_are_rejected(d):
    p = d.NumericPolicy.builder("c").build()
    ok = dict(rows=3, cols=3, depth=4, a_row=4, a_k=1, b_col=4, b_k=1, c_row=3)
    A, Bm = np.ones(12), np.ones(12)
    d.contract(p, d.contraction(**ok), A, Bm, np.zeros(9))
    bad = [
        (dict(ok, depth=5), np.zeros(9)),                        # A and B too short
        (dict(ok), np.zeros(8)),                                 # C too short
        (dict(ok, rows=5, a_row=0, window=d.Window.PREFIX), np.zeros(15)),  # rows > depth
        (dict(ok, a_off=-1), np.zeros(9)),
    ]
    for kw, C in bad:
        with pytest.raises(d.DriftError) as e:
            d.contract(p, d.contraction(**kw), A, Bm, C)
        assert e.value.status == 1
    op = d.contraction(**ok)
    op.window = 7
    with pytest.raises(d.DriftError):
        d.contract(p, op, A, Bm, np.zeros(9))


@pytest.mark.parametrize("acc,order", [(a, o) for a in range(4) for o in range(4)])
def test_full_windows_through_the_tiled_kernel(d, acc, order):
    """Scores and dProb with an even depth: the batch runs as one tiled TMA
    launch whose tiles read past each problem's last row into the next
    problem (t = 70 is not a multiple of the 64-row tile), then the causal
    mask and the score scale are applied."""
    rs = np.random.default_rng(31 * acc + order)
    p = d.NumericPolicy.builder("c").acc(d.Acc(acc)).order(d.Order(order)).acc_block(16).build()
    for B, t, dim in [(3, 70, 16), (2, 128, 64), (5, 33, 40)]:
        for name, op, na, nb, nc in attention_ops(d, B, t, dim, 0.3)[::2]:   # scores, dprob
            got, want, _, _ = run(d, p, op, heavy_tailed(rs, na), heavy_tailed(rs, nb),
                                  np.full(nc, 3.0))
            assert_bits(got, want, f"{name} B={B} t={t} d={dim}")
