"""The stochastically rounded accumulator (Dot.round with STOCHASTIC,
java/src/main/java/io/drift/kernel/Dot.java:171-175) over whole GEMMs: the
dots share one Rng in (i, o) order and draw only for inexact sums. Outputs and
the Rng state afterwards are bit-exact against the oracle's sequential loop,
for data where every sum draws, where many sums are exact (so the draw
offsets only settle after several passes, or by the in-order fallback), and
for every order."""
import numpy as np
import pytest

from helpers import assert_bits, heavy_tailed
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def d():
    import drift_b200
    return drift_b200


def run(d, acc, order, M, N, K, A, B, seed=0x5EED, a_layout=None, bias=None):
    p = (d.NumericPolicy.builder("sr").acc(d.Acc(acc)).order(d.Order(order))
         .acc_rounding(d.Rounding.STOCHASTIC).build())
    a_rs, a_ks = a_layout or (K, 1)
    rng = d.Rng(seed)
    got = d.gemm(p, M, N, K, A, 0, a_rs, a_ks, B, 0, K, 1, bias=bias, rng=rng)
    op = O.policy(acc=acc, order=order, acc_rounding=1)
    want, st = O.gemm(op, M, N, K, A, 0, a_rs, a_ks, B, 0, K, 1, bias=bias, rng_state=seed)
    assert_bits(got, want, f"acc={acc} order={order} M={M} N={N} K={K}")
    assert rng.state() == st
    return p


@pytest.mark.parametrize("acc", [2, 3])
@pytest.mark.parametrize("order", [0, 1, 2, 3])
def test_general_doubles(d, acc, order):
    rs = np.random.default_rng(acc * 10 + order)
    for M, N, K in [(1, 1, 1), (3, 7, 33), (20, 65, 100), (64, 64, 256)]:
        run(d, acc, order, M, N, K, heavy_tailed(rs, M * K), heavy_tailed(rs, N * K))


@pytest.mark.parametrize("acc", [2, 3])
@pytest.mark.parametrize("order", [0, 2, 3])
def test_many_exact_sums(d, acc, order):
    """Small integers make many sums exact, so draw counts depend on the
    earlier draws: the offsets need several passes or the in-order walk."""
    rs = np.random.default_rng(7 + acc + order)
    M, N, K = 12, 40, 77
    A = rs.integers(-4, 5, M * K).astype(np.float64)
    B = rs.integers(-3, 4, N * K).astype(np.float64)
    B[::5] = 0.0
    run(d, acc, order, M, N, K, A, B)


def test_fp8_acc_bf16_sr_flow(d):
    """The reference's fp8-acc-bf16-sr policy (Policies.java:55-56): e4m3
    per-tensor casts, then a BF16 stochastic accumulator, on one Rng."""
    rs = np.random.default_rng(3)
    M, N, K = 32, 48, 512
    X, W = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
    p = d.policies.by_name("fp8-acc-bf16-sr")
    rng = d.Rng(99)
    f = p.input_format
    qx, qw = np.empty_like(X), np.empty_like(W)
    d.Quant.quantize(X, 0, qx, 0, X.size, f, p, d.Quant.per_tensor_scale(f, d.Quant.amax(X)), rng)
    d.Quant.quantize(W, 0, qw, 0, W.size, f, p, d.Quant.per_tensor_scale(f, d.Quant.amax(W)), rng)
    got = d.gemm(p, M, N, K, qx, 0, K, 1, qw, 0, K, 1, rng=rng)
    c = p.to_c()
    op = O.OraclePolicy(*[getattr(c, n) for n, _ in c._fields_])
    st = 99
    ox, _, st = O.quantize(op, f.id, 0, X, O.per_tensor_scale(f.id, O.amax(X)), st)
    ow, _, st = O.quantize(op, f.id, 0, W, O.per_tensor_scale(f.id, O.amax(W)), st)
    want, st = O.gemm(op, M, N, K, ox, 0, K, 1, ow, 0, K, 1, rng_state=st)
    assert_bits(got, want)
    assert rng.state() == st


def test_strided_and_bias(d):
    rs = np.random.default_rng(11)
    M, N, K = 9, 17, 50
    A = heavy_tailed(rs, M * K)
    run(d, 3, 0, M, N, K, A, heavy_tailed(rs, N * K), a_layout=(1, M), bias=heavy_tailed(rs, N))


def test_device_entry_point_advances_device_state(d):
    import torch

    rs = np.random.default_rng(5)
    M, N, K = 30, 70, 200
    A, B = heavy_tailed(rs, M * K), heavy_tailed(rs, N * K)
    p = (d.NumericPolicy.builder("sr").acc(d.Acc.BF16).acc_rounding(d.Rounding.STOCHASTIC).build())
    state = torch.tensor([1234], dtype=torch.int64, device="cuda")
    C = torch.empty((M, N), dtype=torch.float64, device="cuda")
    d.gemm_dev(p, torch.from_numpy(A.reshape(M, K)).cuda(), torch.from_numpy(B.reshape(N, K)).cuda(),
               C, d_rng_state=state)
    want, st = O.gemm(O.policy(acc=3, acc_rounding=1), M, N, K, A, 0, K, 1, B, 0, K, 1,
                      rng_state=1234)
    assert_bits(C.cpu().numpy(), want)
    assert (int(state.item()) & 0xFFFFFFFFFFFFFFFF) == st


def test_missing_rng_fails_only_when_drawing(d):
    p = (d.NumericPolicy.builder("sr").acc(d.Acc.BF16).acc_rounding(d.Rounding.STOCHASTIC).build())
    out = d.gemm(p, 2, 2, 3, np.ones(6), 0, 3, 1, np.ones(6), 0, 3, 1)  # 1, 2, 3 are exact in bf16
    assert (out == 3.0).all()
    with pytest.raises(d.DriftError) as e:
        d.gemm(p, 1, 1, 2, np.array([1.0, 1e-3]), 0, 2, 1, np.ones(2), 0, 2, 1)
    assert e.value.status == 1
