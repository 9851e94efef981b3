"""GPU parity of the FP32-pipe contraction (csrc/gemm32.cu).

An FP32 accumulator over operands whose every product is an exact fp32 number
runs as one fp32 FMA per multiply-accumulate; it must still give the bits of
Dot.java's (float)(s + a*b) chain (Dot.java:50-56), its reversed walk
(:72-84) and BLOCKED's fold (:104-121). Each case also reads which path ran
(drift_gemm_route): narrow operands (bf16 casts, MX-scaled minifloats, few-bit
values down to fp32's subnormal products) take the FP32 pipe (route 1);
operands that break a condition (a 25-bit significand, a product below
2^-149, a product at 2^128, an Inf, a per-tensor scale) are scanned and stay
on the double-precision contraction (route 2); pairwise order, small calls
and chunk lengths off the k tile never scan (route 0 tiled, or 3 for a call
too thin for the tiles). Bit-exact against the oracle either way."""
import numpy as np
import pytest

from helpers import assert_bits, heavy_tailed, tiled_route
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SEQ, REV, PAIR, BLOCK = 0, 1, 2, 3


@pytest.fixture(scope="module")
def d():
    import drift_b200
    return drift_b200


def narrow(rs, n, bits, lo, hi, zeros=0.05):
    """Values of exactly `bits` significant bits (top bit set) with exponents
    uniform in [lo, hi], random signs, and a share of zeros of both signs."""
    m = rs.integers(1 << (bits - 1), 1 << bits, n).astype(np.float64)
    e = rs.integers(lo, hi + 1, n)
    v = np.ldexp(m, e - (bits - 1)) * rs.choice([-1.0, 1.0], n)
    z = rs.random(n) < zeros
    v[z] = rs.choice([0.0, -0.0], int(z.sum()))
    return v


def bf16_cast(x):
    """x cast to bf16 with the oracle (scaling NONE, nearest-even)."""
    q, _, _ = O.quantize(O.policy(input_format=O.BF16), O.BF16, 0, x)
    return q


def mx_cast(x, fmt=O.E4M3):
    q, _, _ = O.quantize(O.policy(input_format=fmt, scaling=2), fmt, 0, x)
    return q


def check(d, order, M, N, K, A, a_rs, a_ks, B, b_rs, b_ks, route, bias=None, blk=32):
    p = d.NumericPolicy.builder("t").acc(d.Acc.FP32).order(d.Order(order)).acc_block(blk).build()
    got = d.gemm(p, M, N, K, A, 0, a_rs, a_ks, B, 0, b_rs, b_ks, bias=bias)
    assert d.gemm_route() == route, f"route order={order} M={M} N={N} K={K}"
    want, _ = O.gemm(O.policy(acc=1, order=order, acc_block=blk), M, N, K, A, 0, a_rs, a_ks, B, 0,
                     b_rs, b_ks, bias=bias, threads=8)
    assert_bits(got, want, f"order={order} M={M} N={N} K={K}")
    return got


@pytest.mark.parametrize("order,blk", [(SEQ, 32), (REV, 32), (BLOCK, 32), (BLOCK, 48),
                                       (BLOCK, 4096)])
def test_bf16_operands(d, order, blk):
    rs = np.random.default_rng(11 + order + blk)
    M = N = K = 512
    A = bf16_cast(heavy_tailed(rs, M * K))
    B = bf16_cast(heavy_tailed(rs, N * K))
    check(d, order, M, N, K, A, K, 1, B, K, 1, route=1, blk=blk)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E5M2, O.E2M1])
def test_mx_operands_ragged_shape(d, fmt):
    """MX-scaled minifloats; no dimension a multiple of the 128 x 128 x 16 tile."""
    rs = np.random.default_rng(fmt)
    M, N, K = 300, 520, 1001
    A = mx_cast(heavy_tailed(rs, M * K), fmt)
    B = mx_cast(heavy_tailed(rs, N * K), fmt)
    bias = heavy_tailed(rs, N)
    for order in (SEQ, REV, BLOCK):
        check(d, order, M, N, K, A, K, 1, B, K, 1, route=1, bias=bias)


def test_strided_operands(d):
    """dgrad / wgrad layouts (Pass.java:222-232): a column-strided B, then both
    operands read down their columns."""
    rs = np.random.default_rng(3)
    M, N, K = 256, 384, 1536
    A = narrow(rs, M * K, 8, -20, 10)
    B = narrow(rs, N * K, 8, -20, 10)
    check(d, SEQ, M, N, K, A, K, 1, B, 1, N, route=1)
    check(d, SEQ, M, N, K, A, 1, M, B, 1, N, route=1)


def test_subnormal_products_and_sums(d):
    """Products down to 2^-149 and sums in fp32's subnormal range: the FMA
    keeps subnormals (no flush to zero)."""
    rs = np.random.default_rng(5)
    M = N = K = 512
    # 3-bit values: A's lowest bit >= 2^-82, B's >= 2^-66, so every product's
    # lowest bit is >= 2^-148; products lie in [2^-144, 2^-136), and 512 of
    # them sum below 2^-127, inside the subnormal range.
    A = narrow(rs, M * K, 3, -80, -77)
    B = narrow(rs, N * K, 3, -64, -61)
    got = check(d, SEQ, M, N, K, A, K, 1, B, K, 1, route=1)
    check(d, BLOCK, M, N, K, A, K, 1, B, K, 1, route=1)
    nz = np.abs(got[got != 0])
    assert nz.size and (nz < 2.0 ** -126).all(), "the sums were meant to be subnormal"


def test_overflow_to_inf_and_nan_in_blocked_fold(d):
    """Sums that overflow fp32 (Inf) and BLOCKED chunk sums of opposite
    infinities (NaN), with every product still a finite fp32 number."""
    rs = np.random.default_rng(7)
    M = N = K = 512
    # Products in [2^124, 2^126): finite fp32 numbers (62 + 62 + 2 <= 128),
    # but 32 of one sign pass FLT_MAX.
    A = narrow(rs, M * K, 4, 62, 62, zeros=0.0)
    B = narrow(rs, N * K, 4, 62, 62, zeros=0.0)
    # Row 0 of A: positive for the first 32 terms, negative after, against an
    # all-positive B row 0, so chunk 0 overflows to +Inf and chunk 1 to -Inf.
    A[:K] = np.abs(A[:K])
    A[32:K] = -A[32:K]
    B[:K] = np.abs(B[:K])
    got = check(d, BLOCK, M, N, K, A, K, 1, B, K, 1, route=1)
    assert np.isnan(got[0, 0]) and np.isinf(got).any()
    check(d, SEQ, M, N, K, A, K, 1, B, K, 1, route=1)


def test_signed_zeros(d):
    """Rows of zeros and products of -0: the FP32 chain starts at +0.0f and
    stays +0 (Dot.java:51)."""
    rs = np.random.default_rng(9)
    M = N = K = 512
    A = narrow(rs, M * K, 8, -5, 5)
    B = narrow(rs, N * K, 8, -5, 5)
    A[:K] = -0.0
    A[K:2 * K] = 0.0
    B[:K] = np.abs(B[:K])
    got = check(d, SEQ, M, N, K, A, K, 1, B, K, 1, route=1)
    assert np.signbit(got[0]).sum() == 0 and (got[0] == 0).all()


@pytest.mark.parametrize("case", ["wide", "tiny_product", "huge_product", "inf", "per_tensor",
                                  "raw"])
def test_ineligible_operands_stay_exact(d, case):
    rs = np.random.default_rng(13)
    M = N = K = 512
    A = narrow(rs, M * K, 8, -10, 10)
    B = narrow(rs, N * K, 8, -10, 10)
    if case == "wide":
        B = narrow(rs, N * K, 16, -10, 10)
        A[77] = np.ldexp(float((1 << 8) + 1), 3)          # 9 bits: 9 + 16 = 25 > 24
    elif case == "tiny_product":
        A[5] = np.ldexp(1.0, -140)                        # with B's lowest bits < 2^-149
    elif case == "huge_product":
        A[9] = np.ldexp(1.0, 120)                         # with B's 2^10: past 2^128
    elif case == "inf":
        A[100] = np.inf
    elif case == "per_tensor":
        f = O.E4M3
        x = heavy_tailed(rs, M * K)
        sa = O.per_tensor_scale(f, float(np.max(np.abs(x))))
        A, _, _ = O.quantize(O.policy(input_format=f, scaling=1), f, 0, x, sa)
    else:
        A = heavy_tailed(rs, M * K)
    # Scanned, stayed on the double-precision contraction (route 2): a call of
    # 64 tiles, which runs one output per thread.
    check(d, SEQ, M, N, K, A, K, 1, B, K, 1, route=2)


def test_pairwise_and_small_stay_on_double_path(d):
    rs = np.random.default_rng(17)
    A = bf16_cast(heavy_tailed(rs, 512 * 512))
    B = bf16_cast(heavy_tailed(rs, 512 * 512))
    # Forced to one output per thread (route 3), then to the tiled kernel.
    # Tiled calls of at least 2^27 MACs take the range proof (route 4).
    big = tiled_route(1, 512, 512, 512, A, B)
    for thin, r, rbig in ((1 << 40, 3, 3), (0, 0, big)):
        d.set_thin_tiles(thin)
        try:
            check(d, PAIR, 512, 512, 512, A, 512, 1, B, 512, 1, route=rbig)
            check(d, SEQ, 256, 256, 256, A, 256, 1, B, 256, 1, route=r)  # below 2^27 MACs
            check(d, BLOCK, 512, 512, 512, A, 512, 1, B, 512, 1, route=rbig, blk=40)  # off-tile
        finally:
            d.set_thin_tiles(-1)
    # By default pairwise over 512 x 512 outputs (64 tiles of 64 x 64) stays
    # tiled, and sequential over 256 x 256 (16 tiles) goes one output per thread.
    check(d, PAIR, 512, 512, 512, A, 512, 1, B, 512, 1, route=big)
    check(d, SEQ, 256, 256, 256, A, 256, 1, B, 256, 1, route=3)


def test_pipelined_host_call_chunks(d):
    """A host-buffer call large enough to travel in row chunks: each chunk
    runs (and scans its operands) on the FP32 pipe."""
    rs = np.random.default_rng(19)
    M, N, K = 2048, 1024, 1024
    A = mx_cast(heavy_tailed(rs, M * K))
    B = mx_cast(heavy_tailed(rs, N * K))
    check(d, SEQ, M, N, K, A, K, 1, B, K, 1, route=1)


def test_device_entry_point(d):
    import torch

    rs = np.random.default_rng(23)
    M, N, K = 512, 640, 512
    A = bf16_cast(heavy_tailed(rs, M * K))
    B = bf16_cast(heavy_tailed(rs, N * K))
    p = d.NumericPolicy.builder("t").acc(d.Acc.FP32).build()
    dA = torch.from_numpy(A.reshape(M, K)).cuda()
    dB = torch.from_numpy(B.reshape(N, K)).cuda()
    dC = torch.empty(M, N, dtype=torch.float64, device="cuda")
    d.gemm_dev(p, dA, dB, dC)
    assert d.gemm_route() == 1
    d.check_dev()
    want, _ = O.gemm(O.policy(acc=1), M, N, K, A, 0, K, 1, B, 0, K, 1, threads=8)
    assert_bits(dC.cpu().numpy(), want, "device entry")
