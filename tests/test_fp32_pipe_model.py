"""CPU check of the arithmetic behind the FP32-pipe contraction (csrc/gemm32.cu).

That kernel runs Dot.java's FP32 chain (float)(s + a*b) (Dot.java:50-56) as
fp32 fused multiply-adds when every product of the two operands is an exact
fp32 number. The claim rests on double rounding being innocuous for a sum of
two floats (53 >= 2*24 + 2). Here a plain float32 chain in numpy (each product
exact, each add rounded to nearest, subnormals kept) is held bit for bit to
the oracle's double-then-float chain on the operand shapes the kernel admits:
bf16 casts, MX-scaled minifloats, subnormal sums, and sums that overflow to
Inf (and NaN where a blocked fold meets opposite infinities). A restatement
of the kernel's admission rule (its operand scan and decision) classifies the
same operands, and the ones it must refuse."""
import numpy as np
import pytest

from helpers import heavy_tailed, same_bits
from oracle import oracle as O

M, N, K = 40, 36, 160


def narrow(rs, n, bits, lo, hi, zeros=0.05):
    """Values of exactly `bits` significant bits with exponents in [lo, hi]."""
    m = rs.integers(1 << (bits - 1), 1 << bits, n).astype(np.float64)
    e = rs.integers(lo, hi + 1, n)
    v = np.ldexp(m, e - (bits - 1)) * rs.choice([-1.0, 1.0], n)
    v[rs.random(n) < zeros] = 0.0
    return v


def scan(x):
    """The operand scan: (widest significand, largest exponent, lowest set
    bit) over the nonzero elements, or None if any is Inf or NaN."""
    x = x[x != 0]
    if not np.isfinite(x).all():
        return None
    if x.size == 0:
        return (0, None, None)
    m, e = np.frexp(np.abs(x))                      # |x| = m * 2^e, m in [0.5, 1)
    mant = (m * 2.0 ** 53).astype(np.uint64)        # 53-bit integer significand
    tz = np.zeros(mant.size, dtype=np.int64)
    for _ in range(53):
        z = (mant & np.uint64(1)) == 0
        if not z.any():
            break
        tz += z
        mant = np.where(z, mant >> np.uint64(1), mant)
    top = e - 1
    low = e - 53 + tz
    return int((top - low + 1).max()), int(top.max()), int(low.min())


def admitted(A, B):
    """The decision: both operands fp32-representable and every product an
    exact fp32 number (width sum <= 24, lowest bits >= 2^-149, below 2^128)."""
    pa, pb = scan(A), scan(B)
    if pa is None or pb is None:
        return False
    for w, top, low in (pa, pb):
        if top is not None and not (w <= 24 and low >= -149 and top <= 127):
            return False
    if pa[1] is not None and pb[1] is not None:
        return pa[0] + pb[0] <= 24 and pa[2] + pb[2] >= -149 and pa[1] + pb[1] + 2 <= 128
    return True


def f32_chain(A, B, order, blk):
    """The kernel's arithmetic: float32 products (exact here) and float32 adds."""
    a = A.reshape(M, K).astype(np.float32)
    b = B.reshape(N, K).astype(np.float32)
    assert (a.astype(np.float64) == A.reshape(M, K)).all()
    s = np.zeros((M, N), np.float32)
    tot = np.zeros((M, N), np.float32)
    ks = range(K - 1, -1, -1) if order == 1 else range(K)
    with np.errstate(all="ignore"):
        for k in ks:
            s = s + a[:, k][:, None] * b[:, k][None, :]
            if order == 3 and ((k + 1) % blk == 0 or k == K - 1):
                tot = tot + s
                s = np.zeros_like(s)
    return (tot if order == 3 else s).astype(np.float64)


def bf16(x):
    return O.quantize(O.policy(input_format=O.BF16), O.BF16, 0, x)[0]


def mx(x, fmt):
    return O.quantize(O.policy(input_format=fmt, scaling=2), fmt, 0, x)[0]


def operands(case, rs):
    if case == "bf16":
        return bf16(heavy_tailed(rs, M * K)), bf16(heavy_tailed(rs, N * K))
    if case in ("e4m3", "e2m1", "e5m2"):
        f = {"e4m3": O.E4M3, "e2m1": O.E2M1, "e5m2": O.E5M2}[case]
        return mx(heavy_tailed(rs, M * K), f), mx(heavy_tailed(rs, N * K), f)
    if case == "subnormal":   # products in [2^-144, 2^-136): fp32 subnormal sums
        return narrow(rs, M * K, 3, -80, -77), narrow(rs, N * K, 3, -64, -61)
    # overflow: products in [2^124, 2^126); row 0 of A turns sign after 32 terms
    A = narrow(rs, M * K, 4, 62, 62, zeros=0.0)
    B = narrow(rs, N * K, 4, 62, 62, zeros=0.0)
    A[:K] = np.abs(A[:K])
    A[32:K] = -A[32:K]
    B[:K] = np.abs(B[:K])
    return A, B


@pytest.mark.parametrize("case", ["bf16", "e4m3", "e2m1", "e5m2", "subnormal", "overflow"])
@pytest.mark.parametrize("order,blk", [(0, 32), (1, 32), (3, 32), (3, 48)])
def test_fp32_chain_matches_double_then_float(case, order, blk):
    rs = np.random.default_rng(sum(map(ord, case)) + 10 * order + blk)
    A, B = operands(case, rs)
    assert admitted(A, B)
    want, _ = O.gemm(O.policy(acc=1, order=order, acc_block=blk), M, N, K, A, 0, K, 1, B, 0, K, 1,
                     threads=4)
    got = f32_chain(A, B, order, blk)
    assert same_bits(got, want.reshape(M, N)).all()
    if case == "overflow" and order == 3:
        assert np.isnan(want.reshape(-1)[0]) and np.isinf(want).any()


@pytest.mark.parametrize("case", ["wide", "tiny_product", "huge_product", "inf", "per_tensor",
                                  "raw"])
def test_admission_refuses(case):
    rs = np.random.default_rng(13)
    A = narrow(rs, M * K, 8, -10, 10)
    B = narrow(rs, N * K, 8, -10, 10)
    assert admitted(A, B)
    if case == "wide":
        B = narrow(rs, N * K, 16, -10, 10)
        assert admitted(A, B)                          # 8 + 16 = 24 bits
        A[77] = np.ldexp(float((1 << 8) + 1), 3)       # 9 + 16 = 25
    elif case == "tiny_product":
        A[5] = np.ldexp(1.0, -140)                     # with B's lowest bits, below 2^-149
    elif case == "huge_product":
        A[9] = np.ldexp(1.0, 120)                      # with B's 2^10, past 2^128
    elif case == "inf":
        A[100] = np.inf
    elif case == "per_tensor":                         # a scale that is not a power of two
        x = heavy_tailed(rs, M * K)
        sa = O.per_tensor_scale(O.E4M3, float(np.max(np.abs(x))))
        A = O.quantize(O.policy(input_format=O.E4M3, scaling=1), O.E4M3, 0, x, sa)[0]
    else:
        A = heavy_tailed(rs, M * K)
    assert not admitted(A, B)
