"""CPU models of two device arithmetic forms, pinned against the oracle.

1. The tiled contraction's fast accumulator rounding (FastForm in codec.cuh):
   r = fma(D, -2^S, fma(D, 2^S, t)) with D = 1.5 * 2^e built from t's high
   word and the previous accumulator value's low word, validated by one
   unsigned running max of t's exponent word. On every sum the validation
   admits, the result must equal Dot.round / (float) (Dot.java:54, :63,
   :141-182), ties included, for every low word an accumulator can hold.

2. The cast's value-domain form (quantize_value in codec.cuh): decode(encode(s))
   computed as min(round(|s| * 2^(mant-e)) * 2^(e-mant), maxFinite) with the
   sign, for every format, rounding mode and special value, with stochastic
   rounding drawing for exactly the elements MiniFloat.encode draws for
   (MiniFloat.java:156-221, :258-278).

Each model is a numpy restatement of the device code's steps; fma(D, 2^S, t)
is an exact product plus one rounded add, so numpy's float64 add restates it.
"""
import numpy as np
import pytest

from helpers import range_limit, range_proven
from oracle import oracle as O


def _pow2(k):
    return ((np.asarray(k, dtype=np.int64) + 1023) << 52).view(np.float64)


# ------------------------------------------------------------------ accumulator rounding

def _fast_round(t, prev_lo, shift, lo_e, hi_e, trunc=False):
    hi = (t.view(np.uint64) >> np.uint64(32)).astype(np.uint32)
    dh = (hi & np.uint32(0x7FF00000)) | np.uint32(0x00080000)
    run = (dh - np.uint32((lo_e << 20) | 0x80000)).astype(np.uint32)     # wraps below lo_e
    valid = run <= np.uint32((hi_e - lo_e) << 20)
    if trunc:
        mask = np.uint32(~((1 << (shift - 32)) - 1) & 0xFFFFFFFF)
        bits = ((hi & mask).astype(np.uint64) << np.uint64(32)) | prev_lo.astype(np.uint64)
        return bits.view(np.float64), valid
    d = ((dh.astype(np.uint64) << np.uint64(32)) | prev_lo.astype(np.uint64)).view(np.float64)
    c = d * float(2 ** shift)                  # exact: a power-of-two scaling
    with np.errstate(all="ignore"):
        return (c + t) - c, valid               # one rounding, then an exact subtraction


def _sums(rs, n, shift, e_lo, e_hi):
    """Doubles across and beyond the accumulator's range, a third of them
    exact ties at the target precision and a third within a few ulps of one."""
    e = rs.integers(e_lo, e_hi, n)
    m = rs.integers(0, 1 << 52, n, dtype=np.int64)
    k = n // 3
    m[:k] = (m[:k] >> shift << shift) | (1 << (shift - 1))
    m[k:2 * k] = ((m[k:2 * k] >> shift << shift) | (1 << (shift - 1))) + rs.integers(-3, 4, k)
    m &= (1 << 52) - 1
    t = np.ldexp(1.0 + m / 2.0 ** 52, e) * np.where(rs.random(n) < 0.5, -1.0, 1.0)
    t[:64] = 0.0
    t[64:70] = [np.inf, -np.inf, np.nan, 5e-324, -1e-310, 1e300]
    return t


@pytest.mark.parametrize("acc", ["fp32", "fp16", "bf16"])
def test_fast_accumulator_rounding_matches_oracle(acc):
    rs = np.random.default_rng(11)
    n = 600_000
    if acc == "fp32":
        shift, lo_e, hi_e = 29, 1023 - 126, 1023 + 126
        t = _sums(rs, n, shift, -150, 130)
        # Any float's low word: 0 or a multiple of 2^29.
        prev_lo = rs.integers(0, 8, n).astype(np.uint32) << np.uint32(29)
        with np.errstate(over="ignore"):
            want = {0: t.astype(np.float32).astype(np.float64)}
    else:
        acc_id = 2 if acc == "fp16" else 3
        mant, min_e, max_e = (10, -14, 15) if acc == "fp16" else (7, -126, 127)
        shift, lo_e, hi_e = 52 - mant, 1023 + min_e, 1023 + max_e - 1
        t = _sums(rs, n, shift, min_e - 10, max_e + 3)
        prev_lo = np.zeros(n, np.uint32)            # FP16/BF16 values have a zero low word
        want = {0: O.acc_round(acc_id, O.NEAREST_EVEN, t)[0],
                2: O.acc_round(acc_id, O.TRUNCATE, t)[0]}
    for rm, w in want.items():
        got, valid = _fast_round(t, prev_lo, shift, lo_e, hi_e, trunc=rm == 2)
        bad = valid & (got.view(np.int64) != w.view(np.int64))
        assert not bad.any(), (acc, rm, t[bad][:3])
        # The fast form takes nearly every in-range sum; zero, Inf, NaN and
        # the subnormal range are always refused.
        assert valid.mean() > 0.6
        assert not valid[:70].any()


# ------------------------------------------------------------------ cast values

def _quantize_value(fmt, s, rm, u=None):
    maxf, minn, minsub, _ = O.format_info(fmt)
    mant = int(round(np.log2(minn / minsub)))
    min_e = int(round(np.log2(minn)))
    a = np.abs(s)
    e = ((a.view(np.uint64) >> np.uint64(52)) & np.uint64(0x7FF)).astype(np.int64) - 1023
    e = np.minimum(np.maximum(e, min_e), 1023)
    drew = np.zeros(s.size, bool)
    with np.errstate(all="ignore"):
        sc = a * _pow2(mant - e)
        if rm == O.NEAREST_EVEN:
            m = (sc + 2.0 ** 52) - 2.0 ** 52
        else:
            m = np.floor(sc)
            if rm == O.STOCHASTIC:
                frac = sc - m
                drew = (frac != 0) & (a < np.inf)
                m = np.where(drew & (u < frac), m + 1, m)
        q = np.copysign(np.fmin(m * _pow2(e - mant), maxf), s)
    return np.where(np.isnan(s), np.nan, q), drew


def _cast_inputs(rs, fmt):
    maxf, _, _, width = O.format_info(fmt)
    x = rs.standard_normal(200_000) * np.exp(rs.standard_normal(200_000) * 3) * maxf / 8
    codes = (np.arange(1 << width, dtype=np.int32) if width <= 16
             else rs.integers(0, 1 << 16, 20_000).astype(np.int32))
    v = np.abs(O.decode(fmt, codes))
    v = np.unique(v[np.isfinite(v)])
    mids = (v[1:] + v[:-1]) / 2
    return np.concatenate([x, v, -v, mids, -mids, np.nextafter(mids, 0), np.nextafter(mids, 9e9),
                           [0.0, -0.0, 5e-324, -1e-310, 1e300, -1e300, np.inf, -np.inf, maxf,
                            maxf * 1.0001, 2 * maxf, -2 * maxf]])


@pytest.mark.parametrize("fmt", range(7))
def test_value_domain_cast_matches_oracle(fmt):
    rs = np.random.default_rng(100 + fmt)
    x = _cast_inputs(rs, fmt)
    if fmt not in (O.E2M1, O.E3M2, O.E2M3):          # formats with NaN
        x = np.concatenate([x, [np.nan, -np.nan]])
    for rm in (O.NEAREST_EVEN, O.TRUNCATE):
        want, _, _ = O.quantize(O.policy(input_format=fmt), fmt, rm, x, 1.0)
        got, _ = _quantize_value(fmt, x, rm)
        same = (got.view(np.int64) == want.view(np.int64)) | (np.isnan(got) & np.isnan(want))
        assert same.all(), (fmt, rm, x[~same][:3])
    # Stochastic rounding: the model draws for the same elements, in order,
    # and the Rng ends in the same state.
    x = x[np.isfinite(x) | np.isinf(x)][:60_000]
    _, drew = _quantize_value(fmt, x, O.STOCHASTIC, np.zeros(x.size))
    u = np.zeros(x.size)
    st = 0x5EED
    for i in np.flatnonzero(drew):
        u[i], st = O.rng_next_double(st)
    got, _ = _quantize_value(fmt, x, O.STOCHASTIC, u)
    want, _, want_st = O.quantize(O.policy(input_format=fmt, input_rounding=O.STOCHASTIC), fmt,
                                  O.STOCHASTIC, x, 1.0, 0x5EED)
    assert st == want_st
    assert (got.view(np.int64) == want.view(np.int64)).all()


# ------------------------------------------------------------------ stochastic accumulator

def _sr_round_bits(x, acc, state):
    """Dot.round(x, acc, STOCHASTIC, rng) on x's bit pattern, the form the
    stochastic-accumulator kernels use for sums in the accumulator's normal
    range below its top binade: with S dropped significand bits, the draw is
    taken only when those bits are non-zero, nextDouble() < frac is
    (mix >>> (64 - S)) < dropped, and rounding up adds 1 at bit S. Returns
    (value or None when the sum needs the general form, new state)."""
    import ctypes

    mant, min_e, max_e = (10, -14, 15) if acc == O.ACC_FP16 else (7, -126, 127)
    S = 52 - mant
    bits = int(np.float64(x).view(np.uint64))
    E = (bits >> 52) & 0x7FF
    if not (1023 + min_e <= E <= 1023 + max_e - 1):
        return None, state
    dropped = bits & ((1 << S) - 1)
    r = bits - dropped
    if dropped:
        st = ctypes.c_uint64(state)
        mix = O.lib().o_rng_next_long(ctypes.byref(st))
        state = st.value
        if (mix >> (64 - S)) < dropped:
            r += 1 << S
    return float(np.uint64(r).view(np.float64)), state


@pytest.mark.parametrize("acc", [O.ACC_FP16, O.ACC_BF16])
def test_bit_pattern_stochastic_rounding_matches_oracle(acc):
    rs = np.random.default_rng(31 + acc)
    n = 20_000
    mant, min_e, max_e = (10, -14, 15) if acc == O.ACC_FP16 else (7, -126, 127)
    x = np.ldexp(rs.random(n) + 1.0, rs.integers(min_e - 3, max_e + 2, n))
    x *= np.where(rs.random(n) < 0.5, -1.0, 1.0)
    # Values with no dropped bits (no draw) and with a single low bit set.
    x[::7] = np.ldexp(rs.integers(1 << mant, 1 << (mant + 1), x[::7].size), -mant)
    x[3::11] = np.nextafter(x[3::11], np.inf)
    state, taken = 0xC0FFEE, 0
    for v in x:
        got, s2 = _sr_round_bits(v, acc, state)
        want, w2 = O.acc_round(acc, O.STOCHASTIC, np.array([v]), state)
        if got is None:        # the general form's range: skip, keep the streams aligned
            state = w2
            continue
        taken += 1
        assert np.float64(got).view(np.int64) == want.view(np.int64)[0], v
        assert s2 == w2, v
        state = s2
    assert taken > n // 2


# ------------------------------------------------------------------ range proof

def _range_limit(acc, K):
    return range_limit(acc == O.ACC_BF16, K)


def _range_proven(acc, a, b, K):
    return range_proven(acc == O.ACC_BF16, a, b, K)


def _proven_operands(rs, n, k, lo, hi, cancel=True):
    """n rows of k terms, nonzero magnitudes in [2^lo, 2^hi), a tenth zeros.
    With `cancel`, every odd term of half the rows repeats its even
    neighbour's product negated, so those partial sums fall back to rounding
    residues again and again (the low side's worst case)."""
    def draw():
        e = rs.integers(lo, hi, (n, k))
        return np.ldexp(1.0 + rs.random((n, k)), e) * np.where(rs.random((n, k)) < 0.5, -1.0, 1.0)
    a, b = draw(), draw()
    if cancel:
        h = n // 2
        a[:h, 1::2] = a[:h, 0::2]
        b[:h, 1::2] = -b[:h, 0::2]
    a[rs.random((n, k)) < 0.05] = 0.0
    b[rs.random((n, k)) < 0.05] = 0.0
    return a, b


def _fast_chain_step(acc_id, t, prev_lo):
    shift = 29 if acc_id == O.ACC_FP32 else 45
    return _fast_round(t, prev_lo, shift, 1023 - 126, 1023 + 126)


def _lo_word(x):
    return (x.view(np.uint64) & np.uint64(0xFFFFFFFF)).astype(np.uint32)


@pytest.mark.parametrize("acc", [O.ACC_FP32, O.ACC_BF16])
@pytest.mark.parametrize("case", ["low", "high"])
def test_range_proof_keeps_every_sum_exact(acc, case):
    """Under the range proof's bounds, the unchecked fast rounding equals
    Dot.round at every step of sequential chains and of pairwise trees
    (leaves of 8, Dot.java:86-102): every sum is in the fast form's range or
    is +0, which the fast form also returns."""
    rs = np.random.default_rng(77 + acc + (case == "high"))
    K = 512
    lo, hi = (-37, 8) if case == "low" else (40, 56)
    a, b = _proven_operands(rs, 600, K, lo, hi, cancel=case == "low")
    if case == "high":
        b = np.abs(b) * np.sign(a + (a == 0))       # every product >= 0: sums grow
    assert _range_proven(acc, a, b, K)
    prods = a * b

    def check_round(t, prev_lo):
        got, valid = _fast_chain_step(acc, t, prev_lo)
        if acc == O.ACC_FP32:
            want = t.astype(np.float32).astype(np.float64)     # Java's (float)
        else:
            want = O.acc_round(acc, O.NEAREST_EVEN, t)[0]
        assert (got.view(np.int64) == want.view(np.int64)).all()
        plus_zero = t.view(np.int64) == 0
        assert (valid | plus_zero).all()
        return want

    # Sequential (Dot.java:50-56).
    s = np.zeros(prods.shape[0])
    for j in range(K):
        s = check_round(s + prods[:, j], _lo_word(s))
    # Pairwise over 8-term leaves, combined as a perfect tree.
    leaves = []
    for l0 in range(0, K, 8):
        s = np.zeros(prods.shape[0])
        for j in range(l0, l0 + 8):
            s = check_round(s + prods[:, j], _lo_word(s))
        leaves.append(s)
    while len(leaves) > 1:
        leaves = [check_round(leaves[i] + leaves[i + 1], _lo_word(leaves[i + 1]))
                  for i in range(0, len(leaves), 2)]


def test_range_proof_rejects_out_of_bound_operands():
    rs = np.random.default_rng(3)
    a, b = _proven_operands(rs, 8, 64, -20, 4)
    assert _range_proven(O.ACC_FP32, a, b, 64)
    for bad in (2.0 ** -60, np.inf, np.nan, 5e-324, 2.0 ** 120):
        a2 = a.copy()
        a2[3, 5] = bad
        assert not _range_proven(O.ACC_FP32, a2, b, 64), bad
    # BF16's growth term: (1 + 2^-8)^(K+1) takes 47 bits at K = 8192.
    assert _range_limit(O.ACC_BF16, 8192) == 126 - 13 - 47
    assert _range_limit(O.ACC_FP32, 8192) == 126 - 13 - 1


def _int_round(t, shift):
    """FastForm.rne_int (codec.cuh) on t's bit pattern: add half a quantum
    less one plus the kept part's lowest bit, clear the dropped bits."""
    u = t.view(np.uint64).copy()
    s = np.uint64(shift)
    u += (np.uint64(1) << (s - np.uint64(1))) - np.uint64(1) + ((u >> s) & np.uint64(1))
    u &= ~((np.uint64(1) << s) - np.uint64(1))
    return u.view(np.float64)


@pytest.mark.parametrize("acc", ["fp32", "fp16", "bf16"])
def test_integer_pipe_rounding_matches_oracle(acc):
    """The integer-pipe form of round-to-nearest-even agrees with Dot.round /
    (float) on every sum the range word admits, ties included."""
    rs = np.random.default_rng(21)
    n = 600_000
    if acc == "fp32":
        shift, lo_e, hi_e = 29, 1023 - 126, 1023 + 126
        t = _sums(rs, n, shift, -150, 130)
        with np.errstate(over="ignore"):
            want = t.astype(np.float32).astype(np.float64)
    else:
        acc_id = 2 if acc == "fp16" else 3
        mant, min_e, max_e = (10, -14, 15) if acc == "fp16" else (7, -126, 127)
        shift, lo_e, hi_e = 52 - mant, 1023 + min_e, 1023 + max_e - 1
        t = _sums(rs, n, shift, min_e - 10, max_e + 3)
        want = O.acc_round(acc_id, O.NEAREST_EVEN, t)[0]
    _, valid = _fast_round(t, np.zeros(n, np.uint32), shift, lo_e, hi_e)
    with np.errstate(all="ignore"):
        got = _int_round(t, shift)
    bad = valid & (got.view(np.int64) != want.view(np.int64))
    assert not bad.any(), (acc, t[bad][:3])
    assert valid.mean() > 0.6
