"""Test inputs and comparisons shared by the parity tests."""
from __future__ import annotations

import numpy as np


def same_bits(a, b) -> np.ndarray:
    """Element-wise bit equality of doubles; any NaN equals any NaN (the JVM
    does not specify NaN payloads, so only NaN-ness is compared)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    both_nan = np.isnan(a) & np.isnan(b)
    return (a.view(np.int64) == b.view(np.int64)) | both_nan


def assert_bits(got, want, what="") -> None:
    ok = same_bits(got, want)
    if not ok.all():
        idx = np.flatnonzero(~ok.reshape(-1))
        g = np.asarray(got, dtype=np.float64).reshape(-1)
        w = np.asarray(want, dtype=np.float64).reshape(-1)
        first = ", ".join(f"[{i}] got {g[i]!r} want {w[i]!r}" for i in idx[:5])
        raise AssertionError(f"{what}: {idx.size} of {ok.size} differ: {first}")


def heavy_tailed(rs: np.random.Generator, n: int, sigma: float = 1.0) -> np.ndarray:
    """N(0,1) x lognormal(0, sigma), the distribution of the sweeps."""
    return rs.standard_normal(n) * np.exp(rs.standard_normal(n) * sigma)


def with_edges(x: np.ndarray, rs: np.random.Generator, nan: bool = True) -> np.ndarray:
    """Plants the special values a cast must handle: signed zeros, double
    subnormals, values far below and above every format, infinities, NaN."""
    x = x.copy()
    n = x.size
    if n < 16:
        return x
    specials = [0.0, -0.0, 5e-324, -1e-310, 1e-45, -3e-8, 1e300, -1e300, np.inf, -np.inf,
                448.0, 449.0, 464.0, 6.0, 7.0, 65504.0, 65520.0]
    if nan:
        specials.append(np.nan)
    pos = rs.choice(n, size=min(n, len(specials) * 3), replace=False)
    for k, p in enumerate(pos):
        x[p] = specials[k % len(specials)]
    return x


def opolicy(p):
    """The oracle's copy of a drift_b200 NumericPolicy."""
    from oracle import oracle as O

    c = p.to_c()
    return O.OraclePolicy(*[getattr(c, f) for f, _ in c._fields_])


class OracleBackend:
    """Casts and contractions on the oracle, for the oracle's pass of the
    training-step mirrors (drift_b200.mlp, drift_b200.attn)."""

    name = "oracle"

    def amax(self, x):
        from oracle import oracle as O
        return O.amax(x)

    def per_tensor_scale(self, f, amax):
        from oracle import oracle as O
        return O.per_tensor_scale(f.id, amax)

    def quantize(self, src, f, p, rm, scale, rng):
        from oracle import oracle as O
        st = rng.state() if rng is not None else None
        dst, clamped, st = O.quantize(opolicy(p), f.id if f is not None else -1, int(rm), src,
                                      scale, st)
        if rng is not None:
            rng.reseed(st)
        return dst, clamped

    def gemm(self, p, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks, bias=None, rng=None):
        from oracle import oracle as O
        st = rng.state() if rng is not None else None
        C, st = O.gemm(opolicy(p), M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks,
                       bias=bias, rng_state=st, threads=16)
        if rng is not None:
            rng.reseed(st)
        return C

    def contract(self, p, op, A, B, C, rng=None):
        from oracle import oracle as O
        st = O.contract(opolicy(p), op, A, B, C, rng.state() if rng is not None else None)
        if rng is not None:
            rng.reseed(st)
        return C


def range_limit(bf16: bool, K: int) -> int:
    """The contraction's range-proof bound on ta + tb + 2 for K terms
    (range_limit_for in gemm.cu): 126 - ceil(log2 K) - ceil(log2 (1+d)^(K+1)),
    d the relative error of a double add then the accumulator's rounding."""
    u = 2.0 ** -8 if bf16 else 2.0 ** -24
    d = u + 2.0 ** -53 + u * 2.0 ** -53
    growth = (K + 1) * np.log1p(d) / np.log(2.0)
    lg = int(np.ceil(np.log2(K))) if K > 1 else 0
    return 126 - lg - int(np.ceil(growth + 1e-9))


def range_proven(bf16: bool, a, b, K: int) -> bool:
    """Whether the contraction's operand scan proves every partial sum of an
    FP32 (or BF16) accumulator in range (range_proven in gemm.cu): no Inf,
    NaN or subnormal; the smallest nonzero magnitudes' binade exponents sum to
    at least -74; the largest ones' plus 2 to at most range_limit."""
    ex = []
    for x in (a, b):
        x = np.abs(np.asarray(x, dtype=np.float64).reshape(-1))
        if np.isnan(x).any() or np.isinf(x).any():
            return False
        x = x[x != 0]
        if x.size == 0:
            return True
        if (x < 2.0 ** -1022).any():
            return False
        e = np.frexp(x)[1] - 1                  # |x| in [2^e, 2^(e+1))
        ex.append((int(e.min()), int(e.max())))
    (la, ta), (lb, tb) = ex
    return la + lb >= -74 and ta + tb + 2 <= range_limit(bf16, K)


def tiled_route(acc: int, M: int, N: int, K: int, a, b, rounding: int = 0) -> int:
    """The route a tiled (not thin, not FP32-pipe) non-stochastic GEMM
    reports: 4 (range proven, no per-step checks) for an FP32 or BF16
    accumulator over at least 2^27 multiply-accumulates whose operands pass
    the proof, else 0."""
    if acc in (1, 3) and rounding in (0, 2) and K > 0 and M * N * K >= 1 << 27:
        if range_proven(acc == 3, a, b, K):
            return 4
    return 0
