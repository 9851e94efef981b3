"""GPU parity of the range-proven contraction (route 4): FP32 and BF16
accumulators whose operand scan proves that every partial sum stays inside
the fast rounding's exact range, so the per-step checks are left out.

The cases sit on both edges of the proof: operands whose nonzero magnitudes
reach down to 2^-37 each (products down to 2^-74) with rows built so that
pairs of products cancel and the sums fall back to rounding residues again and
again; magnitudes whose largest exponents meet the high-side bound exactly,
with every product of one sign; operands of zeros. Just past each edge (one
element too small or too large, an Inf, a NaN, a subnormal) the scan refuses
and the checked build runs. Every order (Dot.java:37-121), both BF16
roundings, the host-built pairwise and blocked schedules. Bit-exact against
the oracle either way."""
import numpy as np
import pytest

from helpers import assert_bits, range_limit, range_proven, tiled_route
from oracle import oracle as O

pytestmark = pytest.mark.gpu

PROVEN, DOUBLE, SCANNED = 4, 0, 2


@pytest.fixture(scope="module")
def d():
    import drift_b200
    d = drift_b200
    d.set_thin_tiles(0)     # every call here on the tiled kernel
    yield d
    d.set_thin_tiles(-1)


def operands(rs, rows, k, lo, hi, cancel=True, zeros=0.05):
    """rows x k doubles with 53-bit significands, nonzero magnitudes in
    [2^lo, 2^hi), random signs, a share of zeros; with `cancel`, half the
    rows repeat each even term in the next odd one (and the caller negates
    the other operand's), so those products cancel pairwise."""
    e = rs.integers(lo, hi, (rows, k))
    x = np.ldexp(1.0 + rs.random((rows, k)), e) * np.where(rs.random((rows, k)) < 0.5, -1.0, 1.0)
    if cancel:
        x[: rows // 2, 1::2] = x[: rows // 2, 0::2]
    x[rs.random((rows, k)) < zeros] = 0.0
    return x


def cancelling_pair(rs, M, N, K, lo, hi):
    A = operands(rs, M, K, lo, hi)
    B = operands(rs, N, K, lo, hi)
    B[: N // 2, 1::2] = -B[: N // 2, 0::2]
    return A, B


def run(d, acc, order, rm, M, N, K, A, B, route, acc_block=32):
    p = (d.NumericPolicy.builder("t").acc(d.Acc(acc)).order(d.Order(order))
         .acc_rounding(d.Rounding(rm)).acc_block(acc_block).build())
    A = np.ascontiguousarray(A, dtype=np.float64).reshape(-1)
    B = np.ascontiguousarray(B, dtype=np.float64).reshape(-1)
    got = d.gemm(p, M, N, K, A, 0, K, 1, B, 0, K, 1)
    assert d.gemm_route() == route, (acc, order, rm, d.gemm_route())
    if route in (PROVEN, DOUBLE):
        assert tiled_route(acc, M, N, K, A, B, rm) == route  # the model agrees
    op = O.policy(acc=acc, order=order, acc_rounding=rm, acc_block=acc_block)
    want, _ = O.gemm(op, M, N, K, A, 0, K, 1, B, 0, K, 1, threads=16)
    assert_bits(got, want, f"acc={acc} order={order} rm={rm} M={M} N={N} K={K}")
    return got


CASES = [(1, o, 0) for o in range(4)] + [(3, o, rm) for o in range(4) for rm in (0, 2)]


@pytest.mark.parametrize("acc,order,rm", CASES)
def test_low_edge_cancellation(d, acc, order, rm):
    rs = np.random.default_rng(100 * acc + 10 * order + rm)
    M = N = K = 512
    A, B = cancelling_pair(rs, M, N, K, -37, 6)
    assert range_proven(acc == 3, A, B, K)
    run(d, acc, order, rm, M, N, K, A, B, PROVEN)


@pytest.mark.parametrize("acc,order,rm", CASES)
def test_high_edge_growth(d, acc, order, rm):
    """The largest exponents meet the bound exactly (ta + tb + 2 == limit)
    and every product is positive, so the sums grow as far as the data can
    take them."""
    rs = np.random.default_rng(7 + 100 * acc + 10 * order + rm)
    M = N = K = 512
    lim = range_limit(acc == 3, K)
    ta = (lim - 2) // 2
    tb = lim - 2 - ta
    A = np.abs(operands(rs, M, K, ta - 6, ta + 1, cancel=False))
    B = np.abs(operands(rs, N, K, tb - 6, tb + 1, cancel=False))
    assert range_proven(acc == 3, A, B, K)
    run(d, acc, order, rm, M, N, K, A, B, PROVEN)


@pytest.mark.parametrize("acc,rm", [(1, 0), (3, 0), (3, 2)])
def test_host_built_schedules(d, acc, rm):
    """Pairwise over a K that is not a power of two and blocked chunks off
    the 16-wide tile run the schedule-driven builds, proven too."""
    rs = np.random.default_rng(31 + acc + rm)
    M, N, K = 640, 640, 328
    A, B = cancelling_pair(rs, M, N, K, -30, 4)
    run(d, acc, 2, rm, M, N, K, A, B, PROVEN)
    M = N = K = 512
    A, B = cancelling_pair(rs, M, N, K, -30, 4)
    run(d, acc, 3, rm, M, N, K, A, B, PROVEN, acc_block=37)


@pytest.mark.parametrize("acc,rm", [(1, 0), (3, 0), (3, 2)])
@pytest.mark.parametrize("plant", ["small", "large", "inf", "nan", "subnormal"])
def test_just_past_the_edge_runs_checked(d, acc, rm, plant):
    rs = np.random.default_rng(53 + acc + rm)
    M = N = K = 512
    A, B = cancelling_pair(rs, M, N, K, -30, 4)
    # la + lb = -30 + -30 = -60: a 2^-45 element takes it to -75.
    value = {"small": 2.0 ** -45, "large": 2.0 ** (range_limit(acc == 3, K) - 2 - 3 + 1),
             "inf": np.inf, "nan": np.nan, "subnormal": 1e-310}[plant]
    A[17, 100] = value
    assert not range_proven(acc == 3, A, B, K)
    for order in range(4):
        # An FP32 accumulator's sequential, reversed and 32-blocked calls
        # first scan for the FP32 pipe, which declines (route 2).
        run(d, acc, order, rm, M, N, K, A, B, SCANNED if acc == 1 and order != 2 else DOUBLE)


@pytest.mark.parametrize("acc,rm", [(1, 0), (3, 0), (3, 2)])
def test_ties(d, acc, rm):
    """Operands of 4 significant bits, so that many sums land exactly
    halfway between two accumulator values (ties go to even) or carry
    nothing below the kept bits; every order, chunks on and off the tile."""
    rs = np.random.default_rng(71 + acc + rm)
    M = N = K = 512

    def few_bits(n):
        m = rs.integers(8, 16, (n, K)).astype(np.float64)
        return np.ldexp(m, rs.integers(-13, 1, (n, K))) * np.where(rs.random((n, K)) < 0.5, -1, 1)
    A, B = few_bits(M), few_bits(N)
    for order, blk in [(0, 32), (1, 32), (2, 32), (3, 32), (3, 37)]:
        route = tiled_route(acc, M, N, K, A, B, rm)
        if acc == 1 and (order in (0, 1) or blk % 16 == 0) and order != 2:
            route = 1      # exact fp32 products: the FP32 pipe takes these
        run(d, acc, order, rm, M, N, K, A, B, route, acc_block=blk)


def test_operand_of_zeros(d):
    rs = np.random.default_rng(61)
    M = N = K = 512
    A = operands(rs, M, K, -30, 4)
    B = np.zeros((N, K))
    B[5] = -0.0
    for acc in (1, 3):
        for order in range(4):
            got = run(d, acc, order, 0, M, N, K, A, B, PROVEN)
            assert (got.view(np.int64) == 0).all()     # every sum +0


def test_launch_counts(d):
    """drift_gemm_launches: the scan and both builds for a proven-route call,
    one kernel for a call below 2^27 MACs or with an FP64 accumulator."""
    import torch

    rs = np.random.default_rng(67)
    A = torch.from_numpy(operands(rs, 512, 512, -20, 4)).cuda()
    B = torch.from_numpy(operands(rs, 512, 512, -20, 4)).cuda()
    C = torch.empty(512, 512, dtype=torch.float64, device="cuda")
    b = d.NumericPolicy.builder
    d.gemm_dev(b("p").acc(d.Acc.BF16).order(d.Order.PAIRWISE).build(), A, B, C)
    assert d.gemm_launches() == 3 and d.gemm_route() == PROVEN
    d.gemm_dev(b("x").acc(d.Acc.FP64).build(), A, B, C)
    assert d.gemm_launches() == 1 and d.gemm_route() == DOUBLE
    # FP32 sequential: the FP32 pipe's two scans, decision and contraction,
    # then the range scan and both double-precision builds.
    d.gemm_dev(b("s").acc(d.Acc.FP32).build(), A, B, C)
    assert d.gemm_launches() == 7 and d.gemm_route() == PROVEN
    Cs = C[:256, :256].contiguous()
    d.gemm_dev(b("s").acc(d.Acc.FP32).order(d.Order.PAIRWISE).build(), A[:256, :256].contiguous(),
               B[:256, :256].contiguous(), Cs)
    assert d.gemm_launches() == 1
    d.check_dev()
