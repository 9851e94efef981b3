"""GPU parity of the contraction: Dot.dot over whole GEMMs, every accumulator
width, order and accumulator rounding, on both double-precision routes (the
tiled kernel and one output per thread), the three layouts of Pass.java
(forward NT, dgrad with a strided W column, wgrad with both operands strided),
offsets, bias, and the values that leave the integer fast path (zeros,
cancellation to -0.0, subnormal sums, overflow, saturation). Bit-exact
against the oracle."""
import numpy as np
import pytest

from helpers import assert_bits, heavy_tailed
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ACCS = [0, 1, 2, 3]
ORDERS = [0, 1, 2, 3]


@pytest.fixture(scope="module")
def d():
    import drift_b200
    return drift_b200


EXPECT_ROUTE = [None]


@pytest.fixture(scope="module", params=["tiled", "staged"], autouse=True)
def kernel_route(request, d):
    """Every case runs twice: on the tiled kernel (thin-call threshold 0) and
    with one output per thread (a threshold above any call here)."""
    d.set_thin_tiles(0 if request.param == "tiled" else 1 << 40)
    EXPECT_ROUTE[0] = d.ROUTE_DOUBLE if request.param == "tiled" else d.ROUTE_STAGED
    yield request.param
    d.set_thin_tiles(-1)


def policies(d):
    for acc in ACCS:
        for order in ORDERS:
            for rm in ([0, 2] if acc >= 2 else [0]):
                yield (acc, order, rm)


def compare(d, acc, order, rm, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks, bias=None,
            acc_block=32):
    p = (d.NumericPolicy.builder("t").acc(d.Acc(acc)).order(d.Order(order))
         .acc_rounding(d.Rounding(rm)).acc_block(acc_block).build())
    got = d.gemm(p, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks, bias=bias)
    assert d.gemm_route() == EXPECT_ROUTE[0]
    op = O.policy(acc=acc, order=order, acc_rounding=rm, acc_block=acc_block)
    want, _ = O.gemm(op, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks, bias=bias, threads=8)
    assert_bits(got, want, f"acc={acc} order={order} rm={rm} M={M} N={N} K={K}")


SHAPES = [(1, 1, 1), (3, 5, 7), (64, 64, 16), (65, 63, 33), (130, 70, 100), (17, 9, 0),
          (2, 3, 1000), (64, 96, 96), (9, 8, 64)]


@pytest.mark.parametrize("acc,order,rm", [(a, o, r) for a in ACCS for o in ORDERS
                                           for r in ([0, 2] if a >= 2 else [0])])
def test_forward_layout(d, acc, order, rm):
    rs = np.random.default_rng(acc * 100 + order * 10 + rm)
    for M, N, K in SHAPES:
        A = heavy_tailed(rs, max(1, M * K))
        B = heavy_tailed(rs, max(1, N * K))
        compare(d, acc, order, rm, M, N, K, A, 0, K, 1, B, 0, K, 1)


@pytest.mark.parametrize("acc,order", [(a, o) for a in ACCS for o in ORDERS])
def test_pass_backward_layouts(d, acc, order):
    """dgrad: dx[i,k] = dot(G row i, W column k) (Pass.java:222-226);
    wgrad: dw[o,k] = dot(G column o, X column k) over the batch (:228-232)."""
    rs = np.random.default_rng(acc * 4 + order)
    batch, inp, out = 20, 70, 96
    G = heavy_tailed(rs, batch * out)
    W = heavy_tailed(rs, out * inp)
    X = heavy_tailed(rs, batch * inp)
    compare(d, acc, order, 0, batch, inp, out, G, 0, out, 1, W, 0, 1, inp)      # dgrad
    compare(d, acc, order, 0, out, inp, batch, G, 0, 1, out, X, 0, 1, inp)      # wgrad


@pytest.mark.parametrize("acc,order", [(a, o) for a in ACCS for o in ORDERS])
def test_offsets_bias_and_general_strides(d, acc, order):
    rs = np.random.default_rng(7 + acc + 5 * order)
    buf_a = heavy_tailed(rs, 5000)
    buf_b = heavy_tailed(rs, 5000)
    bias = heavy_tailed(rs, 13)
    # Odd offsets, strides that are neither 1 nor the row length.
    compare(d, acc, order, 0, 11, 13, 37, buf_a, 3, 41, 3, buf_b, 5, 2, 97, bias=bias)
    # KernelTest.stridesWalkColumns (KernelTest.java:89-96), any accumulator.
    compare(d, acc, order, 0, 1, 1, 2, np.array([1, 2, 3, 4, 5, 6.0]), 1, 0, 3,
            np.array([10, 100.0]), 0, 0, 1)


@pytest.mark.parametrize("acc,order,rm", [(a, o, r) for a in ACCS for o in ORDERS
                                           for r in ([0, 2] if a >= 2 else [0])])
def test_values_off_the_fast_path(d, acc, order, rm):
    rs = np.random.default_rng(99 + acc * 16 + order * 4 + rm)
    M, N, K = 40, 36, 48
    A = heavy_tailed(rs, M * K)
    B = heavy_tailed(rs, N * K)
    A[::7] = 0.0                                    # zero products
    A[:K] = 1.0
    B[:K] = np.tile([1e-3, -1e-3], K // 2)          # exact cancellation to zero
    A[K:2 * K] = 2.0 ** -140                        # sums below every normal range
    A[2 * K:3 * K] = 1e30                           # fp32 overflow, fp16/bf16 saturation
    A[3 * K:4 * K] = -2.0 ** -20                    # fp16 subnormal sums, -0.0 results
    B[K:2 * K] = rs.standard_normal(K) * 1e-3
    A[4 * K] = np.inf
    A[5 * K] = np.nan
    compare(d, acc, order, rm, M, N, K, A, 0, K, 1, B, 0, K, 1)


@pytest.mark.parametrize("acc", ACCS)
@pytest.mark.parametrize("K", [9, 100, 1000, 4099, 40_000])
def test_pairwise_trees_regular_and_irregular(d, acc, K):
    """Dot.pairwise splits with half = count >>> 1 and leaves of at most 8
    (Dot.java:86-102); deep and uneven trees included."""
    rs = np.random.default_rng(K)
    M, N = 3, 66
    A = heavy_tailed(rs, M * K)
    B = heavy_tailed(rs, N * K)
    compare(d, acc, 2, 0, M, N, K, A, 0, K, 1, B, 0, K, 1)


@pytest.mark.parametrize("acc,rm", [(a, r) for a in ACCS for r in ([0, 2] if a >= 2 else [0])])
@pytest.mark.parametrize("acc_block", [1, 7, 32, 37, 64, 96, 1000])
def test_blocked_any_chunk(d, acc, rm, acc_block):
    """Chunks on and off the 16-wide k tile, both accumulator roundings; 70
    columns cover every column slot of a thread's 4 x 4 block."""
    rs = np.random.default_rng(acc_block)
    M, N, K = 5, 70, 300
    A = heavy_tailed(rs, M * K)
    B = heavy_tailed(rs, N * K)
    compare(d, acc, 3, rm, M, N, K, A, 0, K, 1, B, 0, K, 1, acc_block=acc_block)


def test_summation_order_changes_fp32_answer(d):
    """KernelTest.summationOrderChangesTheAnswerInFp32 (KernelTest.java:78-87)."""
    a, ones = np.array([1.0, 1e8, -1e8]), np.ones(3)
    seq = d.NumericPolicy.builder("s").acc(d.Acc.FP32).order(d.Order.SEQUENTIAL).build()
    rev = d.NumericPolicy.builder("r").acc(d.Acc.FP32).order(d.Order.REVERSED).build()
    assert d.Dot.dot(a, 0, 1, ones, 0, 1, 3, seq) == 0.0
    assert d.Dot.dot(a, 0, 1, ones, 0, 1, 3, rev) == 1.0


def test_every_order_agrees_in_fp64(d):
    """KernelTest.everyOrderAgreesInFp64 (KernelTest.java:60-76), accBlock 37."""
    rs = np.random.default_rng(5)
    a, b = rs.standard_normal(1000), rs.standard_normal(1000)
    plain = float(np.sum(a * b))
    for o in d.Order:
        p = d.NumericPolicy.builder("t").acc(d.Acc.FP64).order(o).acc_block(37).build()
        assert abs(d.Dot.dot(a, 0, 1, b, 0, 1, 1000, p) - plain) <= 1e-12 * abs(plain)


def test_large_fp32_sampled_outputs(d):
    """A 1024 x 1024 x 2048 product: every sampled output equals the oracle."""
    import torch

    rs = np.random.default_rng(3)
    M = N = 1024
    K = 2048
    A = heavy_tailed(rs, M * K).reshape(M, K)
    B = heavy_tailed(rs, N * K).reshape(N, K)
    for acc, order in [(1, 0), (2, 2), (3, 3), (0, 1)]:
        p = d.NumericPolicy.builder("t").acc(d.Acc(acc)).order(d.Order(order)).build()
        dA = torch.from_numpy(A).cuda()
        dB = torch.from_numpy(B).cuda()
        dC = torch.empty((M, N), dtype=torch.float64, device="cuda")
        d.gemm_dev(p, dA, dB, dC)
        got = dC.cpu().numpy()
        rows = rs.choice(M, 16, replace=False)
        op = O.policy(acc=acc, order=order)
        want, _ = O.gemm(op, 16, N, K, A[rows].copy(), 0, K, 1, B, 0, K, 1, threads=8)
        assert_bits(got[rows], want, f"acc={acc} order={order}")
