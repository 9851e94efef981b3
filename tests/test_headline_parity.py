"""The policy sweep at its full size, bit for bit against the oracle.

The sweep's GEMM is M = N = K = 8192 on N(0,1) x lognormal(0,1) doubles with
full 53-bit significands (generated on the device by the same seeded generator
the bench uses), under RealDotSweep's 12 policies
(java/src/main/java/io/drift/tools/RealDotSweep.java:97-108) plus the FP64
exact GEMM. Every contraction runs on the device at full size, on the route
it takes in the sweep (the double-precision tiled kernel, or the FP32 pipe for
the bf16 and MX-e4m3 casts); then a sample of 16 rows x 128 columns of each
output, spread over many 64 x 64 and 128 x 128 tiles, is recomputed by the
oracle over the full K = 8192 terms from the device's cast operands, and those
cast rows are themselves checked against the oracle's cast of the host copy
(per-tensor scales from the full tensors). No tolerance: every sampled output
bit, every sampled cast bit and the clamp counts.
"""
import numpy as np
import pytest

from helpers import assert_bits, opolicy

pytestmark = pytest.mark.gpu

SIZE = 8192
ROWS = np.array([0, 1, 63, 64, 127, 1000, 2047, 2048, 3333, 4095, 4096, 5001, 6143, 7000, 8190,
                 8191])
COLS = np.unique(np.concatenate([np.arange(0, 8192, 67), [63, 64, 127, 128, 8127, 8191]]))[:128]


@pytest.fixture(scope="module")
def sweep():
    import torch

    import drift_b200 as d
    from drift_b200 import sweeps

    dev = torch.device("cuda", 0)
    A, B = sweeps.policy_sweep_inputs(SIZE, 0, dev)
    hA, hB = A.cpu().numpy(), B.cpu().numpy()
    return d, torch, A, B, hA, hB


def _cast_dev(d, torch, p, src, dst):
    f = p.input_format
    clamped = torch.zeros(1, dtype=torch.int64, device=src.device)
    if p.scaling == d.Scaling.PER_TENSOR:
        amax = torch.zeros(1, dtype=torch.float64, device=src.device)
        scale = torch.zeros(1, dtype=torch.float64, device=src.device)
        d.amax_dev(src, amax)
        d.per_tensor_scale_dev(f, amax, scale)
        d.quantize_dev(p, f, p.input_rounding, src, dst, d_scale=scale, d_clamped=clamped)
    else:
        d.quantize_dev(p, f, p.input_rounding, src, dst, d_clamped=clamped)
    return int(clamped.item())


def _proven(torch, a, b, bf16):
    """The contraction's range proof (gemm.cu range_proven) on device
    operands with no Inf, NaN or subnormal: exponents of the smallest nonzero
    magnitudes sum to at least -74, of the largest to at most the limit."""
    from helpers import range_limit

    ex = []
    for t in (a, b):
        m = t.abs()
        assert bool(torch.isfinite(m).all())
        nz = m[m != 0]
        assert float(nz.min()) >= 2.0 ** -1022
        ex.append((int(torch.frexp(nz.min())[1]) - 1, int(torch.frexp(nz.max())[1]) - 1))
    (la, ta), (lb, tb) = ex
    return la + lb >= -74 and ta + tb + 2 <= range_limit(bf16, SIZE)


def _names():
    from drift_b200 import sweeps
    return ["exact fp64"] + [p.name for p in sweeps.policy_sweep_policies()]


@pytest.mark.parametrize("name", _names())
def test_full_size_contraction_sampled_against_oracle(sweep, name):
    from drift_b200 import sweeps
    from oracle import oracle as O

    d, torch, A, B, hA, hB = sweep
    pols = {p.name: p for p in sweeps.policy_sweep_policies()}
    p = d.NumericPolicy.exact() if name == "exact fp64" else pols[name]
    op = opolicy(p)
    K = SIZE
    a_rows, b_rows = hA[ROWS], hB[COLS]
    a, b = A, B
    if p.input_format is not None:
        f = p.input_format
        qA, qB = torch.empty_like(A), torch.empty_like(B)
        cl_a = _cast_dev(d, torch, p, A, qA)
        cl_b = _cast_dev(d, torch, p, B, qB)
        d.check_dev()
        a, b = qA, qB
        sa = sb = 1.0
        if p.scaling == d.Scaling.PER_TENSOR:
            sa = O.per_tensor_scale(f.id, O.amax(hA))
            sb = O.per_tensor_scale(f.id, O.amax(hB))
        # The sampled rows of the device casts against the oracle's cast of the
        # same rows (MX blocks of 32 along K never cross a row of 8192).
        o_a, _, _ = O.quantize(op, f.id, int(p.input_rounding), a_rows, sa)
        o_b, _, _ = O.quantize(op, f.id, int(p.input_rounding), b_rows, sb)
        assert_bits(qA[torch.from_numpy(ROWS).cuda()].cpu().numpy(), o_a, f"{name} cast of A")
        assert_bits(qB[torch.from_numpy(COLS).cuda()].cpu().numpy(), o_b, f"{name} cast of B")
        if p.scaling != d.Scaling.MX_BLOCK:
            # Whole-tensor clamp counts (Quant.java:67, :75) against the oracle.
            assert cl_a == O.quantize(op, f.id, int(p.input_rounding), hA, sa)[1]
            assert cl_b == O.quantize(op, f.id, int(p.input_rounding), hB, sb)[1]
        a_rows, b_rows = o_a, o_b
    C = torch.empty((SIZE, SIZE), dtype=torch.float64, device=A.device)
    d.gemm_dev(p, a, b, C)
    route = d.gemm_route()
    d.check_dev()
    if name in ("bf16 cast", "e4m3 mx32 cast"):
        assert route == d.ROUTE_FP32, route     # the FP32 pipe at full size
    else:
        # The 53-bit inputs keep the double-precision contraction; FP32 and
        # BF16 accumulators run it without per-step checks when the operand
        # scan proves the range.
        if p.acc in (d.Acc.FP32, d.Acc.BF16) and _proven(torch, a, b, p.acc == d.Acc.BF16):
            assert route == d.ROUTE_PROVEN, route
        else:
            assert route in (d.ROUTE_DOUBLE, d.ROUTE_SCANNED), route
    got = C[torch.from_numpy(ROWS).cuda()][:, torch.from_numpy(COLS).cuda()].cpu().numpy()
    del C
    want, _ = O.gemm(op, len(ROWS), len(COLS), K, a_rows, 0, K, 1, b_rows, 0, K, 1, threads=16)
    assert_bits(got, want, f"{name} outputs")
