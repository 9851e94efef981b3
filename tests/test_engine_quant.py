"""GPU parity of the cast pass: Quant.amax / perTensorScale / quantize.

Every case compares the engine with the oracle on the same seeded input:
effective doubles bit for bit, the clamp count, and the Rng state after the
call. Inputs carry the special values of helpers.with_edges.
"""
import math

import numpy as np
import pytest

from helpers import assert_bits, heavy_tailed, with_edges
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def d():
    import drift_b200
    return drift_b200


def run_both(d, fid, rm, scaling, x, block=32, headroom=0, seed=77):
    f = d.Formats.ALL[fid]
    p = (d.NumericPolicy.builder("t").input(f).scaling(d.Scaling(scaling))
         .scale_block(block).mx_headroom(headroom).build())
    scale = 1.0
    if scaling == 1:
        scale = d.Quant.per_tensor_scale(f, d.Quant.amax(x))
        assert scale == O.per_tensor_scale(fid, O.amax(x))
    dst = np.empty_like(x)
    rng = d.Rng(seed)
    clamped = d.Quant.quantize(x, 0, dst, 0, x.size, f, p, scale, rng, d.Rounding(rm))
    op = O.policy(input_format=fid, scaling=scaling, scale_block=block, mx_headroom=headroom)
    want, want_cl, want_state = O.quantize(op, fid, rm, x, scale, seed)
    assert_bits(dst, want, f"{f.name} rm={rm} scaling={scaling} block={block} n={x.size}")
    assert clamped == want_cl
    assert rng.state() == want_state


@pytest.mark.parametrize("fid", range(7))
@pytest.mark.parametrize("scaling", [0, 1, 2])
@pytest.mark.parametrize("rm", [0, 1, 2])
def test_quantize_matches_oracle(d, fid, scaling, rm):
    rs = np.random.default_rng(fid * 31 + scaling * 7 + rm)
    finite_fmt = fid in (2, 3, 4)
    for n in (1, 31, 32, 33, 1000, 65_537):
        x = with_edges(heavy_tailed(rs, n) * (3.0 if fid == 2 else 50.0), rs, nan=not finite_fmt)
        run_both(d, fid, rm, scaling, x)


@pytest.mark.parametrize("block,headroom", [(32, 1), (37, 0), (1, 0), (64, 1), (5, 0)])
@pytest.mark.parametrize("fid", [0, 2, 6])
@pytest.mark.parametrize("rm", [0, 1])
def test_mx_blocks_any_length(d, block, headroom, fid, rm):
    """Blocks follow the flattened span and the last one may be short
    (Quant.java:101-103)."""
    rs = np.random.default_rng(block * 13 + fid)
    x = with_edges(heavy_tailed(rs, 4099), rs, nan=fid not in (2, 3, 4))
    x[100:164] = 0.0  # whole zero blocks draw nothing (Quant.java:105-110)
    x[200] = np.inf   # an infinite block amax zeroes the block, no clamps
    run_both(d, fid, rm, 2, x, block=block, headroom=headroom)


@pytest.mark.parametrize("rm", [0, 1])
def test_large_stochastic_cast_many_ctas(d, rm):
    """Several thousand CTAs: the draw offsets cross CTA boundaries."""
    rs = np.random.default_rng(5)
    x = heavy_tailed(rs, 3_000_017) * 40
    run_both(d, 0, rm, 1, x, seed=0xC0FFEE)
    run_both(d, 2, rm, 2, x / 40, seed=0xC0FFEE)


def test_amax_ignores_nan_and_sees_inf(d):
    x = np.array([1.0, -3.0, np.nan, 2.0])
    assert d.Quant.amax(x) == 3.0
    assert d.Quant.amax(np.array([np.nan, np.nan])) == 0.0
    assert d.Quant.amax(np.array([-np.inf, 1.0])) == np.inf
    assert d.Quant.amax(np.array([-0.0])) == 0.0
    rs = np.random.default_rng(1)
    y = heavy_tailed(rs, 1_000_003)
    assert d.Quant.amax(y) == O.amax(y)


def test_no_format_is_a_copy(d):
    x = np.array([1.5, -0.0, np.inf, 3e-310])
    dst = np.zeros_like(x)
    p = d.NumericPolicy.builder("n").build()
    assert d.Quant.quantize(x, 0, dst, 0, 4, None, p, 1.0, None) == 0
    assert_bits(dst, x)


def test_offsets_follow_java(d):
    """Quant.quantize(src, srcOff, dst, dstOff, n, ...) casts the span only."""
    x = np.array([100.0, 2.5, 3.5, 100.0])
    dst = np.full(6, -1.0)
    p = d.NumericPolicy.builder("e").input(d.Formats.E2M1).build()
    d.Quant.quantize(x, 1, dst, 2, 2, d.Formats.E2M1, p, 1.0, None)
    assert list(dst) == [-1.0, -1.0, 2.0, 4.0, -1.0, -1.0]


def test_spec_exponent_clamps_and_headroom_does_not(d):
    """KernelTest.specExponentClampsAndHeadroomDoesNot (KernelTest.java:123-135)."""
    block = np.zeros(32)
    block[0], block[1] = 7.0, 0.3
    q = np.zeros(32)
    spec = d.NumericPolicy.builder("s").input(d.Formats.E2M1).scaling(d.Scaling.MX_BLOCK).build()
    head = spec.to_builder("h").mx_headroom(1).build()
    assert d.Quant.quantize(block, 0, q, 0, 32, d.Formats.E2M1, spec, 1.0, None) == 1
    assert q[0] == 6.0
    assert d.Quant.quantize(block, 0, q, 0, 32, d.Formats.E2M1, head, 1.0, None) == 0
    assert q[0] == 8.0


def test_mx_dequantisation_is_exact(d):
    """KernelTest.mxScalesArePowersOfTwoSoDequantisationIsExact (:98-116)."""
    rs = np.random.default_rng(2)
    x = rs.standard_normal(256) * 3
    q = np.zeros(256)
    p = d.NumericPolicy.builder("mx").input(d.Formats.E2M1).scaling(d.Scaling.MX_BLOCK).build()
    d.Quant.quantize(x, 0, q, 0, 256, d.Formats.E2M1, p, 1.0, None)
    for s in range(0, 256, 32):
        shared = math.frexp(d.Quant.amax(x[s:s + 32]))[1] - 1 - 2
        el = np.ldexp(q[s:s + 32], -shared)
        assert (d.Formats.E2M1.quantize(el) == el).all()


def test_nan_into_finite_format_raises(d):
    p = d.NumericPolicy.builder("e").input(d.Formats.E2M1).build()
    with pytest.raises(d.DriftError) as e:
        d.Quant.quantize(np.array([1.0, np.nan]), 0, np.zeros(2), 0, 2, d.Formats.E2M1, p, 1.0, None)
    assert e.value.status == 2


@pytest.mark.parametrize("name", ["fp8", "fp8-e4m3-grads", "bf16", "mxfp4"])
def test_rowwise_casts_equal_one_cast_per_row(d, name):
    """drift_quantize_rows_dev against drift_quantize on each row: values and
    clamps (rows with zeros, infinities and a NaN included). MX and stochastic
    rounding are refused: they are cast one tensor at a time."""
    import torch

    p = d.policies.by_name(name)
    f = p.input_format
    rs = np.random.default_rng(3)
    rows, n = 9, 777
    X = heavy_tailed(rs, rows * n).reshape(rows, n)
    X[2] = 0.0
    X[3, 5] = np.inf
    X[4, 7] = np.nan if f.specials != d.Specials.FINITE else 1.0
    src = torch.from_numpy(X).cuda()
    dst = torch.empty_like(src)
    cl = torch.zeros(rows, dtype=torch.int64, device="cuda")
    if p.scaling == d.Scaling.MX_BLOCK:
        with pytest.raises(d.DriftError):
            d.kernel.quantize_rows_dev(p, f, p.input_rounding, src, dst, d_clamped=cl)
        return
    d.kernel.quantize_rows_dev(p, f, p.input_rounding, src, dst, d_clamped=cl)
    d.check_dev()
    got, gcl = dst.cpu().numpy(), cl.cpu().numpy()
    for r in range(rows):
        s = d.Quant.per_tensor_scale(f, d.Quant.amax(X[r])) if p.scaling == d.Scaling.PER_TENSOR \
            else 1.0
        want = np.empty(n)
        c = d.Quant.quantize(X[r], 0, want, 0, n, f, p, s, None)
        assert_bits(got[r], want, f"{name} row {r}")
        assert gcl[r] == c
    sr = p.to_builder("sr").input_rounding(d.Rounding.STOCHASTIC).build()
    with pytest.raises(d.DriftError):
        d.kernel.quantize_rows_dev(sr, f, d.Rounding.STOCHASTIC, src, dst)
