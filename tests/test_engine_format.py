"""GPU parity of the format layer: MiniFloat.encode/decode and Dot.round.

Expected values come from the reference's exact-rational codec (golden
fixtures) and, for stochastic rounding and truncation, from the oracle. Every
call goes through the engine's C ABI.
"""
import math

import numpy as np
import pytest

from helpers import assert_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FORMATS = ["e4m3", "e5m2", "e2m1", "e3m2", "e2m3", "fp16", "bf16"]


@pytest.fixture(scope="module")
def d():
    import drift_b200
    return drift_b200


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(golden_dir / "formats.npz")


@pytest.mark.parametrize("fid,name", list(enumerate(FORMATS)))
def test_decode_every_code(d, golden, fid, name):
    f = d.Formats.ALL[fid]
    want = golden[f"{name}_values"].astype(np.float64)
    assert_bits(f.decode(np.arange(len(want), dtype=np.int32)), want, name)


@pytest.mark.parametrize("fid,name", list(enumerate(FORMATS)))
def test_products_and_sums_round_once(d, golden, fid, name):
    """python/verify_oracle.py:77-102 on the device encoder."""
    f = d.Formats.ALL[fid]
    va = golden[f"{name}_values"].astype(np.float64)[golden[f"{name}_pair_a"]]
    vb = golden[f"{name}_values"].astype(np.float64)[golden[f"{name}_pair_b"]]
    with np.errstate(all="ignore"):
        prod, summ = va * vb, va + vb
    if f.specials == d.Specials.FINITE:  # no NaN can arise from finite codes
        assert not np.isnan(prod).any()
    assert (f.encode(prod) == golden[f"{name}_prod"]).all()
    assert (f.encode(summ) == golden[f"{name}_sum"]).all()


@pytest.mark.parametrize("fid,name", list(enumerate(FORMATS)))
def test_encode_random_doubles(d, golden, fid, name):
    f = d.Formats.ALL[fid]
    assert (f.encode(golden[f"{name}_rand_x"]) == golden[f"{name}_rand_code"]).all()


@pytest.mark.parametrize("fid", range(7))
@pytest.mark.parametrize("rm", [1, 2])
@pytest.mark.parametrize("n", [1, 33, 5000, 300_001])
def test_encode_stochastic_and_truncate_match_oracle(d, golden, fid, rm, n):
    """Codes and the Rng state afterwards equal the oracle's (the draw stream
    is consumed only by inexact elements, MiniFloat.java:264-273)."""
    f = d.Formats.ALL[fid]
    rs = np.random.default_rng(fid * 100 + rm * 10 + n % 7)
    x = rs.standard_normal(n) * np.exp2(rs.uniform(-12, 12, n)) * f.max_finite / 64
    x[:: 5] = np.round(x[:: 5])  # exact values: no draw
    rng = d.Rng(0x1234 + n)
    got = f.encode(x, d.Rounding(rm), rng)
    want, state = O.encode(fid, rm, x, 0x1234 + n)
    assert (got == want).all()
    assert rng.state() == state


@pytest.mark.parametrize("acc,fid", [(2, 5), (3, 6)])
@pytest.mark.parametrize("rm", [0, 1, 2])
def test_fast_accumulator_rounding_matches_minifloat(d, acc, fid, rm):
    """KernelTest.fastAccumulatorRoundingMatchesMiniFloat (KernelTest.java:25-48)
    on the device: Dot.round equals MiniFloat.quantize, bits and Rng state."""
    rs = np.random.default_rng(11)
    n = 400_000
    x = rs.choice([-1.0, 1.0], n) * np.ldexp(1 + rs.random(n), rs.integers(-150, 150, n))
    x[::97] = np.rint(x[::97])
    r1, r2 = d.Rng(99), d.Rng(99)
    fast = d.Dot.round(x, d.Acc(acc), d.Rounding(rm), r1)
    slow = d.Formats.ALL[fid].quantize(x, d.Rounding(rm), r2)
    assert_bits(fast, slow, "round vs quantize")
    assert r1.state() == r2.state()
    want, state = O.acc_round(acc, rm, x, 99)
    assert_bits(fast, want, "round vs oracle")
    assert r1.state() == state


# ------------------------------------------- MiniFloatTest on the device

def test_published_ranges(d):
    F = d.Formats
    assert F.E4M3.max_finite == 448.0 and F.E4M3.min_subnormal == 2 ** -9
    assert F.E5M2.max_finite == 57344.0 and F.E5M2.min_subnormal == 2 ** -16
    assert F.E2M1.max_finite == 6.0 and F.E2M1.min_subnormal == 0.5
    assert F.FP16.max_finite == 65504.0
    assert F.BF16.max_finite == math.ldexp(255.0, 120)


def test_every_code_round_trips(d):
    for f in d.Formats.ALL:
        codes = np.arange(f.code_count(), dtype=np.int32)
        v = f.decode(codes)
        keep = np.isfinite(v)
        assert (f.encode(v[keep]) == codes[keep]).all(), f.name


def test_specials_ties_saturation_negative_zero(d):
    F = d.Formats
    assert math.isnan(F.E4M3.decode(0x7F)) and F.E4M3.decode(0x7E) == 448.0
    assert F.E5M2.decode(0x7C) == math.inf and math.isnan(F.E5M2.decode(0x7D))
    assert list(F.E2M1.quantize([2.5, 3.5, 1.25, 1.75])) == [2.0, 4.0, 1.0, 2.0]
    assert list(F.E4M3.quantize([1e6, -1e6])) == [448.0, -448.0]
    assert F.E2M1.quantize(7.9) == 6.0 and F.E5M2.quantize(math.inf) == 57344.0
    assert F.E4M3.encode(-0.0) == 0x80
    assert math.copysign(1.0, F.E4M3.decode(0x80)) < 0


def test_stochastic_rounding_is_unbiased(d):
    q = d.Formats.E2M1.quantize(np.full(400_000, 2.25), d.Rounding.STOCHASTIC, d.Rng(3))
    assert abs(q.mean() - 2.25) < 4e-3


def test_errors_match_java(d):
    """NaN into a finite format throws (MiniFloat.java:157-160); a decode of
    a code wider than the format throws (:118-120); SR without an Rng throws
    only when it needs a draw (:270-272)."""
    with pytest.raises(d.DriftError) as e:
        d.Formats.E2M1.encode([1.0, math.nan])
    assert e.value.status == 2
    with pytest.raises(d.DriftError):
        d.Formats.E2M1.decode([16])
    assert list(d.Formats.E2M1.quantize([1.0, 6.0], d.Rounding.STOCHASTIC, None)) == [1.0, 6.0]
    with pytest.raises(d.DriftError) as e:
        d.Formats.E2M1.quantize([2.25], d.Rounding.STOCHASTIC, None)
    assert e.value.status == 1
    # The context is still usable after a device-side error.
    assert d.Formats.E2M1.quantize(2.5) == 2.0
