"""The no-allocation cast entry point, drift_quantize_dev_noalloc.

It serves host programs that reserve all device memory up front and do not let
a library allocate while they run; its stochastic-rounding scratch lives in a
fixed array inside the library instead of a workspace. These tests call it
through the C ABI on device buffers and hold it, bit for bit (the tolerance
every cast test here uses), to the ordinary entry point drift_quantize_dev and
to the oracle, on calls in a row so that scratch left over from one call
cannot leak into the next. The cases reach the array's last slot (a
stochastic call of exactly DRIFT_NOALLOC_MAX_ITEMS items, with 32-element
items and with 37-element MX blocks), and a nearest-even call larger than that
limit, which needs no scratch. The file name sorts last so that a run stopping
at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from helpers import opolicy

pytestmark = pytest.mark.gpu

MAX_ITEMS = 1 << 18  # DRIFT_NOALLOC_MAX_ITEMS


@pytest.fixture(scope="module")
def env():
    import torch

    import drift_b200 as d
    from drift_b200 import _lib

    return d, _lib, torch


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _noalloc(d, _lib, torch, p, f, rm, src, dst, state, clamped, err, d_scale=None, scale=1.0):
    pc = p.to_c()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return _lib.load().drift_quantize_dev_noalloc(
        ctypes.byref(pc), f.id, int(rm), _ptr(src), _ptr(dst), src.numel(), _ptr(d_scale),
        float(scale), _ptr(state), _ptr(clamped), _ptr(err), stream)


def _reference(d, torch, p, f, rm, src, d_scale=None, scale=1.0, seed=0):
    """The same cast through the existing entry point (drift_quantize_dev)."""
    dst = torch.empty_like(src)
    state = torch.tensor([seed], dtype=torch.int64, device="cuda")
    clamped = torch.zeros(1, dtype=torch.int64, device="cuda")
    d.quantize_dev(p, f, rm, src, dst, scale=scale, d_scale=d_scale, d_rng_state=state,
                   d_clamped=clamped)
    d.check_dev()
    return dst, int(state.item()), int(clamped.item())


def _policy(d, case):
    F, S, R = d.Formats, d.Scaling, d.Rounding
    f, scaling, block, rm = {
        "e2m1-mx32-sr": (F.E2M1, S.MX_BLOCK, 32, R.STOCHASTIC),
        "e4m3-mx37-sr": (F.E4M3, S.MX_BLOCK, 37, R.STOCHASTIC),
        "e4m3-per-tensor-sr": (F.E4M3, S.PER_TENSOR, 32, R.STOCHASTIC),
        "e5m2-none-sr": (F.E5M2, S.NONE, 32, R.STOCHASTIC),
        "e4m3-per-tensor-rne": (F.E4M3, S.PER_TENSOR, 32, R.NEAREST_EVEN),
    }[case]
    b = d.NumericPolicy.builder(case).input(f).scaling(scaling).input_rounding(rm)
    if scaling == S.MX_BLOCK:
        b = b.scale_block(block)
    return b.build(), f, scaling, block, rm


def _sizes(case, block):
    """Three calls in a row: a large one, one that fills the scratch array to
    its last item (stochastic cases), and a small one."""
    full = block * MAX_ITEMS
    if case.endswith("rne"):
        return (full + 12_345, 70_001, 1_000_003)   # beyond the stochastic limit
    return (1_000_003, full, 70_001)


@pytest.mark.parametrize("case", ["e2m1-mx32-sr", "e4m3-mx37-sr", "e4m3-per-tensor-sr",
                                  "e5m2-none-sr", "e4m3-per-tensor-rne"])
def test_calls_in_a_row_match_the_allocating_entry_point_and_oracle(env, case):
    from oracle import oracle as O

    d, _lib, torch = env
    S = d.Scaling
    p, f, scaling, block, rm = _policy(d, case)
    rs = np.random.default_rng(17)
    state = torch.tensor([0x5EED], dtype=torch.int64, device="cuda")
    clamped = torch.zeros(1, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    seed = 0x5EED
    # The Rng state carries from one call into the next, as a caller sharing
    # one stream would carry it.
    for n in _sizes(case, block):
        x = rs.standard_normal(n) * np.exp(rs.standard_normal(n)) * (3.0 if f.id == 2 else 40.0)
        x[rs.integers(0, n, 64)] = 0.0                # zero elements draw nothing
        src = torch.from_numpy(x).cuda()
        d_scale = None
        scale = 1.0
        if scaling == S.PER_TENSOR:
            scale = d.Quant.per_tensor_scale(f, float(np.abs(x).max()))
            d_scale = torch.tensor([scale], dtype=torch.float64, device="cuda")
        want, want_state, want_clamped = _reference(d, torch, p, f, rm, src, d_scale, scale, seed)
        dst = torch.full_like(src, np.nan)
        clamped.zero_()
        rc = _noalloc(d, _lib, torch, p, f, rm, src, dst, state, clamped, err, d_scale, scale)
        assert rc == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = dst.cpu().numpy()
        assert (got.view(np.int64) == want.cpu().numpy().view(np.int64)).all(), n
        assert int(state.item()) == want_state, n
        assert int(clamped.item()) == want_clamped, n
        # The oracle on the same input and Rng state.
        o_dst, o_clamped, o_state = O.quantize(opolicy(p), f.id, int(rm), x, scale,
                                               seed if rm == d.Rounding.STOCHASTIC else None)
        assert (got.view(np.int64) == o_dst.view(np.int64)).all(), n
        assert int(clamped.item()) == o_clamped, n
        if rm == d.Rounding.STOCHASTIC:
            assert int(state.item()) & 0xFFFFFFFFFFFFFFFF == o_state, n
        seed = want_state


@pytest.mark.parametrize("block", [32, 37])
def test_rejects_stochastic_calls_beyond_the_scratch_size(env, block):
    d, _lib, torch = env
    n = block * (MAX_ITEMS + 1)
    src = torch.ones(n, dtype=torch.float64, device="cuda")
    dst = torch.zeros_like(src)
    state = torch.zeros(1, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    b = d.NumericPolicy.builder("e").input(d.Formats.E4M3).input_rounding(d.Rounding.STOCHASTIC)
    if block != 32:
        b = b.scaling(d.Scaling.MX_BLOCK).scale_block(block)
    p = b.build()
    rc = _noalloc(d, _lib, torch, p, d.Formats.E4M3, d.Rounding.STOCHASTIC, src, dst, state, None,
                  err)
    assert rc == _lib.ENOMEM
    assert "DRIFT_NOALLOC_MAX_ITEMS" in _lib.last_error()
    torch.cuda.synchronize()
    assert float(dst.abs().max()) == 0.0  # nothing ran
    assert int(state.item()) == 0
