"""The no-allocation cast entry point, drift_quantize_dev_noalloc.

It serves host programs that reserve all device memory up front and do not let
a library allocate while they run; its stochastic-rounding scratch lives in a
fixed array inside the library instead of a workspace. These tests call it
through the C ABI on device buffers and hold it to the ordinary entry point,
drift_quantize_dev, bit for bit (the tolerance every cast test here uses), on
two calls in a row so that scratch left over from the first call cannot leak
into the second. The file name sorts last so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


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


@pytest.mark.parametrize("case", ["e2m1-mx32", "e4m3-per-tensor", "e5m2-none"])
def test_two_calls_match_the_allocating_entry_point(env, case):
    d, _lib, torch = env
    F, S = d.Formats, d.Scaling
    f, scaling = {"e2m1-mx32": (F.E2M1, S.MX_BLOCK), "e4m3-per-tensor": (F.E4M3, S.PER_TENSOR),
                  "e5m2-none": (F.E5M2, S.NONE)}[case]
    p = d.NumericPolicy.builder(case).input(f).scaling(scaling).build()
    rm = d.Rounding.STOCHASTIC
    rs = np.random.default_rng(17)
    state = torch.tensor([0x5EED], dtype=torch.int64, device="cuda")
    clamped = torch.zeros(1, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    seed = 0x5EED
    # Two calls in a row on different inputs and sizes, the Rng state carried
    # from the first into the second as a caller sharing one stream would.
    for n in (1_000_003, 70_001):
        x = rs.standard_normal(n) * np.exp(rs.standard_normal(n)) * (3.0 if f is F.E2M1 else 40.0)
        src = torch.from_numpy(x).cuda()
        d_scale = None
        scale = 1.0
        if scaling == S.PER_TENSOR:
            scale = d.Quant.per_tensor_scale(f, float(src.abs().max()))
            d_scale = torch.tensor([scale], dtype=torch.float64, device="cuda")
        want, want_state, want_clamped = _reference(d, torch, p, f, rm, src, d_scale, scale, seed)
        dst = torch.full_like(src, np.nan)
        clamped.zero_()
        rc = _noalloc(d, _lib, torch, p, f, rm, src, dst, state, clamped, err, d_scale, scale)
        assert rc == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = dst.cpu().numpy()
        ref = want.cpu().numpy()
        assert (got.view(np.int64) == ref.view(np.int64)).all()
        assert int(state.item()) == want_state
        assert int(clamped.item()) == want_clamped
        seed = want_state


def test_rejects_calls_beyond_the_scratch_size(env):
    d, _lib, torch = env
    max_items = 1 << 18  # DRIFT_NOALLOC_MAX_ITEMS
    n = 32 * (max_items + 1)
    src = torch.ones(n, dtype=torch.float64, device="cuda")
    dst = torch.zeros_like(src)
    state = torch.zeros(1, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = d.NumericPolicy.builder("e").input(d.Formats.E4M3).build()
    rc = _noalloc(d, _lib, torch, p, d.Formats.E4M3, d.Rounding.STOCHASTIC, src, dst, state, None,
                  err)
    assert rc == _lib.ENOMEM
    assert "DRIFT_NOALLOC_MAX_ITEMS" in _lib.last_error()
    torch.cuda.synchronize()
    assert float(dst.abs().max()) == 0.0  # nothing ran
