"""Statistics of an emulated GEMM against its exact twin, on the device.

RMS ratio (RealDotSweep.java:142, :149-155) from two sums, and exact order
statistics of the relative error (the medians of DotSweep.java:152-153 and
RealDotSweep.java:140-141) by radix selection. With a process group, every
rank's outputs take part: the per-pass histograms and the sums are
all-reduced, so all ranks select the same element.
"""
from __future__ import annotations

import ctypes
import struct

from . import _lib
from .kernel import _stream_ptr, _tptr

RADIX_PASSES = 6
RADIX_BINS = 2048


def select_rel_error_dev(got, exact, k: int, state, hist, dist=None, stream=None,
                         ctx=None) -> None:
    """Leaves the bit pattern of the k-th smallest (0-based) relative error in
    state[0] (an int64 tensor of two on the device), without a host wait.
    `hist` is device scratch of RADIX_BINS int64. With `dist`, all ranks'
    elements take part."""
    ctx = ctx or _lib.Context.current()
    state[0] = 0
    state[1] = k
    L = _lib.load()
    for ps in range(RADIX_PASSES):
        _lib.check(L.drift_radix_hist_dev(ctx.handle, _tptr(got), _tptr(exact), got.numel(), ps,
                                          _tptr(state), _tptr(hist), _stream_ptr(stream)))
        if dist is not None:
            dist.all_reduce(hist)
        _lib.check(L.drift_radix_select_dev(ctx.handle, ps, _tptr(hist), _tptr(state),
                                            _stream_ptr(stream)))


def bits_to_double(bits: int) -> float:
    return struct.unpack("<d", struct.pack("<Q", int(bits) & 0xFFFFFFFFFFFFFFFF))[0]


def kth_rel_error(got, exact, k: int, dist=None, stream=None, ctx=None) -> float:
    """The k-th smallest (0-based) of |got - exact| / |exact| over all
    elements (of all ranks when `dist` is a process group)."""
    import torch

    state = torch.zeros(2, dtype=torch.int64, device=got.device)
    hist = torch.empty(RADIX_BINS, dtype=torch.int64, device=got.device)
    select_rel_error_dev(got, exact, k, state, hist, dist, stream, ctx)
    return bits_to_double(state[0].item())


def upper_median_rel_error(got, exact, total: int, dist=None, **kw) -> float:
    """DotSweep's summary statistic: errs[k/2] of the sorted errors."""
    return kth_rel_error(got, exact, total // 2, dist, **kw)


def true_median_rel_error(got, exact, total: int, dist=None, **kw) -> float:
    """RealDotSweep's median: the mean of the two middle values."""
    lo = kth_rel_error(got, exact, total // 2 - 1, dist, **kw)
    hi = kth_rel_error(got, exact, total // 2, dist, **kw)
    return 0.5 * (lo + hi)


def group_kth_rel_error_dev(got, exact, groups: int, n: int, k: int, out, stream=None,
                            ctx=None) -> None:
    """out[g] = the k-th smallest (0-based) relative error within group g of
    n consecutive outputs (n <= 4096), for `groups` groups in one launch."""
    ctx = ctx or _lib.Context.current()
    _lib.check(_lib.load().drift_group_kth_rel_error_dev(ctx.handle, _tptr(got), _tptr(exact),
                                                         groups, n, k, _tptr(out),
                                                         _stream_ptr(stream)))
