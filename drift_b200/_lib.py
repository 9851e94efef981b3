"""ctypes binding of libdrift_b200.so (include/drift_b200.h).

The library is the only compute path: if it cannot be loaded, importing the
package fails. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import os

PKG = Path(__file__).resolve().parent
# DRIFT_B200_LIB names another build of the same library (for instance one
# compiled with different tuning flags); by default the in-tree build is used.
LIB_PATH = Path(os.environ.get("DRIFT_B200_LIB", PKG / "libdrift_b200.so"))

OK, EINVAL, ENAN_FINITE, ECUDA, ETIMEOUT, EUNSUPPORTED, ENOMEM = range(7)

_STATUS_NAMES = {
    EINVAL: "DRIFT_EINVAL", ENAN_FINITE: "DRIFT_ENAN_FINITE", ECUDA: "DRIFT_ECUDA",
    ETIMEOUT: "DRIFT_ETIMEOUT", EUNSUPPORTED: "DRIFT_EUNSUPPORTED", ENOMEM: "DRIFT_ENOMEM",
}


class DriftError(RuntimeError):
    """A non-OK status from the engine. `status` is the DRIFT_* code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class DriftPolicy(ctypes.Structure):
    """struct drift_policy (include/drift_b200.h)."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "input_format", "grad_format", "input_rounding", "grad_rounding", "scaling",
        "scale_block", "amax_history", "mx_headroom", "acc", "order", "acc_block",
        "acc_rounding", "master_fp32", "cast_scores", "cast_probs", "reserved")]


class DriftContraction(ctypes.Structure):
    """struct drift_contraction (include/drift_b200.h)."""

    _fields_ = [(n, ctypes.c_int64) for n in (
        "batch", "rows", "cols", "depth", "a_off", "a_batch", "a_row", "a_k", "b_off", "b_batch",
        "b_col", "b_k", "c_off", "c_batch", "c_row", "c_col")] + [
        ("alpha", ctypes.c_double), ("window", ctypes.c_int32), ("causal", ctypes.c_int32),
        ("accumulate", ctypes.c_int32), ("reserved", ctypes.c_int32)]


# Every exported symbol with its ctypes signature, in header order.
_P = ctypes.POINTER
_vp, _i32, _i64, _d = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_double
_int = ctypes.c_int
SIGNATURES = {
    "drift_open": (_int, [_int, _P(_vp)]),
    "drift_close": (_int, [_vp]),
    "drift_last_error": (ctypes.c_char_p, []),
    "drift_version": (ctypes.c_char_p, []),
    "drift_format_info": (_int, [_int, _P(_d), _P(_d), _P(_d), _P(_i32)]),
    "drift_encode": (_int, [_vp, _int, _int, _vp, _vp, _i64, _P(ctypes.c_uint64)]),
    "drift_decode": (_int, [_vp, _int, _vp, _vp, _i64]),
    "drift_value_table": (_int, [_vp, _int, _vp]),
    "drift_pair_table": (_int, [_vp, _int, _int, ctypes.c_uint64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "drift_value_table_dev": (_int, [_vp, _int, _vp, _vp]),
    "drift_pair_table_dev": (_int, [_vp, _int, _int, ctypes.c_uint64, _i64, _i64, _vp, _vp, _vp,
                                    _vp, _vp]),
    "drift_acc_round": (_int, [_vp, _int, _int, _vp, _vp, _i64, _P(ctypes.c_uint64)]),
    "drift_amax": (_int, [_vp, _vp, _i64, _P(_d)]),
    "drift_per_tensor_scale": (_int, [_int, _d, _P(_d)]),
    "drift_quantize": (_int, [_vp, _P(DriftPolicy), _int, _int, _vp, _vp, _i64, _d,
                              _P(ctypes.c_uint64), _P(_i64)]),
    "drift_gemm": (_int, [_vp, _P(DriftPolicy), _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp,
                          _i64, _i64, _i64, _vp, _vp, _i64, _P(ctypes.c_uint64)]),
    "drift_contract": (_int, [_vp, _P(DriftPolicy), _P(DriftContraction), _vp, _i64, _vp, _i64,
                              _vp, _i64, _P(ctypes.c_uint64)]),
    "drift_contract_dev": (_int, [_vp, _P(DriftPolicy), _P(DriftContraction), _vp, _vp, _vp, _vp,
                                  _vp]),
    "drift_amax_dev": (_int, [_vp, _vp, _i64, _vp, _vp]),
    "drift_quantize_dev": (_int, [_vp, _P(DriftPolicy), _int, _int, _vp, _vp, _i64, _vp, _d,
                                  _vp, _vp, _vp]),
    "drift_quantize_dev_noalloc": (_int, [_P(DriftPolicy), _int, _int, _vp, _vp, _i64, _vp, _d,
                                          _vp, _vp, _vp, _vp]),
    "drift_quantize_rows_dev": (_int, [_vp, _P(DriftPolicy), _int, _int, _vp, _vp, _i64, _i64,
                                       _vp, _vp]),
    "drift_quantize_draws_dev": (_int, [_vp, _P(DriftPolicy), _int, _int, _vp, _i64, _vp, _d,
                                        _vp, _vp]),
    "drift_per_tensor_scale_dev": (_int, [_vp, _int, _vp, _vp, _vp]),
    "drift_gemm_dev": (_int, [_vp, _P(DriftPolicy), _i64, _i64, _i64, _vp, _i64, _i64, _vp,
                              _i64, _i64, _vp, _vp, _i64, _vp, _vp]),
    "drift_gemm_route": (_int, [_vp, _P(_int), _vp]),
    "drift_gemm_launches": (_int, [_vp, _P(_int)]),
    "drift_set_thin_tiles": (_int, [_vp, _i64]),
    "drift_error_sums_dev": (_int, [_vp, _vp, _vp, _i64, _vp, _vp]),
    "drift_radix_hist_dev": (_int, [_vp, _vp, _vp, _i64, _int, _vp, _vp, _vp]),
    "drift_radix_select_dev": (_int, [_vp, _int, _vp, _vp, _vp]),
    "drift_group_kth_rel_error_dev": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "drift_real_dot_sweep": (_int, [_vp, _vp, _int, _i64, _i64, _i64, _vp, _vp, ctypes.c_uint64,
                                    _vp]),
    "drift_embed_gather_dev": (_int, [_vp, _vp, _i64, _vp, _i64, _i64, _vp, _vp]),
    "drift_embed_grad_dev": (_int, [_vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp]),
    "drift_bias_grad_dev": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "drift_tanh_backward_dev": (_int, [_vp, _vp, _vp, _i64, _vp]),
    "drift_scale_for_dev": (_int, [_vp, _int, _vp, _vp, _i32, _vp, _vp, _vp]),
    "drift_adam_dev": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _d, _i32, _vp]),
    "drift_probe_fp64": (_int, [_vp, _P(_d)]),
    "drift_probe_fp32": (_int, [_vp, _P(_d)]),
    "drift_check_dev": (_int, [_vp, _vp]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Loads the engine library, building it first if it is missing or stale."""
    global _lib
    with _lock:
        if _lib is None:
            from . import build as _build

            if LIB_PATH == _build.LIB and not _build.up_to_date():
                _build.build()
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return load().drift_last_error().decode()


def check(status: int) -> None:
    if status != OK:
        raise DriftError(status, last_error())


class Context:
    """A drift_ctx: one CUDA stream and workspace on one device. Use one per
    thread (the C library's rule); `Context.current()` gives each thread its
    own on device 0, or on the device set with `Context.use_device`."""

    _tls = threading.local()
    _default_device = 0

    def __init__(self, device: int = 0):
        self.device = device
        h = ctypes.c_void_p()
        check(load().drift_open(device, ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            load().drift_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @classmethod
    def use_device(cls, device: int) -> None:
        cls._default_device = device
        cls._tls.ctx = None

    @classmethod
    def current(cls) -> "Context":
        ctx = getattr(cls._tls, "ctx", None)
        if ctx is None or ctx.handle is None:
            ctx = Context(cls._default_device)
            cls._tls.ctx = ctx
        return ctx
