"""ctypes front end of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: the oracle the CUDA engine is compared against.
Only tests/, the smoke check and bench.py's CPU-baseline leg import this
module. It restates the reference's Java arithmetic in C; see
drift_oracle.c for the line-by-line citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB = None

# Format ids and enum ordinals, as in include/drift_b200.h.
E4M3, E5M2, E2M1, E3M2, E2M3, FP16, BF16 = range(7)
FMT_NONE = -1
NEAREST_EVEN, STOCHASTIC, TRUNCATE = 0, 1, 2
SCALE_NONE, PER_TENSOR, MX_BLOCK = 0, 1, 2
ACC_FP64, ACC_FP32, ACC_FP16, ACC_BF16 = 0, 1, 2, 3
SEQUENTIAL, REVERSED, PAIRWISE, BLOCKED = 0, 1, 2, 3


class OraclePolicy(ctypes.Structure):
    """Byte layout of drift_policy (include/drift_b200.h)."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "input_format", "grad_format", "input_rounding", "grad_rounding",
        "scaling", "scale_block", "amax_history", "mx_headroom", "acc",
        "order", "acc_block", "acc_rounding", "master_fp32", "cast_scores",
        "cast_probs", "reserved")]


def policy(input_format=FMT_NONE, grad_format=FMT_NONE, input_rounding=NEAREST_EVEN,
           grad_rounding=-1, scaling=SCALE_NONE, scale_block=32, amax_history=0,
           mx_headroom=0, acc=ACC_FP32, order=SEQUENTIAL, acc_block=32,
           acc_rounding=NEAREST_EVEN) -> OraclePolicy:
    """A policy with NumericPolicy.Builder's defaults
    (java/src/main/java/io/drift/kernel/NumericPolicy.java:180-203)."""
    return OraclePolicy(input_format, grad_format, input_rounding, grad_rounding,
                        scaling, scale_block, amax_history, mx_headroom, acc, order,
                        acc_block, acc_rounding, 1, 1, 1, 0)


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (a few seconds)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _HERE / "liboracle.so"


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = _HERE / "liboracle.so"
        src = _HERE / "drift_oracle.c"
        if not path.exists() or path.stat().st_mtime < src.stat().st_mtime:
            build()
        L = ctypes.CDLL(str(path))
        P = ctypes.POINTER
        d, i64, i32, u64 = ctypes.c_double, ctypes.c_int64, ctypes.c_int32, ctypes.c_uint64
        vp = ctypes.c_void_p
        L.o_format_info.argtypes = [ctypes.c_int, P(d), P(d), P(d), P(i32)]
        L.o_rng_next_long.argtypes = [P(u64)]
        L.o_rng_next_long.restype = u64
        L.o_rng_next_double.argtypes = [P(u64)]
        L.o_rng_next_double.restype = d
        L.o_encode.argtypes = [ctypes.c_int, ctypes.c_int, vp, vp, i64, P(u64)]
        L.o_decode.argtypes = [ctypes.c_int, vp, vp, i64]
        L.o_acc_round.argtypes = [ctypes.c_int, ctypes.c_int, vp, vp, i64, P(u64)]
        L.o_amax.argtypes = [vp, i64]
        L.o_amax.restype = d
        L.o_per_tensor_scale.argtypes = [ctypes.c_int, d]
        L.o_per_tensor_scale.restype = d
        L.o_quantize.argtypes = [P(OraclePolicy), ctypes.c_int, ctypes.c_int, vp, vp, i64, d,
                                 P(u64), P(i64)]
        L.o_dot.argtypes = [vp, i64, i64, vp, i64, i64, i64, P(OraclePolicy), P(u64),
                            P(ctypes.c_int)]
        L.o_dot.restype = d
        L.o_gemm.argtypes = [P(OraclePolicy), i64, i64, i64, vp, i64, i64, i64, vp, i64, i64,
                             i64, vp, vp, i64, P(u64), ctypes.c_int]
        L.o_contract.argtypes = [P(OraclePolicy), vp, vp, vp, vp, P(u64)]
        L.o_dotsweep_fill.argtypes = [vp, vp, i64, i64]
        _LIB = L
    return _LIB


class OracleError(RuntimeError):
    def __init__(self, status: int):
        super().__init__(f"oracle status {status}")
        self.status = status


def _check(st: int) -> None:
    if st:
        raise OracleError(st)


def _dptr(a: np.ndarray) -> int:
    assert a.dtype == np.float64 and a.flags.c_contiguous
    return a.ctypes.data


def format_info(fmt: int):
    mx, mn, ms, w = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int32()
    _check(lib().o_format_info(fmt, mx, mn, ms, w))
    return mx.value, mn.value, ms.value, w.value


def _rng(state):
    return None if state is None else ctypes.c_uint64(state & 0xFFFFFFFFFFFFFFFF)


def encode(fmt: int, rm: int, v, rng_state=None):
    """MiniFloat.encode over an array. Returns (codes int32, new rng state)."""
    v = np.ascontiguousarray(v, dtype=np.float64)
    codes = np.zeros(v.shape, dtype=np.int32)
    r = _rng(rng_state)
    _check(lib().o_encode(fmt, rm, _dptr(v), codes.ctypes.data, v.size,
                          None if r is None else ctypes.byref(r)))
    return codes, (None if r is None else r.value)


def decode(fmt: int, codes):
    codes = np.ascontiguousarray(codes, dtype=np.int32)
    out = np.zeros(codes.shape, dtype=np.float64)
    _check(lib().o_decode(fmt, codes.ctypes.data, out.ctypes.data, codes.size))
    return out


def acc_round(acc: int, rm: int, x, rng_state=None):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.zeros_like(x)
    r = _rng(rng_state)
    _check(lib().o_acc_round(acc, rm, _dptr(x), y.ctypes.data, x.size,
                             None if r is None else ctypes.byref(r)))
    return y, (None if r is None else r.value)


def amax(x) -> float:
    x = np.ascontiguousarray(x, dtype=np.float64)
    return lib().o_amax(_dptr(x), x.size)


def per_tensor_scale(fmt: int, amax_value: float) -> float:
    return lib().o_per_tensor_scale(fmt, amax_value)


def quantize(p: OraclePolicy, fmt: int, rm: int, src, scale: float = 1.0, rng_state=None):
    """Quant.quantize. Returns (dst, clamped, new rng state)."""
    src = np.ascontiguousarray(src, dtype=np.float64)
    dst = np.zeros_like(src)
    r = _rng(rng_state)
    cl = ctypes.c_int64()
    _check(lib().o_quantize(ctypes.byref(p), fmt, rm, _dptr(src), dst.ctypes.data, src.size,
                            scale, None if r is None else ctypes.byref(r), ctypes.byref(cl)))
    return dst, cl.value, (None if r is None else r.value)


def dot(a, a_off, a_stride, b, b_off, b_stride, n, p: OraclePolicy, rng_state=None):
    a = np.ascontiguousarray(a, dtype=np.float64)
    b = np.ascontiguousarray(b, dtype=np.float64)
    r = _rng(rng_state)
    err = ctypes.c_int()
    v = lib().o_dot(_dptr(a), a_off, a_stride, _dptr(b), b_off, b_stride, n, ctypes.byref(p),
                    None if r is None else ctypes.byref(r), ctypes.byref(err))
    _check(err.value)
    return v, (None if r is None else r.value)


def gemm(p: OraclePolicy, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks, bias=None,
         rng_state=None, threads: int = 1, C=None, c_rs=None):
    """The (i, o) loop over Dot.dot. Returns (C, new rng state)."""
    A = np.ascontiguousarray(A, dtype=np.float64)
    B = np.ascontiguousarray(B, dtype=np.float64)
    if C is None:
        C = np.zeros((M, N), dtype=np.float64)
        c_rs = N
    bptr = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float64)
        bptr = _dptr(bias)
    r = _rng(rng_state)
    _check(lib().o_gemm(ctypes.byref(p), M, N, K, _dptr(A), a_off, a_rs, a_ks, _dptr(B), b_off,
                        b_rs, b_ks, bptr, C.ctypes.data, c_rs,
                        None if r is None else ctypes.byref(r), threads))
    return C, (None if r is None else r.value)


class OracleContraction(ctypes.Structure):
    """Byte layout of drift_contraction (include/drift_b200.h)."""

    _fields_ = [(n, ctypes.c_int64) for n in (
        "batch", "rows", "cols", "depth", "a_off", "a_batch", "a_row", "a_k", "b_off", "b_batch",
        "b_col", "b_k", "c_off", "c_batch", "c_row", "c_col")] + [
        ("alpha", ctypes.c_double), ("window", ctypes.c_int32), ("causal", ctypes.c_int32),
        ("accumulate", ctypes.c_int32), ("reserved", ctypes.c_int32)]


def contract(p: OraclePolicy, op, A, B, C, rng_state=None):
    """AttnPass's loops for one contraction (op: any ctypes structure with
    drift_contraction's layout). C (flat float64) is updated in place.
    Returns the new rng state."""
    A = np.ascontiguousarray(A, dtype=np.float64)
    B = np.ascontiguousarray(B, dtype=np.float64)
    assert C.dtype == np.float64 and C.flags.c_contiguous
    r = _rng(rng_state)
    _check(lib().o_contract(ctypes.byref(p), ctypes.addressof(op), _dptr(A), _dptr(B), C.ctypes.data,
                            None if r is None else ctypes.byref(r)))
    return None if r is None else r.value


def dotsweep_fill(n: int, seed: int):
    """DotSweep.fill(a, b, seed) restated (java.util.Random + host libm)."""
    a = np.zeros(n, dtype=np.float64)
    b = np.zeros(n, dtype=np.float64)
    lib().o_dotsweep_fill(a.ctypes.data, b.ctypes.data, n, seed)
    return a, b


def rng_next_double(state: int):
    r = ctypes.c_uint64(state & 0xFFFFFFFFFFFFFFFF)
    v = lib().o_rng_next_double(ctypes.byref(r))
    return v, r.value
