"""Kernel layer: NumericPolicy, Quant, Dot, and the whole-GEMM entry points.

Mirrors the reference's io.drift.kernel package
(java/src/main/java/io/drift/kernel/): the same names, argument meanings and
errors. Quant.quantize and Dot.dot run on the GPU through the engine's C ABI.
`gemm` / `gemm_dev` are the whole-matmul calls that replace the reference's
(i, o) loops over Dot.dot (java/.../train/Pass.java:200-232).
"""
from __future__ import annotations

import ctypes
import dataclasses
from enum import IntEnum
from typing import Optional

import numpy as np

from . import _lib
from .fmt import Formats, MiniFloat, Rng, Rounding


class Acc(IntEnum):
    """NumericPolicy.Acc (NumericPolicy.java:26-41)."""

    FP64 = 0
    FP32 = 1
    FP16 = 2
    BF16 = 3

    def format(self) -> Optional[MiniFloat]:
        return {Acc.FP16: Formats.FP16, Acc.BF16: Formats.BF16}.get(self)


class Order(IntEnum):
    """NumericPolicy.Order (NumericPolicy.java:44-53)."""

    SEQUENTIAL = 0
    REVERSED = 1
    PAIRWISE = 2
    BLOCKED = 3


class Scaling(IntEnum):
    """NumericPolicy.Scaling (NumericPolicy.java:56-63)."""

    NONE = 0
    PER_TENSOR = 1
    MX_BLOCK = 2


@dataclasses.dataclass(frozen=True)
class NumericPolicy:
    """Every arithmetic decision a matmul makes
    (java/src/main/java/io/drift/kernel/NumericPolicy.java:58-96).
    Field defaults are NumericPolicy.Builder's (:180-203)."""

    name: str
    input_format: Optional[MiniFloat] = None
    grad_format: Optional[MiniFloat] = None
    input_rounding: Rounding = Rounding.NEAREST_EVEN
    grad_rounding: Optional[Rounding] = None
    scaling: Scaling = Scaling.NONE
    scale_block: int = 32
    amax_history: int = 0
    mx_headroom: int = 0
    acc: Acc = Acc.FP32
    order: Order = Order.SEQUENTIAL
    acc_block: int = 32
    acc_rounding: Rounding = Rounding.NEAREST_EVEN
    master_fp32: bool = True
    cast_scores: bool = True
    cast_probs: bool = True

    def grad_cast_rounding(self) -> Rounding:
        """NumericPolicy.gradCastRounding (:101-103)."""
        return self.grad_rounding if self.grad_rounding is not None else self.input_rounding

    def grad_cast_format(self) -> Optional[MiniFloat]:
        """NumericPolicy.gradCastFormat (:106-108)."""
        return self.grad_format if self.grad_format is not None else self.input_format

    @staticmethod
    def exact() -> "NumericPolicy":
        """FP64 throughout, nothing cast (:128-130)."""
        return NumericPolicy("exact", acc=Acc.FP64, master_fp32=False)

    @staticmethod
    def builder(name: str) -> "Builder":
        return Builder(name)

    def to_builder(self, new_name: str) -> "Builder":
        b = Builder(new_name)
        b._f = dataclasses.asdict(self) | {"name": new_name}
        # asdict deep-copies MiniFloat objects; keep the shared instances.
        b._f["input_format"] = self.input_format
        b._f["grad_format"] = self.grad_format
        return b

    def describe(self) -> str:
        """NumericPolicy.describe (:139-156)."""
        g = self.grad_cast_format()
        return (f"name={self.name} input={self.input_format.name if self.input_format else 'none'}"
                f" grad={g.name if g else 'none'} inputRounding={self.input_rounding.name}"
                f" gradRounding={self.grad_cast_rounding().name} scaling={self.scaling.name}"
                f" scaleBlock={self.scale_block} amaxHistory={self.amax_history}"
                f" mxHeadroom={self.mx_headroom} acc={self.acc.name} order={self.order.name}"
                f" accBlock={self.acc_block} accRounding={self.acc_rounding.name}"
                f" masterFp32={str(self.master_fp32).lower()}"
                f" castScores={str(self.cast_scores).lower()}"
                f" castProbs={str(self.cast_probs).lower()}")

    def to_c(self) -> _lib.DriftPolicy:
        """The POD this policy crosses the C ABI as (include/drift_b200.h)."""
        return _lib.DriftPolicy(
            self.input_format.id if self.input_format else -1,
            self.grad_format.id if self.grad_format else -1,
            int(self.input_rounding),
            int(self.grad_rounding) if self.grad_rounding is not None else -1,
            int(self.scaling), self.scale_block, self.amax_history, self.mx_headroom,
            int(self.acc), int(self.order), self.acc_block, int(self.acc_rounding),
            int(self.master_fp32), int(self.cast_scores), int(self.cast_probs), 0)

    def __str__(self) -> str:
        return self.name


class Builder:
    """NumericPolicy.Builder (NumericPolicy.java:180-221)."""

    def __init__(self, name: str):
        self._f = {"name": name}

    def _set(self, k, v) -> "Builder":
        self._f[k] = v
        return self

    def input(self, f): return self._set("input_format", f)
    def grad(self, f): return self._set("grad_format", f)
    def input_rounding(self, r): return self._set("input_rounding", Rounding(r))
    def grad_rounding(self, r): return self._set("grad_rounding", None if r is None else Rounding(r))
    def scaling(self, s): return self._set("scaling", Scaling(s))
    def scale_block(self, n): return self._set("scale_block", int(n))
    def amax_history(self, n): return self._set("amax_history", int(n))
    def mx_headroom(self, n): return self._set("mx_headroom", int(n))
    def acc(self, a): return self._set("acc", Acc(a))
    def order(self, o): return self._set("order", Order(o))
    def acc_block(self, n): return self._set("acc_block", int(n))
    def acc_rounding(self, r): return self._set("acc_rounding", Rounding(r))
    def master_fp32(self, b): return self._set("master_fp32", bool(b))
    def cast_scores(self, b): return self._set("cast_scores", bool(b))
    def cast_probs(self, b): return self._set("cast_probs", bool(b))

    def build(self) -> NumericPolicy:
        return NumericPolicy(**self._f)


def _state_in(rng: Optional[Rng]):
    return ctypes.c_uint64(rng.state()) if rng is not None else None


def _state_out(rng: Optional[Rng], st) -> None:
    if rng is not None:
        rng.reseed(st.value)


def _dptr(a: np.ndarray) -> int:
    if a.dtype != np.float64 or not a.flags.c_contiguous:
        raise TypeError("expected a C-contiguous float64 array")
    return a.ctypes.data


class Quant:
    """java/src/main/java/io/drift/kernel/Quant.java."""

    @staticmethod
    def amax(x, off: int = 0, n: Optional[int] = None) -> float:
        """Quant.amax (Quant.java:25-34): largest magnitude, NaN ignored."""
        x = np.asarray(x, dtype=np.float64).reshape(-1)
        n = x.size - off if n is None else n
        span = np.ascontiguousarray(x[off:off + n])
        out = ctypes.c_double()
        _lib.check(_lib.load().drift_amax(_lib.Context.current().handle, span.ctypes.data,
                                          span.size, ctypes.byref(out)))
        return out.value

    @staticmethod
    def per_tensor_scale(f: MiniFloat, amax: float) -> float:
        """Quant.perTensorScale (Quant.java:37-42)."""
        out = ctypes.c_double()
        _lib.check(_lib.load().drift_per_tensor_scale(f.id, float(amax), ctypes.byref(out)))
        return out.value

    @staticmethod
    def quantize(src, src_off: int, dst: np.ndarray, dst_off: int, n: int,
                 f: Optional[MiniFloat], p: NumericPolicy, scale: float, rng: Optional[Rng],
                 rm: Optional[Rounding] = None) -> int:
        """Quant.quantize (Quant.java:50-82): casts src[src_off:src_off+n] into
        dst[dst_off:...] as effective doubles and returns the clamp count.
        `rm` defaults to the policy's input rounding, as the 9-argument Java
        overload does."""
        rm = p.input_rounding if rm is None else Rounding(rm)
        s = np.ascontiguousarray(np.asarray(src, dtype=np.float64).reshape(-1)[src_off:src_off + n])
        # The engine writes into dst itself when dst is contiguous float64
        # (no temporary, no second host copy).
        direct = (isinstance(dst, np.ndarray) and dst.dtype == np.float64
                  and dst.flags.c_contiguous)
        out = dst.reshape(-1)[dst_off:dst_off + n] if direct else np.empty(n, dtype=np.float64)
        st = _state_in(rng)
        clamped = ctypes.c_int64()
        pc = p.to_c()
        _lib.check(_lib.load().drift_quantize(
            _lib.Context.current().handle, ctypes.byref(pc), f.id if f is not None else -1,
            int(rm), s.ctypes.data, out.ctypes.data, n, float(scale),
            ctypes.byref(st) if st is not None else None, ctypes.byref(clamped)))
        _state_out(rng, st)
        if not direct:
            dst.reshape(-1)[dst_off:dst_off + n] = out
        return int(clamped.value)


class Dot:
    """java/src/main/java/io/drift/kernel/Dot.java."""

    @staticmethod
    def dot(a, a_off: int, a_stride: int, b, b_off: int, b_stride: int, n: int,
            p: NumericPolicy, rng: Optional[Rng] = None) -> float:
        """Dot.dot (Dot.java:26-35): one inner product under the policy."""
        out = np.empty((1, 1), dtype=np.float64)
        gemm(p, 1, 1, n, a, a_off, 0, a_stride, b, b_off, 0, b_stride, out=out, rng=rng)
        return float(out[0, 0])

    @staticmethod
    def round(x, acc: Acc, rm: Rounding, rng: Optional[Rng] = None):
        """Dot.round (Dot.java:141-182) for FP16/BF16, element-wise."""
        scalar = np.ndim(x) == 0
        v = np.ascontiguousarray(np.asarray(x, dtype=np.float64)).reshape(-1)
        y = np.empty_like(v)
        st = _state_in(rng)
        _lib.check(_lib.load().drift_acc_round(_lib.Context.current().handle, int(acc), int(rm),
                                               v.ctypes.data, y.ctypes.data, v.size,
                                               ctypes.byref(st) if st is not None else None))
        _state_out(rng, st)
        return float(y[0]) if scalar else y.reshape(np.shape(x))


def gemm(p: NumericPolicy, M: int, N: int, K: int, A, a_off: int, a_rs: int, a_ks: int,
         B, b_off: int, b_rs: int, b_ks: int, bias=None, out: Optional[np.ndarray] = None,
         rng: Optional[Rng] = None) -> np.ndarray:
    """C[i, o] = Dot.dot(A, a_off + i*a_rs, a_ks, B, b_off + o*b_rs, b_ks, K, p, rng)
    (+ bias[o]) over host arrays: the loops of Pass.java:200-232 in one call."""
    A = np.ascontiguousarray(np.asarray(A, dtype=np.float64)).reshape(-1)
    B = np.ascontiguousarray(np.asarray(B, dtype=np.float64)).reshape(-1)
    if out is None:
        out = np.empty((M, N), dtype=np.float64)
    c_rs = out.strides[0] // 8 if out.ndim == 2 else N
    bptr = None
    if bias is not None:
        bias = np.ascontiguousarray(np.asarray(bias, dtype=np.float64))
        bptr = bias.ctypes.data
    st = _state_in(rng)
    pc = p.to_c()
    _lib.check(_lib.load().drift_gemm(
        _lib.Context.current().handle, ctypes.byref(pc), M, N, K, A.ctypes.data, a_off, a_rs,
        a_ks, B.ctypes.data, b_off, b_rs, b_ks, bptr, out.ctypes.data, c_rs,
        ctypes.byref(st) if st is not None else None))
    _state_out(rng, st)
    return out


class Window(IntEnum):
    """The k window of row i of a contraction (include/drift_b200.h)."""

    FULL = 0     # [0, depth): score and dProb matmuls (AttnPass.java:245-255, :373-381)
    PREFIX = 1   # [0, i]: context and dq matmuls (:283-288, :412-417)
    SUFFIX = 2   # [i, depth): dv and dk matmuls (:382-388, :419-424)


def contraction(*, rows: int, cols: int, depth: int, a_row: int, a_k: int, b_col: int, b_k: int,
                c_row: int, batch: int = 1, a_off: int = 0, a_batch: int = 0, b_off: int = 0,
                b_batch: int = 0, c_off: int = 0, c_batch: int = 0, c_col: int = 1,
                alpha: float = 1.0, window: Window = Window.FULL, causal: bool = False,
                accumulate: bool = False) -> "_lib.DriftContraction":
    """A drift_contraction: output (t, i, o) at C[c_off + t*c_batch + i*c_row +
    o*c_col] is Dot.dot(A, a_off + t*a_batch + i*a_row + lo*a_k, a_k,
    B, b_off + t*b_batch + o*b_col + lo*b_k, b_k, n) * alpha (added into C when
    accumulating) over row i's window (lo, n); 0.0 for o > i when causal."""
    return _lib.DriftContraction(batch, rows, cols, depth, a_off, a_batch, a_row, a_k, b_off,
                                 b_batch, b_col, b_k, c_off, c_batch, c_row, c_col, float(alpha),
                                 int(window), int(bool(causal)), int(bool(accumulate)), 0)


def contract(p: NumericPolicy, op, A: np.ndarray, B: np.ndarray, C: np.ndarray,
             rng: Optional[Rng] = None) -> np.ndarray:
    """One contraction over host arrays (flat float64), C updated in place
    and returned: the Dot.dot loops of AttnPass.java:245-427 in one call."""
    A = np.ascontiguousarray(np.asarray(A, dtype=np.float64)).reshape(-1)
    B = np.ascontiguousarray(np.asarray(B, dtype=np.float64)).reshape(-1)
    if C.dtype != np.float64 or not C.flags.c_contiguous:
        raise TypeError("C must be a contiguous float64 array")
    st = _state_in(rng)
    pc = p.to_c()
    _lib.check(_lib.load().drift_contract(
        _lib.Context.current().handle, ctypes.byref(pc), ctypes.byref(op), A.ctypes.data, A.size,
        B.ctypes.data, B.size, C.ctypes.data, C.size,
        ctypes.byref(st) if st is not None else None))
    _state_out(rng, st)
    return C


# ----------------------------------------------------------- device-resident calls
# These take torch CUDA tensors (float64) and run on torch's current stream.

def _stream_ptr(stream=None):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _tptr(t) -> int:
    if t is None:
        return None
    if not t.is_cuda:
        raise TypeError("expected a CUDA tensor")
    return t.data_ptr()


def gemm_dev(p: NumericPolicy, A, B, C, *, M=None, N=None, K=None, a_rs=None, a_ks=1,
             b_rs=None, b_ks=1, c_rs=None, bias=None, d_rng_state=None, stream=None,
             ctx=None) -> None:
    """The contraction on device tensors. Defaults describe the forward layout:
    A is M x K and B is N x K, both K-contiguous; C is M x N. A stochastic
    accumulator needs d_rng_state (an int64 device tensor of one element
    holding the Rng state's bits), which it advances."""
    M = A.shape[0] if M is None else M
    K = A.shape[1] if K is None else K
    N = B.shape[0] if N is None else N
    a_rs = K if a_rs is None else a_rs
    b_rs = K if b_rs is None else b_rs
    c_rs = N if c_rs is None else c_rs
    ctx = ctx or _lib.Context.current()
    pc = p.to_c()
    _lib.check(_lib.load().drift_gemm_dev(ctx.handle, ctypes.byref(pc), M, N, K, _tptr(A), a_rs,
                                          a_ks, _tptr(B), b_rs, b_ks, _tptr(bias), _tptr(C), c_rs,
                                          _tptr(d_rng_state), _stream_ptr(stream)))


def contract_dev(p: NumericPolicy, op, A, B, C, *, d_rng_state=None, stream=None,
                 ctx=None) -> None:
    """One contraction on device tensors (float64, addressed through `op`'s
    offsets and strides); a stochastic accumulator needs d_rng_state."""
    ctx = ctx or _lib.Context.current()
    pc = p.to_c()
    _lib.check(_lib.load().drift_contract_dev(ctx.handle, ctypes.byref(pc), ctypes.byref(op),
                                              _tptr(A), _tptr(B), _tptr(C), _tptr(d_rng_state),
                                              _stream_ptr(stream)))


def quantize_dev(p: NumericPolicy, f: Optional[MiniFloat], rm: Rounding, src, dst, *,
                 scale: float = 1.0, d_scale=None, d_rng_state=None, d_clamped=None,
                 stream=None, ctx=None) -> None:
    """Quant.quantize on device tensors; clamp counts are added to d_clamped
    (int64 tensor of one element) and the Rng state lives in d_rng_state
    (int64 tensor of one element holding the state's bits)."""
    ctx = ctx or _lib.Context.current()
    pc = p.to_c()
    _lib.check(_lib.load().drift_quantize_dev(
        ctx.handle, ctypes.byref(pc), f.id if f is not None else -1, int(rm), _tptr(src),
        _tptr(dst), src.numel(), _tptr(d_scale), float(scale), _tptr(d_rng_state),
        _tptr(d_clamped), _stream_ptr(stream)))


def quantize_rows_dev(p: NumericPolicy, f: Optional[MiniFloat], rm: Rounding, src, dst, *,
                      d_clamped=None, stream=None, ctx=None) -> None:
    """Each row of the 2-D tensor src cast as its own tensor (its own
    per-tensor scale under PER_TENSOR scaling), one launch; clamps added to
    d_clamped[row]. Nearest-even or truncate, no MX scaling."""
    ctx = ctx or _lib.Context.current()
    pc = p.to_c()
    rows, length = src.shape
    _lib.check(_lib.load().drift_quantize_rows_dev(
        ctx.handle, ctypes.byref(pc), f.id if f is not None else -1, int(rm), _tptr(src),
        _tptr(dst), rows, length, _tptr(d_clamped), _stream_ptr(stream)))


def amax_dev(x, d_amax, *, stream=None, ctx=None) -> None:
    ctx = ctx or _lib.Context.current()
    _lib.check(_lib.load().drift_amax_dev(ctx.handle, _tptr(x), x.numel(), _tptr(d_amax),
                                          _stream_ptr(stream)))


def per_tensor_scale_dev(f: MiniFloat, d_amax, d_scale, *, stream=None, ctx=None) -> None:
    """Quant.perTensorScale from a device amax into a device scale."""
    ctx = ctx or _lib.Context.current()
    _lib.check(_lib.load().drift_per_tensor_scale_dev(ctx.handle, f.id, _tptr(d_amax),
                                                      _tptr(d_scale), _stream_ptr(stream)))


def error_sums_dev(got, exact, d_sums, *, stream=None, ctx=None) -> None:
    """Adds sum((got-exact)^2) and sum(exact^2) into the 2-element tensor d_sums."""
    ctx = ctx or _lib.Context.current()
    _lib.check(_lib.load().drift_error_sums_dev(ctx.handle, _tptr(got), _tptr(exact),
                                                got.numel(), _tptr(d_sums), _stream_ptr(stream)))


ROUTE_DOUBLE, ROUTE_FP32, ROUTE_SCANNED, ROUTE_STAGED, ROUTE_PROVEN = 0, 1, 2, 3, 4


def gemm_route(stream=None, ctx=None) -> int:
    """The path of the context's last non-stochastic GEMM: ROUTE_FP32 for the
    FP32 pipe (narrow products under an FP32 accumulator), ROUTE_SCANNED for a
    candidate whose operands kept it on the double-precision contraction,
    ROUTE_STAGED for one output per thread (a call too thin to fill the GPU
    with 64 x 64 tiles), ROUTE_PROVEN for the double-precision contraction
    of an FP32/BF16 accumulator whose operand scan proved every partial sum in
    range (no per-step checks), ROUTE_DOUBLE for the tiled double-precision
    contraction alone. Synchronises the stream."""
    ctx = ctx or _lib.Context.current()
    out = ctypes.c_int()
    _lib.check(_lib.load().drift_gemm_route(ctx.handle, ctypes.byref(out), _stream_ptr(stream)))
    return out.value


def gemm_launches(ctx=None) -> int:
    """How many kernels the context's last non-stochastic GEMM call queued
    (scans, decisions and both builds of a scanned route included)."""
    ctx = ctx or _lib.Context.current()
    out = ctypes.c_int()
    _lib.check(_lib.load().drift_gemm_launches(ctx.handle, ctypes.byref(out)))
    return out.value


def set_thin_tiles(tiles: int, ctx=None) -> None:
    """GEMM calls with fewer than `tiles` 64 x 64 output tiles run one output
    per thread (ROUTE_STAGED); negative restores the default (measured per
    policy: under two thirds of a tile per SM for sequential, reversed and
    32-aligned blocked orders with a rounding accumulator, a third otherwise),
    0 sends every call to the tiled kernel. Results do not change."""
    ctx = ctx or _lib.Context.current()
    _lib.check(_lib.load().drift_set_thin_tiles(ctx.handle, int(tiles)))


def probe_fp64(ctx=None) -> float:
    """The FP64 pipe's measured DMUL+DADD rate, in operations per second."""
    ctx = ctx or _lib.Context.current()
    out = ctypes.c_double()
    _lib.check(_lib.load().drift_probe_fp64(ctx.handle, ctypes.byref(out)))
    return out.value


def probe_fp32(ctx=None) -> float:
    """The FP32 pipe's measured FFMA rate, in fused multiply-adds per second."""
    ctx = ctx or _lib.Context.current()
    out = ctypes.c_double()
    _lib.check(_lib.load().drift_probe_fp32(ctx.handle, ctypes.byref(out)))
    return out.value


def check_dev(stream=None, ctx=None) -> None:
    """Raises the first device-side error since the last check (synchronises)."""
    ctx = ctx or _lib.Context.current()
    _lib.check(_lib.load().drift_check_dev(ctx.handle, _stream_ptr(stream)))
