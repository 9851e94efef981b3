"""Format layer: MiniFloat, Formats, Rounding, Rng.

Mirrors the reference's io.drift.fmt package
(java/src/main/java/io/drift/fmt/): the same names, argument meanings and
errors. Every encode/decode/quantize runs on the GPU through the engine's C
ABI; this module only holds the format constants and the Rng state.
"""
from __future__ import annotations

import ctypes
from enum import IntEnum
from typing import Optional

import numpy as np

from . import _lib

_MASK64 = 0xFFFFFFFFFFFFFFFF


class Rounding(IntEnum):
    """java/src/main/java/io/drift/fmt/Rounding.java:14-20 (ordinals kept)."""

    NEAREST_EVEN = 0
    STOCHASTIC = 1
    TRUNCATE = 2


class Specials(IntEnum):
    """MiniFloat.Specials (MiniFloat.java:22-33)."""

    IEEE = 0
    FN = 1
    FINITE = 2


class Rng:
    """splitmix64 with a mutable 64-bit state (java/.../fmt/Rng.java:10-36).

    The engine consumes draws from the same stream: pass an Rng to a cast and
    its state afterwards is the state the Java Rng would hold.
    """

    __slots__ = ("_state",)

    def __init__(self, seed: int):
        self._state = seed & _MASK64

    def next_long(self) -> int:
        """Rng.nextLong (Rng.java:17-22), as an unsigned 64-bit int."""
        self._state = (self._state + 0x9E3779B97F4A7C15) & _MASK64
        z = self._state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK64
        return z ^ (z >> 31)

    def next_double(self) -> float:
        """Rng.nextDouble (Rng.java:25-27)."""
        return (self.next_long() >> 11) * 2.0 ** -53

    def state(self) -> int:
        return self._state

    def reseed(self, seed: int) -> None:
        self._state = seed & _MASK64


def _as_doubles(v) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(v, dtype=np.float64))


class MiniFloat:
    """One of the formats of Formats (java/.../fmt/Formats.java:20-45), with the
    derived constants of the MiniFloat constructor (MiniFloat.java:70-107)."""

    def __init__(self, name: str, fmt_id: int, exp_bits: int, mant_bits: int, bias: int,
                 specials: Specials):
        self.name = name
        self.id = fmt_id
        self.exp_bits = exp_bits
        self.mant_bits = mant_bits
        self.bias = bias
        self.specials = specials
        self.width = 1 + exp_bits + mant_bits
        self.min_normal_exp = 1 - bias
        self.min_normal = 2.0 ** self.min_normal_exp
        self.min_subnormal = 2.0 ** (self.min_normal_exp - mant_bits)
        if specials == Specials.IEEE:
            top_exp, top_mant = (1 << exp_bits) - 2, (1 << mant_bits) - 1
        elif specials == Specials.FN:
            top_exp, top_mant = (1 << exp_bits) - 1, (1 << mant_bits) - 2
        else:
            top_exp, top_mant = (1 << exp_bits) - 1, (1 << mant_bits) - 1
        self.max_finite = (1.0 + top_mant / (1 << mant_bits)) * 2.0 ** (top_exp - bias)

    def code_count(self) -> int:
        return 1 << self.width

    # -------------------------------------------------------------- codec
    def encode(self, v, rm: Rounding = Rounding.NEAREST_EVEN, rng: Optional[Rng] = None):
        """MiniFloat.encode (MiniFloat.java:156-211). A scalar gives an int, an
        array gives an int32 array. Raises DriftError(DRIFT_ENAN_FINITE) where
        Java throws ArithmeticException."""
        scalar = np.ndim(v) == 0
        x = _as_doubles(v).reshape(-1)
        codes = np.empty(x.size, dtype=np.int32)
        ctx = _lib.Context.current()
        st = ctypes.c_uint64(rng.state()) if rng is not None else None
        _lib.check(_lib.load().drift_encode(ctx.handle, self.id, int(rm), x.ctypes.data,
                                            codes.ctypes.data, x.size,
                                            ctypes.byref(st) if st is not None else None))
        if rng is not None:
            rng.reseed(st.value)
        return int(codes[0]) if scalar else codes.reshape(np.shape(v))

    def decode(self, bits):
        """MiniFloat.decode (MiniFloat.java:117-142)."""
        scalar = np.ndim(bits) == 0
        c = np.ascontiguousarray(np.asarray(bits, dtype=np.int32)).reshape(-1)
        out = np.empty(c.size, dtype=np.float64)
        ctx = _lib.Context.current()
        _lib.check(_lib.load().drift_decode(ctx.handle, self.id, c.ctypes.data, out.ctypes.data,
                                            c.size))
        return float(out[0]) if scalar else out.reshape(np.shape(bits))

    def quantize(self, v, rm: Rounding = Rounding.NEAREST_EVEN, rng: Optional[Rng] = None):
        """MiniFloat.quantize (MiniFloat.java:214-221): decode(encode(v))."""
        return self.decode(self.encode(v, rm, rng))

    def __repr__(self) -> str:
        return self.name

    __str__ = __repr__


class Formats:
    """java/src/main/java/io/drift/fmt/Formats.java:20-58."""

    E4M3 = MiniFloat("e4m3", 0, 4, 3, 7, Specials.FN)
    E5M2 = MiniFloat("e5m2", 1, 5, 2, 15, Specials.IEEE)
    E2M1 = MiniFloat("e2m1", 2, 2, 1, 1, Specials.FINITE)
    E3M2 = MiniFloat("e3m2", 3, 3, 2, 3, Specials.FINITE)
    E2M3 = MiniFloat("e2m3", 4, 2, 3, 1, Specials.FINITE)
    FP16 = MiniFloat("fp16", 5, 5, 10, 15, Specials.IEEE)
    BF16 = MiniFloat("bf16", 6, 8, 7, 127, Specials.IEEE)
    ALL = (E4M3, E5M2, E2M1, E3M2, E2M3, FP16, BF16)

    @staticmethod
    def by_name(name: str) -> MiniFloat:
        for f in Formats.ALL:
            if f.name.lower() == name.lower():
                return f
        raise ValueError(f"unknown format: {name}")
