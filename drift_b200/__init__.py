"""drift_b200 — a B200-native engine for drift's policy-parameterised emulated matmul.

The Python surface mirrors the reference's Java API (io.drift.fmt and
io.drift.kernel): Formats / MiniFloat / Rounding / Rng, NumericPolicy, Quant,
Dot, and the named Policies. Every cast and every contraction runs in the
CUDA engine (libdrift_b200.so, sm_100a) through its C ABI
(include/drift_b200.h); importing the package loads it and fails if it cannot.
"""
from . import _lib
from ._lib import Context, DriftError
from .fmt import Formats, MiniFloat, Rng, Rounding, Specials
from .kernel import (Acc, Dot, NumericPolicy, Order, Quant, Scaling, Window, amax_dev,
                     check_dev, contract, contract_dev, contraction, error_sums_dev, gemm,
                     per_tensor_scale_dev, probe_fp32, probe_fp64, gemm_dev, gemm_launches,
                     gemm_route, quantize_dev, set_thin_tiles, ROUTE_DOUBLE, ROUTE_FP32,
                     ROUTE_SCANNED, ROUTE_STAGED, ROUTE_PROVEN)
from . import policies

_lib.load()

__all__ = ["Context", "DriftError", "Formats", "MiniFloat", "Rng", "Rounding", "Specials", "Acc",
           "Dot", "NumericPolicy", "Order", "Quant", "Scaling", "Window", "contraction", "contract",
           "contract_dev", "gemm", "gemm_dev", "gemm_launches", "gemm_route", "quantize_dev",
           "ROUTE_DOUBLE", "ROUTE_FP32", "ROUTE_SCANNED", "ROUTE_STAGED", "ROUTE_PROVEN", "set_thin_tiles",
           "amax_dev", "check_dev", "policies"]
