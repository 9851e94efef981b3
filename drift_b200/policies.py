"""The named policy registry (java/src/main/java/io/drift/train/Policies.java).

Each policy differs from a named parent in one field (Policies.java:14-16).
"""
from __future__ import annotations

from typing import Dict

from .fmt import Formats, Rounding
from .kernel import Acc, NumericPolicy, Order, Scaling


def all_policies() -> Dict[str, NumericPolicy]:
    """Policies.all (Policies.java:23-92), in the same order."""
    m: Dict[str, NumericPolicy] = {}
    m["exact"] = NumericPolicy.exact()
    fp32 = NumericPolicy.builder("fp32").build()
    m["fp32"] = fp32
    m["bf16"] = NumericPolicy.builder("bf16").input(Formats.BF16).build()
    fp8 = (NumericPolicy.builder("fp8").input(Formats.E4M3).grad(Formats.E5M2)
           .scaling(Scaling.PER_TENSOR).build())
    m["fp8"] = fp8
    m["fp8-delayed"] = fp8.to_builder("fp8-delayed").amax_history(16).build()
    m["fp8-e4m3-grads"] = fp8.to_builder("fp8-e4m3-grads").grad(Formats.E4M3).build()
    m["fp8-mx"] = fp8.to_builder("fp8-mx").grad(Formats.E4M3).scaling(Scaling.MX_BLOCK).build()
    m["fp8-mx-headroom"] = (fp8.to_builder("fp8-mx-headroom").grad(Formats.E4M3)
                            .scaling(Scaling.MX_BLOCK).mx_headroom(1).build())
    m["fp8-reversed"] = fp8.to_builder("fp8-reversed").order(Order.REVERSED).build()
    m["fp8-acc-fp16"] = fp8.to_builder("fp8-acc-fp16").acc(Acc.FP16).build()
    m["fp8-acc-fp16-pairwise"] = (fp8.to_builder("fp8-acc-fp16-pairwise").acc(Acc.FP16)
                                  .order(Order.PAIRWISE).build())
    m["fp8-acc-bf16"] = fp8.to_builder("fp8-acc-bf16").acc(Acc.BF16).build()
    m["fp8-acc-bf16-pairwise"] = (fp8.to_builder("fp8-acc-bf16-pairwise").acc(Acc.BF16)
                                  .order(Order.PAIRWISE).build())
    m["fp8-acc-bf16-blocked"] = (fp8.to_builder("fp8-acc-bf16-blocked").acc(Acc.BF16)
                                 .order(Order.BLOCKED).acc_block(32).build())
    m["fp8-acc-bf16-sr"] = (fp8.to_builder("fp8-acc-bf16-sr").acc(Acc.BF16)
                            .acc_rounding(Rounding.STOCHASTIC).build())
    mxfp4 = NumericPolicy.builder("mxfp4").input(Formats.E2M1).scaling(Scaling.MX_BLOCK).build()
    m["mxfp4"] = mxfp4
    m["mxfp4-headroom"] = mxfp4.to_builder("mxfp4-headroom").mx_headroom(1).build()
    m["mxfp4-sr"] = mxfp4.to_builder("mxfp4-sr").input_rounding(Rounding.STOCHASTIC).build()
    m["mxfp4-sr-fwd"] = (mxfp4.to_builder("mxfp4-sr-fwd").input_rounding(Rounding.STOCHASTIC)
                         .grad_rounding(Rounding.NEAREST_EVEN).build())
    m["mxfp4-sr-bwd"] = (mxfp4.to_builder("mxfp4-sr-bwd").input_rounding(Rounding.NEAREST_EVEN)
                         .grad_rounding(Rounding.STOCHASTIC).build())
    fp8mx = m["fp8-mx"]
    m["fp8-mx-precise-probs"] = fp8mx.to_builder("fp8-mx-precise-probs").cast_probs(False).build()
    m["fp8-mx-precise-scores"] = fp8mx.to_builder("fp8-mx-precise-scores").cast_scores(False).build()
    m["mxfp4-precise-probs"] = mxfp4.to_builder("mxfp4-precise-probs").cast_probs(False).build()
    m["mxfp4-precise-scores"] = mxfp4.to_builder("mxfp4-precise-scores").cast_scores(False).build()
    m["mxfp4-precise-attn"] = (mxfp4.to_builder("mxfp4-precise-attn").cast_probs(False)
                               .cast_scores(False).build())
    m["acc-fp16"] = fp32.to_builder("acc-fp16").acc(Acc.FP16).build()
    m["acc-fp16-pairwise"] = fp32.to_builder("acc-fp16-pairwise").acc(Acc.FP16).order(Order.PAIRWISE).build()
    m["acc-bf16"] = fp32.to_builder("acc-bf16").acc(Acc.BF16).build()
    m["acc-bf16-pairwise"] = fp32.to_builder("acc-bf16-pairwise").acc(Acc.BF16).order(Order.PAIRWISE).build()
    m["acc-bf16-blocked"] = (fp32.to_builder("acc-bf16-blocked").acc(Acc.BF16)
                             .order(Order.BLOCKED).acc_block(32).build())
    return m


FOLLOW_UP = frozenset({  # Policies.java:95-99
    "mxfp4-sr-fwd", "mxfp4-sr-bwd", "fp8-mx-precise-probs", "fp8-mx-precise-scores",
    "mxfp4-precise-probs", "mxfp4-precise-scores", "mxfp4-precise-attn", "acc-fp16",
    "acc-fp16-pairwise", "acc-bf16", "acc-bf16-pairwise", "acc-bf16-blocked"})


def main_sweep() -> Dict[str, NumericPolicy]:
    """Policies.mainSweep (Policies.java:102-106): the 18 main-sweep policies."""
    return {k: v for k, v in all_policies().items() if k not in FOLLOW_UP}


def by_name(name: str) -> NumericPolicy:
    p = all_policies().get(name)
    if p is None:
        raise ValueError(f"unknown policy {name}; known: {list(all_policies())}")
    return p
