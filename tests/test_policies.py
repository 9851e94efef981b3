"""The named-policy registry, as the reference's PoliciesTest checks it
(java/src/test/java/io/drift/net/PoliciesTest.java)."""


def test_main_sweep_is_the_eighteen_in_the_readme():
    """PoliciesTest.mainSweepIsTheEighteenInTheReadme (:15-20)."""
    from drift_b200 import policies

    assert len(policies.main_sweep()) == 18
    assert "acc-bf16" not in policies.main_sweep()
    assert "acc-bf16" in policies.all_policies()


def test_stochastic_rounding_split_changes_only_one_half():
    """PoliciesTest.stochasticRoundingSplitChangesOnlyOneHalf (:22-30)."""
    from drift_b200 import Rounding, policies

    fwd, bwd = policies.by_name("mxfp4-sr-fwd"), policies.by_name("mxfp4-sr-bwd")
    assert fwd.input_rounding == Rounding.STOCHASTIC
    assert fwd.grad_cast_rounding() == Rounding.NEAREST_EVEN
    assert bwd.input_rounding == Rounding.NEAREST_EVEN
    assert bwd.grad_cast_rounding() == Rounding.STOCHASTIC


def test_uncast_accumulator_policies_only_change_the_accumulator():
    """PoliciesTest.uncastAccumulatorPoliciesOnlyChangeTheAccumulator (:32-44)."""
    from drift_b200 import policies

    base = policies.by_name("fp32")
    for name in ("acc-fp16", "acc-fp16-pairwise", "acc-bf16", "acc-bf16-pairwise",
                 "acc-bf16-blocked"):
        p = policies.by_name(name)
        assert p.input_format is None, name
        assert p.scaling == base.scaling and p.master_fp32 == base.master_fp32, name
        assert p.acc != base.acc, name
