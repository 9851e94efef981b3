"""The emulated MLP training step (Pass / Trainer mirror): every cast and
every forward, dgrad and wgrad contraction on the engine, checked bit for bit
against the same pass run on the oracle, gradients and Rng state included."""
import numpy as np
import pytest

from helpers import OracleBackend
from oracle import oracle as O


def test_host_pieces_without_gpu():
    """Net shapes, delayed-scaling history and the Adam update need no GPU."""
    from drift_b200 import mlp
    net = mlp.Net(11, 3, 4, 7, 5)
    assert [t.size for t in net.tensors()] == [44, 84, 7, 49, 7, 77, 11]
    p = [np.ones(3)]
    g = [np.full(3, 0.5)]
    m, v = [np.zeros(3)], [np.zeros(3)]
    mlp.adam(p, g, m, v, 1, 0.1, True)
    assert np.allclose(p[0], 0.9, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("policy", ["fp8-delayed-sr-grads", "fp8", "mxfp4-sr", "fp8-acc-bf16-pairwise",
                                    "acc-fp16", "bf16", "fp8-acc-bf16-sr"])
def test_training_step_matches_oracle(policy):
    import drift_b200 as d
    from drift_b200 import mlp

    if policy == "fp8-delayed-sr-grads":
        p = (d.policies.by_name("fp8-delayed").to_builder(policy)
             .grad_rounding(d.Rounding.STOCHASTIC).build())
    else:
        p = d.policies.by_name(policy)
    kw = dict(vocab=23, ctx=5, emb=6, hidden=40, batch=12, steps=6, measure_every=3)
    got = mlp.train(p, 3, **kw)
    want = mlp.train(p, 3, backend=OracleBackend(), **kw)
    assert got["rng_state"] == want["rng_state"]
    for a, b in zip(got["grads"], want["grads"]):
        assert (a.view(np.int64) == b.view(np.int64)).all()
    for r1, r2 in zip(got["records"], want["records"]):
        assert r1.loss == r2.loss and r1.cos == r2.cos and r1.clamp_g == r2.clamp_g


@pytest.mark.gpu
def test_training_step_full_size_first_steps():
    """The training-step configuration at full size (vocab 96, ctx 32, emb 64,
    hidden 2048, batch 64) under fp8 delayed scaling with stochastic gradient
    rounding: two steps, every gradient bit-equal to the oracle's."""
    import drift_b200 as d
    from drift_b200 import mlp

    p = (d.policies.by_name("fp8-delayed").to_builder("c4")
         .grad_rounding(d.Rounding.STOCHASTIC).build())
    got = mlp.train(p, 0, steps=2, measure_every=25)
    want = mlp.train(p, 0, steps=2, measure_every=25, backend=OracleBackend())
    assert got["rng_state"] == want["rng_state"]
    for a, b in zip(got["grads"], want["grads"]):
        assert (a.view(np.int64) == b.view(np.int64)).all()
    r = got["records"][0]
    assert 0.5 < r.cos <= 1.0 and r.clamp_x >= 0.0
