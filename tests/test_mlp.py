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


# PassTest (java/src/test/java/io/drift/net/PassTest.java:17-24)
P_VOCAB, P_CTX, P_EMB, P_HIDDEN, P_BATCH = 7, 3, 4, 5, 4
P_CONTEXTS = np.array([0, 1, 2, 3, 4, 5, 6, 0, 1, 2, 2, 2])
P_TARGETS = np.array([3, 6, 1, 0])


@pytest.mark.gpu
def test_exact_gradients_match_finite_differences():
    """PassTest.exactGradientsMatchFiniteDifferences (:26-51): central
    differences, step 1e-6, worst relative error below 1e-5, the exact
    policy on the engine. (Weights come from numpy, not java.util.Random.)"""
    import drift_b200 as d
    from drift_b200 import mlp

    net = mlp.Net(P_VOCAB, P_CTX, P_EMB, P_HIDDEN, 17)
    pas = mlp.Pass(d.NumericPolicy.exact(), net, P_BATCH, 1)
    _, grads = pas.loss_and_grads(P_CONTEXTS, P_TARGETS)
    h, worst = 1e-6, 0.0
    for t, params in enumerate(net.tensors()):
        for i in range(params.size):
            keep = params[i]
            params[i] = keep + h
            up = pas.forward(P_CONTEXTS, P_TARGETS)
            params[i] = keep - h
            down = pas.forward(P_CONTEXTS, P_TARGETS)
            params[i] = keep
            numeric = (up - down) / (2 * h)
            err = abs(numeric - grads[t][i]) / max(1e-6, abs(numeric) + abs(grads[t][i]))
            worst = max(worst, err)
    assert worst < 1e-5, worst


@pytest.mark.gpu
def test_uncast_fp32_pass_stays_close_to_exact():
    """PassTest.uncastFp32PassStaysCloseToExact (:69-90): the builder's
    default policy (FP32 accumulator, no casts) against the exact pass,
    gradient cosine above 1 - 1e-9."""
    import drift_b200 as d
    from drift_b200 import mlp

    net = mlp.Net(P_VOCAB, P_CTX, P_EMB, P_HIDDEN, 17)
    _, ge = mlp.Pass(d.NumericPolicy.exact(), net, P_BATCH, 1).loss_and_grads(P_CONTEXTS, P_TARGETS)
    _, gf = mlp.Pass(d.NumericPolicy.builder("fp32").build(), net, P_BATCH, 1).loss_and_grads(
        P_CONTEXTS, P_TARGETS)
    a, b = np.concatenate(gf), np.concatenate(ge)
    assert np.dot(a, b) / np.sqrt(np.dot(b, b) * np.dot(a, a)) > 1 - 1e-9
