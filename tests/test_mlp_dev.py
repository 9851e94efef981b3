"""The device-resident MLP training step (drift_b200.mlp_dev): its kernels
against the host loops they replace, and whole training runs against the host
mirror (drift_b200.mlp, itself bit-exact against the oracle), bit for bit:
losses, measured cos/gain/rel, clamp rates, gradients, weights after Adam and
the Rng state."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    return torch


def _call(name, *args):
    from drift_b200 import _lib
    _lib.check(getattr(_lib.load(), name)(_lib.Context.current().handle, *args))


def _p(t):
    return t.data_ptr()


def test_embedding_lookup_and_ordered_gradient(torch):
    import drift_b200  # noqa: F401

    rs = np.random.default_rng(0)
    vocab, width, n = 37, 300, 1000          # width > one CTA's 256 columns
    table = rs.standard_normal(vocab * width)
    tok = rs.integers(0, vocab, n).astype(np.int32)
    tok[:50] = 3                              # many repeats of one row
    rows = rs.standard_normal(n * width) * np.exp(rs.standard_normal(n * width) * 4)
    g0 = rs.standard_normal(vocab * width)
    dt = torch.from_numpy(tok).cuda()
    out = torch.empty(n * width, dtype=torch.float64, device="cuda")
    _call("drift_embed_gather_dev", _p(dt), n, _p(torch.from_numpy(table).cuda()), vocab, width,
          _p(out), None)
    assert (out.cpu().numpy() == table.reshape(vocab, width)[tok].reshape(-1)).all()
    grad = torch.from_numpy(g0.copy()).cuda()
    _call("drift_embed_grad_dev", _p(dt), n, _p(torch.from_numpy(rows).cuda()), width, _p(grad),
          vocab, None)
    want = g0.copy().reshape(vocab, width)
    np.add.at(want, tok, rows.reshape(n, width))     # in index order, as Pass.java:168-179
    assert (grad.cpu().numpy().view(np.int64) == want.reshape(-1).view(np.int64)).all()


def test_bad_token_is_reported(torch):
    import drift_b200 as d

    tok = torch.tensor([0, 5, 9], dtype=torch.int32, device="cuda")
    out = torch.empty(6, dtype=torch.float64, device="cuda")
    _call("drift_embed_gather_dev", _p(tok), 3, _p(torch.zeros(12, dtype=torch.float64,
                                                                device="cuda")), 6, 2, _p(out), None)
    with pytest.raises(d.DriftError):
        d.check_dev()
    d.check_dev()   # the flag is cleared


def test_bias_grad_tanh_backward_and_adam(torch):
    import drift_b200  # noqa: F401
    from drift_b200 import mlp

    rs = np.random.default_rng(1)
    dy = rs.standard_normal(64 * 333) * np.exp(rs.standard_normal(64 * 333) * 3)
    db = torch.empty(333, dtype=torch.float64, device="cuda")
    _call("drift_bias_grad_dev", _p(torch.from_numpy(dy).cuda()), 64, 333, _p(db), None)
    want = np.cumsum(dy.reshape(64, 333), axis=0)[-1]
    assert (db.cpu().numpy().view(np.int64) == want.view(np.int64)).all()

    out = np.tanh(rs.standard_normal(5000))
    grad = rs.standard_normal(5000)
    dg = torch.from_numpy(grad.copy()).cuda()
    _call("drift_tanh_backward_dev", _p(torch.from_numpy(out).cuda()), _p(dg), 5000, None)
    grad *= 1.0 - out * out
    assert (dg.cpu().numpy().view(np.int64) == grad.view(np.int64)).all()

    for fp32 in (0, 1):
        p, g, m, v = (rs.standard_normal(4097) for _ in range(4))
        v = np.abs(v)
        dp, dg, dm, dv = (torch.from_numpy(x.copy()).cuda() for x in (p, g, m, v))
        hp, hm, hv = [p.copy()], [m.copy()], [v.copy()]
        for step in (1, 2, 7):
            _call("drift_adam_dev", _p(dp), _p(dg), _p(dm), _p(dv), 4097, step, 1e-3, fp32, None)
            mlp.adam(hp, [g], hm, hv, step, 1e-3, bool(fp32))
        for a, b in ((dp, hp[0]), (dm, hm[0]), (dv, hv[0])):
            assert (a.cpu().numpy().view(np.int64) == b.view(np.int64)).all()


def test_delayed_scale_history(torch):
    """Pass.scaleFor with amaxHistory 4 over 9 steps, against the host mirror."""
    import drift_b200 as d
    from drift_b200 import mlp

    p = d.policies.by_name("fp8-delayed")
    f = p.input_format
    net = mlp.Net(5, 2, 3, 4, 0)
    host = mlp.Pass(p.to_builder("h").amax_history(4).build(), net, 2, 1)
    hist = torch.zeros(4, dtype=torch.float64, device="cuda")
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    amax = torch.zeros(1, dtype=torch.float64, device="cuda")
    scale = torch.zeros(1, dtype=torch.float64, device="cuda")
    rs = np.random.default_rng(2)
    for step in range(9):
        x = rs.standard_normal(50) * (10.0 ** rs.integers(-3, 4))
        want = host._scale_for(0, 0, f, x)
        d.amax_dev(torch.from_numpy(x).cuda(), amax)
        _call("drift_scale_for_dev", f.id, _p(amax), _p(hist), 4, _p(count), _p(scale), None)
        assert float(scale.item()) == want, step


@pytest.mark.parametrize("policy", ["fp8-delayed-sr-grads", "mxfp4-sr", "fp8-acc-bf16-sr", "bf16",
                                    "fp8-mx", "exact-fp64-master"])
def test_training_run_matches_host_mirror(torch, policy):
    import drift_b200 as d
    from drift_b200 import mlp, mlp_dev

    if policy == "fp8-delayed-sr-grads":
        p = (d.policies.by_name("fp8-delayed").to_builder(policy)
             .grad_rounding(d.Rounding.STOCHASTIC).build())
    elif policy == "exact-fp64-master":
        p = d.policies.by_name("exact")     # no casts, FP64 masters
    else:
        p = d.policies.by_name(policy)
    kw = dict(vocab=23, ctx=5, emb=6, hidden=40, batch=12, steps=7, measure_every=3)
    got = mlp_dev.train(p, 3, **kw)
    want = mlp.train(p, 3, **kw)
    assert got["rng_state"] == want["rng_state"]
    for r1, r2 in zip(got["records"], want["records"]):
        assert (r1.loss, r1.loss_exact, r1.cos, r1.gain, r1.rel) == \
               (r2.loss, r2.loss_exact, r2.cos, r2.gain, r2.rel), r1.step
        assert (r1.clamp_x, r1.clamp_w, r1.clamp_g) == (r2.clamp_x, r2.clamp_w, r2.clamp_g)
    for a, b in zip(got["grads"], want["grads"]):
        assert (a.view(np.int64) == b.view(np.int64)).all()
    for a, b in zip(got["params"], want["net"].tensors()):
        assert (a.view(np.int64) == b.view(np.int64)).all()


def test_full_size_25_steps_with_exact_recompute_matches_oracle(torch):
    """The training-step configuration as the reference runs it: vocab 96,
    ctx 32, emb 64, hidden 2048, batch 64, fp8 delayed scaling (history 16)
    with stochastic gradient rounding, 25 steps, the exact FP64 recompute at
    steps 1 and 25 (Trainer.java:140, compare at :272-288). The timed
    device-resident step against the same run with every cast and contraction
    on the oracle: losses, cos/gain/rel at both measurement steps, clamp
    rates, the last step's gradients, the weights after 25 Adam updates and
    the Rng state, bit for bit."""
    import drift_b200 as d
    from drift_b200 import mlp, mlp_dev
    from helpers import OracleBackend

    p = (d.policies.by_name("fp8-delayed").to_builder("fp8-delayed-sr-grads")
         .grad_rounding(d.Rounding.STOCHASTIC).build())
    got = mlp_dev.train(p, 0, steps=25)
    want = mlp.train(p, 0, steps=25, backend=OracleBackend())
    assert got["rng_state"] == want["rng_state"]
    measured = [r.step for r in want["records"] if r.cos is not None]
    assert measured == [1, 25]
    for r1, r2 in zip(got["records"], want["records"]):
        assert (r1.loss, r1.loss_exact, r1.cos, r1.gain, r1.rel) == \
               (r2.loss, r2.loss_exact, r2.cos, r2.gain, r2.rel), r1.step
        assert (r1.clamp_x, r1.clamp_w, r1.clamp_g) == (r2.clamp_x, r2.clamp_w, r2.clamp_g)
    for a, b in zip(got["grads"], want["grads"]):
        assert (a.view(np.int64) == b.view(np.int64)).all()
    for a, b in zip(got["params"], want["net"].tensors()):
        assert (a.view(np.int64) == b.view(np.int64)).all()
