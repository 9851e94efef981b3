"""The study drivers on the engine against the oracle, at the configurations'
own shapes: the dot sweep (lengths 16..4096), the real-shape batch
(4096 x 64 x 2048, every output) and the block-scaled GEMM (4096^3, sampled
outputs)."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _op(p):
    c = p.to_c()
    return O.OraclePolicy(*[getattr(c, f) for f, _ in c._fields_])


def _oracle_dot_run(p, a, b, seed):
    rng = 0xD1F7 + seed
    f = p.input_format
    fid = f.id if f is not None else -1
    sa = 1.0 if f is None else O.per_tensor_scale(fid, O.amax(a))
    sb = 1.0 if f is None else O.per_tensor_scale(fid, O.amax(b))
    op = _op(p)
    qa, ca, rng = O.quantize(op, fid, int(p.input_rounding), a, sa, rng)
    qb, cb, rng = O.quantize(op, fid, int(p.input_rounding), b, sb, rng)
    v, _ = O.dot(qa, 0, 1, qb, 0, 1, a.size, op, rng)
    return v, ca + cb


def test_dot_sweep_baseline_shapes():
    from drift_b200 import sweeps

    out = sweeps.dot_sweep(seeds=12)
    seen = 0
    pols = {p.name: p for p in sweeps.dot_sweep_policies()}
    for name, n, seed, value, exact, clamped in out["rows"]:
        rs = np.random.default_rng(seed * 7919 + n)
        a, b = sweeps.heavy_tailed(rs, n), sweeps.heavy_tailed(rs, n)
        v, c = _oracle_dot_run(pols[name], a, b, seed)
        assert v == value and c == clamped, (name, n, seed)
        seen += 1
    assert seen == 9 * 12 * 10
    t = out["table"]
    assert set(t["fp32 sequential"]) == {16, 32, 64, 128, 256, 512, 1024, 2048, 4096}


def test_real_shape_batch_every_output():
    from drift_b200 import sweeps

    X, W = sweeps.real_dot_inputs()
    M, K = X.shape
    N = W.shape[0]
    clamps = {}
    for p in sweeps.real_dot_policies():
        got, clamped = sweeps.policy_outputs(p, X, W)
        f = p.input_format
        fid = f.id if f is not None else -1
        qx, qw, c1, c2 = X, W, 0, 0
        rng = 7
        if f is not None:
            op = _op(p)
            qx, c1, rng = O.quantize(op, fid, 0, X.reshape(-1), O.per_tensor_scale(fid, O.amax(X)), rng)
            qw, c2, rng = O.quantize(op, fid, 0, W.reshape(-1), O.per_tensor_scale(fid, O.amax(W)), rng)
        want, _ = O.gemm(_op(p), M, N, K, qx, 0, K, 1, qw, 0, K, 1, threads=16)
        assert (got.view(np.int64) == want.view(np.int64)).all(), p.name
        assert clamped == c1 + c2
        clamps[p.name] = (c1, c2)
    stats = sweeps.real_dot_batch(X, W)
    assert stats["fp32 sequential"]["median_rel_error"] < stats["bf16 sequential"]["median_rel_error"]
    # The device-resident driver: the same true medians bit for bit (order
    # statistics of the same bit-exact outputs), RMS ratios to rounding.
    dev = sweeps.real_dot_batch_dev(X, W)
    assert dev.keys() == stats.keys()
    for name in stats:
        assert dev[name]["median_rel_error"] == stats[name]["median_rel_error"], name
        assert dev[name]["rms_error_ratio"] == pytest.approx(stats[name]["rms_error_ratio"],
                                                             rel=1e-12), name
    # The whole loop in one host-buffer call: the same statistics, and the
    # clamp counts of each operand's cast.
    one = sweeps.real_dot_sweep(X, W)
    assert one.keys() == stats.keys()
    for name in stats:
        assert one[name]["median_rel_error"] == stats[name]["median_rel_error"], name
        assert one[name]["rms_error_ratio"] == pytest.approx(stats[name]["rms_error_ratio"],
                                                             rel=1e-12), name
        assert (one[name]["clamped_x"], one[name]["clamped_w"]) == clamps[name], name


def _oracle_real_dot_stats(p, X, W, seed):
    """RealDotSweep's per-policy flow (:235-257) on the oracle: Rng(seed), the
    per-tensor casts of X then W, the contraction on the same Rng, the true
    median and the RMS ratio against the FP64 outputs."""
    from drift_b200.kernel import NumericPolicy

    M, K = X.shape
    N = W.shape[0]
    op = _op(p)
    f = p.input_format
    rng, qx, qw, c1, c2 = seed, X.reshape(-1), W.reshape(-1), 0, 0
    if f is not None:
        rm = int(p.input_rounding)
        qx, c1, rng = O.quantize(op, f.id, rm, qx, O.per_tensor_scale(f.id, O.amax(X)), rng)
        qw, c2, rng = O.quantize(op, f.id, rm, qw, O.per_tensor_scale(f.id, O.amax(W)), rng)
    got, _ = O.gemm(op, M, N, K, qx, 0, K, 1, qw, 0, K, 1, rng_state=rng, threads=8)
    ex, _ = O.gemm(_op(NumericPolicy.exact()), M, N, K, X, 0, K, 1, W, 0, K, 1, threads=8)
    err = (got - ex).reshape(-1)
    rel = np.sort(np.abs(err) / np.abs(ex.reshape(-1)))
    n = rel.size
    return (0.5 * (rel[n // 2 - 1] + rel[n // 2]),
            np.sqrt(np.sum(err * err) / np.sum(ex * ex)), c1, c2)


def test_real_dot_sweep_stochastic_policies_against_oracle():
    """The one-call loop on policies the real-shape batch does not hold:
    stochastic casts, stochastic accumulation (the contraction kernels'
    Rng path), blocked order, a format that clamps, a seed other than 7."""
    from drift_b200 import sweeps
    from drift_b200.fmt import Formats, Rounding
    from drift_b200.kernel import Acc, NumericPolicy, Order, Scaling

    b = NumericPolicy.builder
    pols = [b("e4m3 sr cast").input(Formats.E4M3).input_rounding(Rounding.STOCHASTIC)
            .scaling(Scaling.PER_TENSOR).build(),
            b("bf16 sr acc").acc(Acc.BF16).acc_rounding(Rounding.STOCHASTIC).build(),
            b("fp16 sr acc blocked").acc(Acc.FP16).order(Order.BLOCKED)
            .acc_rounding(Rounding.STOCHASTIC).build(),
            b("e2m1 truncated").input(Formats.E2M1).input_rounding(Rounding.TRUNCATE).build(),
            b("fp32 reversed").order(Order.REVERSED).build()]
    rs = np.random.default_rng(5)
    X = rs.standard_normal((96, 320)) * np.exp(rs.standard_normal((96, 320)))
    W = rs.standard_normal((40, 320))
    one = sweeps.real_dot_sweep(X, W, pols, rng_seed=1234)
    for p in pols:
        med, rms, c1, c2 = _oracle_real_dot_stats(p, X, W, 1234)
        got = one[p.name]
        assert got["median_rel_error"] == med, p.name
        assert got["rms_error_ratio"] == pytest.approx(rms, rel=1e-12), p.name
        assert (got["clamped_x"], got["clamped_w"]) == (c1, c2), p.name


def test_mx_gemm_sampled_outputs():
    import torch

    import drift_b200 as d
    from drift_b200 import sweeps

    S = 4096
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    A = (torch.randn(S, S, device=dev, generator=g) *
         torch.exp(torch.randn(S, S, device=dev, generator=g))).double()
    W = (torch.randn(S, S, device=dev, generator=g) *
         torch.exp(torch.randn(S, S, device=dev, generator=g))).double()
    rs = np.random.default_rng(0)
    rows = np.sort(rs.choice(S, 8, replace=False))
    cols = np.sort(rs.choice(S, 64, replace=False))
    for p in sweeps.mx_policies():
        f = p.input_format
        qa, qw, C = torch.empty_like(A), torch.empty_like(W), torch.empty_like(A)
        scal = torch.zeros(4, dtype=torch.float64, device=dev)
        scales = [1.0, 1.0]
        for k, (src, dst) in enumerate(((A, qa), (W, qw))):
            if p.scaling == d.Scaling.PER_TENSOR:
                d.amax_dev(src, scal[k:k + 1])
                d.per_tensor_scale_dev(f, scal[k:k + 1], scal[2 + k:3 + k])
                d.quantize_dev(p, f, d.Rounding.NEAREST_EVEN, src, dst, d_scale=scal[2 + k:3 + k])
            else:
                d.quantize_dev(p, f, d.Rounding.NEAREST_EVEN, src, dst)
        d.gemm_dev(p, qa, qw, C)
        d.check_dev()
        scales = [float(x) for x in scal[2:4].cpu()]
        a_rows = A[rows].cpu().numpy().reshape(-1)
        w_rows = W[cols].cpu().numpy().reshape(-1)
        op = _op(p)
        oqa, _, _ = O.quantize(op, f.id, 0, a_rows, scales[0])
        oqw, _, _ = O.quantize(op, f.id, 0, w_rows, scales[1])
        assert (qa[rows].cpu().numpy().reshape(-1).view(np.int64) == oqa.view(np.int64)).all()
        want, _ = O.gemm(op, len(rows), len(cols), S, oqa, 0, S, 1, oqw, 0, S, 1, threads=16)
        got = C[rows][:, cols].cpu().numpy()
        assert (got.view(np.int64) == want.view(np.int64)).all(), p.name
    res = sweeps.mx_gemm(1024, policies=sweeps.mx_policies()[:2])
    assert res["e4m3 mx32 spec"]["clamped_per_pair"] > 0.0


def test_device_dot_sweep_equals_host_sweep():
    """dot_sweep_dev (one batched contraction per policy and length) gives
    the same rows as dot_sweep (one host call per dot): values, exact values,
    clamp counts and the summary table."""
    from drift_b200 import sweeps

    host = sweeps.dot_sweep(lengths=(16, 100, 1024), seeds=7)
    dev = sweeps.dot_sweep_dev(lengths=(16, 100, 1024), seeds=7, host_inputs=True)
    key = lambda r: (r[0], r[1], r[2])
    h, g = sorted(host["rows"], key=key), sorted(dev["rows"], key=key)
    assert len(h) == len(g)
    for a, b in zip(h, g):
        assert a[:3] == b[:3] and a[5] == b[5]
        assert np.float64(a[3]).view(np.int64) == np.float64(b[3]).view(np.int64), a[:3]
        assert np.float64(a[4]).view(np.int64) == np.float64(b[4]).view(np.int64), a[:3]
    assert host["table"] == dev["table"]


def test_device_dot_sweep_full_shape_against_oracle():
    """The dot sweep at its configuration (200 seeds x lengths 16..4096, 10
    policies) with inputs generated on the device: every dot and clamp count
    against the oracle on the same vectors (read back for the check), and the
    device medians against the upper median of the rows."""
    from drift_b200 import sweeps

    lengths = tuple(2 ** k for k in range(4, 13))
    out = sweeps.dot_sweep_dev(lengths=lengths, seeds=200, keep_inputs=True)
    pols = {p.name: p for p in sweeps.dot_sweep_policies()}
    errs = {}
    for name, n, seed, value, exact, clamped in out["rows"]:
        a, b = out["inputs"][n][0][seed], out["inputs"][n][1][seed]
        v, c = _oracle_dot_run(pols[name], a, b, seed)
        assert np.float64(v).view(np.int64) == np.float64(value).view(np.int64), (name, n, seed)
        assert c == clamped, (name, n, seed)
        ex, _ = O.dot(a, 0, 1, b, 0, 1, n, _op(sweeps.NumericPolicy.exact()))
        assert ex == exact
        errs.setdefault((name, n), []).append(abs(value - exact) / abs(exact))
    for (name, n), e in errs.items():
        assert out["table"][name][n]["median_rel_error"] == sorted(e)[len(e) // 2], (name, n)
