"""The reference's own golden rows (results/dot_sweep.csv, kept where the
inputs regenerate exactly) reproduced by the engine: DotSweep.run
(java/src/main/java/io/drift/tools/DotSweep.java:112-122) with every cast and
dot on the GPU, stochastic-rounding rows included."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dotsweep_cases(d):
    """DotSweep.cases (DotSweep.java:66-106)."""
    F, A, Ord, S = d.Formats, d.Acc, d.Order, d.Scaling
    b = d.NumericPolicy.builder
    cs = []
    for acc in (A.FP32, A.FP16, A.BF16):
        for o in Ord:
            cs.append(b("a").acc(acc).order(o).acc_block(32).build())
    for acc in (A.FP32, A.FP16, A.BF16):
        for o in (Ord.SEQUENTIAL, Ord.PAIRWISE):
            cs.append(b("c").input(F.BF16).acc(acc).order(o).build())
    for f in (F.E4M3, F.E2M1):
        cs.append(b("n").input(f).scaling(S.NONE).build())
        cs.append(b("p").input(f).scaling(S.PER_TENSOR).build())
        cs.append(b("m").input(f).scaling(S.MX_BLOCK).build())
        cs.append(b("h").input(f).scaling(S.MX_BLOCK).mx_headroom(1).build())
    cs.append(b("n").input(F.E2M1).scaling(S.MX_BLOCK).build())
    cs.append(b("s").input(F.E2M1).scaling(S.MX_BLOCK).input_rounding(d.Rounding.STOCHASTIC).build())
    return cs


def test_dot_sweep_golden_rows_on_the_engine(golden_dir):
    import drift_b200 as d

    g = np.load(golden_dir / "dot_sweep.npz")
    cases = dotsweep_cases(d)
    exact_p = d.NumericPolicy.exact()
    for k in range(len(g["n"])):
        n, seed = int(g["n"][k]), int(g["seed"][k])
        a, b = O.dotsweep_fill(n, seed * 7919 + n)
        assert d.Dot.dot(a, 0, 1, b, 0, 1, n, exact_p) == g["exact"][k]
        for c, p in enumerate(cases):
            rng = d.Rng(0xD1F7 + seed)
            f = p.input_format
            sa = 1.0 if f is None else d.Quant.per_tensor_scale(f, d.Quant.amax(a))
            sb = 1.0 if f is None else d.Quant.per_tensor_scale(f, d.Quant.amax(b))
            qa, qb = np.empty(n), np.empty(n)
            clamped = d.Quant.quantize(a, 0, qa, 0, n, f, p, sa, rng)
            clamped += d.Quant.quantize(b, 0, qb, 0, n, f, p, sb, rng)
            v = d.Dot.dot(qa, 0, 1, qb, 0, 1, n, p, rng)
            assert v == g["result"][k, c], (n, seed, str(g["labels"][c]))
            assert clamped == g["clamped"][k, c]
