"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run once, in a container that has the reference checked out (read-only):

    python tests/golden/make_golden.py --reference /path/to/drift

Two fixtures come out, both produced by the reference, not by this project:

formats.npz
    From the reference's exact-rational oracle (python/drift/minifloat.py,
    which its CI runs against the Java codec: python/verify_oracle.py:61-139).
    For each of the 7 formats: the value of every code; the code of the exact
    product and exact sum of every ordered pair of codes for formats of at
    most 8 bits, and of the first SAMPLED pairs of the DumpTables sample stream
    (java/src/main/java/io/drift/tools/DumpTables.java:106-120, Rng seed
    0x51ED1EA5) for fp16/bf16; and the nearest-even code of a set of random
    doubles spread over the format's range (Fraction(x) is exact).

dot_sweep.npz
    Rows of results/dot_sweep.csv (written by java/.../tools/DotSweep.java)
    whose inputs this host regenerates bit for bit. DotSweep.fill uses
    java.util.Random.nextGaussian (StrictMath.log) and Math.exp; host libm can
    differ from the JVM by an ulp, so a (n, seed) group is kept only when the
    FP64 sequential dot of the regenerated inputs equals the CSV's `exact`
    column exactly. For kept groups all 28 policy rows are stored.

The second step calls the CPU oracle only to regenerate the inputs and the
FP64 dot used as the filter; the stored expected values are the CSV's.
"""
from __future__ import annotations

import argparse
import csv
import math
import sys
import time
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import oracle as O  # noqa: E402

SAMPLED_PAIRS = 20_000          # first pairs of the DumpTables sample stream
RANDOM_VALUES = 4_000           # random doubles per format for encode checks
FORMAT_NAMES = ["e4m3", "e5m2", "e2m1", "e3m2", "e2m3", "fp16", "bf16"]


def splitmix_next_long(state: int):
    state = (state + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31), state


def to_double(mf, v) -> float:
    if v == mf.NAN:
        return math.nan
    if v == mf.POS_INF:
        return math.inf
    if v == mf.NEG_INF:
        return -math.inf
    if v == mf.NEG_ZERO:
        return -0.0
    return float(v)  # exact for every minifloat value


def make_formats(mf, out: Path) -> None:
    arrays = {}
    rs = np.random.default_rng(20251201)
    for fmt in mf.ALL:
        t0 = time.time()
        n = fmt.codes
        values = np.array([to_double(mf, fmt.decode(c)) for c in range(n)], dtype=np.float64)
        # Every minifloat value is exactly a float32, which halves the file.
        arrays[f"{fmt.name}_values"] = values.astype(np.float32)
        if fmt.width <= 8:
            a = np.repeat(np.arange(n, dtype=np.int32), n)
            b = np.tile(np.arange(n, dtype=np.int32), n)
        else:
            state = 0x51ED1EA5
            a_l, b_l = [], []
            for _ in range(SAMPLED_PAIRS):
                z, state = splitmix_next_long(state)
                a_l.append((z >> 1) % n)
                z, state = splitmix_next_long(state)
                b_l.append((z >> 1) % n)
            a = np.array(a_l, dtype=np.int32)
            b = np.array(b_l, dtype=np.int32)
        dec = [fmt.decode(c) for c in range(n)]
        prod = np.array([fmt.encode(mf.mul(fmt, dec[x], dec[y])) for x, y in zip(a, b)],
                        dtype=np.int32)
        summ = np.array([fmt.encode(mf.add(fmt, dec[x], dec[y])) for x, y in zip(a, b)],
                        dtype=np.int32)
        arrays[f"{fmt.name}_pair_a"] = a
        arrays[f"{fmt.name}_pair_b"] = b
        arrays[f"{fmt.name}_prod"] = prod
        arrays[f"{fmt.name}_sum"] = summ
        # Random doubles: signed, log-uniform from far below the smallest
        # subnormal to far above the maximum, plus exact ties.
        mx = float(fmt.max_finite)
        lo = math.log2(float(mf.pow2(fmt.min_normal_exp - fmt.mant_bits))) - 4
        hi = math.log2(mx) + 3
        x = np.exp2(rs.uniform(lo, hi, RANDOM_VALUES)) * rs.choice([-1.0, 1.0], RANDOM_VALUES)
        ties = values[np.isfinite(values)]
        ties = ties[: len(ties) - 1]
        mids = (ties[:-1] + ties[1:]) / 2  # midpoints of neighbouring codes
        mids = mids[np.isfinite(mids)]
        x[: min(len(mids), RANDOM_VALUES // 4)] = rs.permutation(mids)[: RANDOM_VALUES // 4]
        x = x.astype(np.float64)
        codes = np.array([fmt.encode(Fraction(float(v))) for v in x], dtype=np.int32)
        arrays[f"{fmt.name}_rand_x"] = x
        arrays[f"{fmt.name}_rand_code"] = codes
        print(f"{fmt.name}: {n} codes, {len(a)} pairs, {len(x)} randoms ({time.time() - t0:.1f}s)")
    np.savez_compressed(out, **arrays)


def dotsweep_cases():
    """The 28 cases of DotSweep.cases (java/.../tools/DotSweep.java:66-106)."""
    cs = []
    for acc in (O.ACC_FP32, O.ACC_FP16, O.ACC_BF16):
        for o in range(4):
            cs.append(O.policy(acc=acc, order=o, acc_block=32))
    for acc in (O.ACC_FP32, O.ACC_FP16, O.ACC_BF16):
        for o in (O.SEQUENTIAL, O.PAIRWISE):
            cs.append(O.policy(input_format=O.BF16, acc=acc, order=o))
    for f in (O.E4M3, O.E2M1):
        cs.append(O.policy(input_format=f, scaling=O.SCALE_NONE))
        cs.append(O.policy(input_format=f, scaling=O.PER_TENSOR))
        cs.append(O.policy(input_format=f, scaling=O.MX_BLOCK))
        cs.append(O.policy(input_format=f, scaling=O.MX_BLOCK, mx_headroom=1))
    cs.append(O.policy(input_format=O.E2M1, scaling=O.MX_BLOCK))
    cs.append(O.policy(input_format=O.E2M1, scaling=O.MX_BLOCK, input_rounding=O.STOCHASTIC))
    return cs


def make_dot_sweep(reference: Path, out: Path) -> None:
    rows = list(csv.DictReader(open(reference / "results" / "dot_sweep.csv")))
    groups = {}
    for r in rows:
        groups.setdefault((int(r["n"]), int(r["seed"])), []).append(r)
    labels = [r["label"] for r in groups[min(groups)]]
    assert len(labels) == 28
    kept_n, kept_seed, exact, result, clamped = [], [], [], [], []
    for (n, seed), rs in sorted(groups.items()):
        assert [r["label"] for r in rs] == labels
        a, b = O.dotsweep_fill(n, seed * 7919 + n)
        e, _ = O.dot(a, 0, 1, b, 0, 1, n, O.policy(acc=O.ACC_FP64))
        if e != float(rs[0]["exact"]):
            continue
        kept_n.append(n)
        kept_seed.append(seed)
        exact.append(e)
        result.append([float(r["result"]) for r in rs])
        clamped.append([int(r["clamped"]) for r in rs])
    np.savez_compressed(out, n=np.array(kept_n), seed=np.array(kept_seed),
                        exact=np.array(exact), result=np.array(result),
                        clamped=np.array(clamped), labels=np.array(labels))
    print(f"dot_sweep: kept {len(kept_n)} of {len(groups)} (n, seed) groups")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--only", choices=["formats", "dot_sweep"], default=None)
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference / "python"))
    from drift import minifloat as mf  # the reference's exact-rational oracle

    assert [f.name for f in mf.ALL] == FORMAT_NAMES
    if args.only in (None, "dot_sweep"):
        make_dot_sweep(args.reference, HERE / "dot_sweep.npz")
    if args.only in (None, "formats"):
        make_formats(mf, HERE / "formats.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
