"""DumpTables on the device: the format tables an exact-rational verification reads.

Mirrors io.drift.tools.DumpTables (java/src/main/java/io/drift/tools/DumpTables.java)
file for file: for every format of Formats.ALL a ``values_<name>.csv`` with the
raw double bits of every code, and a ``pairs_<name>.csv`` with the nearest-even
code of the exact product and sum of every ordered code pair (formats of up to
8 bits) or of 200,000 pairs drawn from ``Rng(0x51ED1EA5)`` (fp16, bf16). The
codes come from the engine's device codec (``drift_value_table`` /
``drift_pair_table``), so the reference's ``python/verify_oracle.py`` run on
this directory checks the B200 encoder and decoder exhaustively.

    python -m drift_b200.dump_tables [out_dir]
"""
from __future__ import annotations

import ctypes
import math
import sys
from decimal import Decimal
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import Context, check
from .fmt import Formats, MiniFloat, Specials

EXHAUSTIVE_PAIR_WIDTH = 8        # DumpTables.java:31
SAMPLED_PAIRS = 200_000          # :41
SAMPLE_SEED = 0x51ED1EA5         # :108
PAIRS_EXHAUSTIVE, PAIRS_SAMPLED = 0, 1


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def value_bits(f: MiniFloat, ctx: Context | None = None) -> np.ndarray:
    """uint64 raw bits of decode(c) for every code c (DumpTables.java:61-79)."""
    ctx = ctx or Context.current()
    out = np.empty(f.code_count(), dtype=np.uint64)
    check(_lib.load().drift_value_table(ctx.handle, f.id, _ptr(out)))
    return out


def pair_codes(f: MiniFloat, mode: int, n: int, first: int = 0, seed: int = SAMPLE_SEED,
               ctx: Context | None = None):
    """(a, b, prod_code, sum_code) int32 arrays for rows first..first+n-1 of
    the pair table (DumpTables.java:87-124)."""
    ctx = ctx or Context.current()
    a, b, prod, s = (np.empty(n, dtype=np.int32) for _ in range(4))
    check(_lib.load().drift_pair_table(ctx.handle, f.id, mode, ctypes.c_uint64(seed), first, n,
                                       _ptr(a), _ptr(b), _ptr(prod), _ptr(s)))
    return a, b, prod, s


def java_g17(v: float) -> str:
    """String.format(Locale.ROOT, "%.17g", v) for a finite double.

    java.util.Formatter takes the double's shortest round-trip decimal digits
    and pads them with zeros to 17 significant digits; it writes plain
    decimals for 1e-4 <= |v| < 1e17 and otherwise d.ddd…e±XX with at least two
    exponent digits. A zero keeps its sign."""
    neg = math.copysign(1.0, v) < 0
    a = abs(v)
    if a == 0.0:
        body = "0." + "0" * 16
    else:
        t = Decimal(repr(a)).normalize().as_tuple()
        digits = "".join(map(str, t.digits))
        e10 = len(digits) - 1 + t.exponent
        digits = (digits + "0" * 17)[:17]
        if -4 <= e10 < 17:
            if e10 >= 0:
                body = digits[:e10 + 1] + "." + digits[e10 + 1:]
            else:
                body = "0." + "0" * (-e10 - 1) + digits
        else:
            body = f"{digits[0]}.{digits[1:]}e{'-' if e10 < 0 else '+'}{abs(e10):02d}"
    return ("-" if neg else "") + body


def describe(bits: int) -> str:
    """DumpTables.describe (:126-134) of the double with these raw bits."""
    v = float(np.uint64(bits).view(np.float64))
    if math.isnan(v):
        return "nan"
    if math.isinf(v):
        return "inf" if v > 0 else "-inf"
    return java_g17(v)


def write_values(f: MiniFloat, path: Path, ctx: Context | None = None) -> None:
    bits = value_bits(f, ctx)
    lines = [f"# format={f.name} expBits={f.exp_bits} mantBits={f.mant_bits} bias={f.bias}"
             f" specials={Specials(f.specials).name} overflow=SATURATE codes={f.code_count()}\n",
             "code,double_bits_hex,value\n"]
    # Every format of Formats.ALL saturates on overflow (Formats.java:20-45).
    lines += [f"{c},{int(b):x},{describe(int(b))}\n" for c, b in enumerate(bits)]
    path.write_text("".join(lines))


def write_pairs(f: MiniFloat, path: Path, ctx: Context | None = None) -> None:
    n = f.code_count()
    if f.width <= EXHAUSTIVE_PAIR_WIDTH:
        header = f"# format={f.name} mode=exhaustive pairs={n * n}\n"
        a, b, prod, s = pair_codes(f, PAIRS_EXHAUSTIVE, n * n, ctx=ctx)
    else:
        header = f"# format={f.name} mode=sampled seed=0x{SAMPLE_SEED:X} pairs={SAMPLED_PAIRS}\n"
        a, b, prod, s = pair_codes(f, PAIRS_SAMPLED, SAMPLED_PAIRS, ctx=ctx)
    rows = np.stack([a, b, prod, s], axis=1)
    body = "\n".join(",".join(map(str, r)) for r in rows.tolist())
    path.write_text(header + "a,b,prod_code,sum_code\n" + body + "\n")


def main(argv: list[str] | None = None) -> int:
    """DumpTables.main (:43-55)."""
    argv = sys.argv[1:] if argv is None else argv
    out = Path(argv[0] if argv else "../results/oracle")
    out.mkdir(parents=True, exist_ok=True)
    for f in Formats.ALL:
        write_values(f, out / f"values_{f.name}.csv")
        write_pairs(f, out / f"pairs_{f.name}.csv")
    print(f"wrote oracle tables to {out.resolve()}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
