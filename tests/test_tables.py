"""DumpTables on the device (java/src/main/java/io/drift/tools/DumpTables.java):
the value of every code and the nearest-even codes of exact products and sums,
against the golden tables restated from the reference's exact-rational codec,
and the files laid out as DumpTables writes them."""
import numpy as np
import pytest

from pathlib import Path

GOLDEN = Path(__file__).parent / "golden"


def test_java_general_format_known_answers():
    """Formatter %.17g: shortest digits padded to 17 significant digits."""
    from drift_b200.dump_tables import java_g17

    assert java_g17(1.0) == "1.0000000000000000"
    assert java_g17(-0.0) == "-0.0000000000000000"
    assert java_g17(0.0) == "0.0000000000000000"
    assert java_g17(448.0) == "448.00000000000000"
    assert java_g17(0.1) == "0.10000000000000000"
    assert java_g17(0.001953125) == "0.0019531250000000000"
    assert java_g17(2.0 ** -24) == "5.9604644775390630e-08"
    assert java_g17(-57344.0) == "-57344.000000000000"
    assert java_g17(1e17) == "1.0000000000000000e+17"
    assert java_g17(1e-4) == "0.00010000000000000000"
    assert java_g17(3.3895313892515355e38) == "3.3895313892515355e+38"


def test_describe_specials():
    from drift_b200.dump_tables import describe

    assert describe(0x7FF8000000000000) == "nan"
    assert describe(0x7FF0000000000000) == "inf"
    assert describe(0xFFF0000000000000) == "-inf"
    assert describe(0x3FF8000000000000) == "1.5000000000000000"


@pytest.mark.gpu
def test_value_tables_match_golden():
    from drift_b200 import Formats
    from drift_b200.dump_tables import value_bits

    z = np.load(GOLDEN / "formats.npz")
    for f in Formats.ALL:
        got = value_bits(f).view(np.float64)
        want = z[f"{f.name}_values"].astype(np.float64)
        nan = np.isnan(want)
        assert (np.isnan(got) == nan).all(), f.name
        assert (got[~nan].view(np.int64) == want[~nan].view(np.int64)).all(), f.name


@pytest.mark.gpu
def test_pair_tables_match_golden():
    from drift_b200 import Formats
    from drift_b200.dump_tables import PAIRS_EXHAUSTIVE, PAIRS_SAMPLED, pair_codes

    z = np.load(GOLDEN / "formats.npz")
    for f in Formats.ALL:
        n = f.code_count()
        if f.width <= 8:
            a, b, prod, s = pair_codes(f, PAIRS_EXHAUSTIVE, n * n)
            assert (a == np.repeat(np.arange(n), n)).all() and (b == np.tile(np.arange(n), n)).all()
        else:
            a, b, prod, s = pair_codes(f, PAIRS_SAMPLED, 20_000)
            # A later window of the same stream: rows first.. match the full run.
            a2, b2, p2, s2 = pair_codes(f, PAIRS_SAMPLED, 1000, first=12_345)
            assert (a2 == a[12_345:13_345]).all() and (p2 == prod[12_345:13_345]).all()
            assert (s2 == s[12_345:13_345]).all() and (b2 == b[12_345:13_345]).all()
        for key, got in (("pair_a", a), ("pair_b", b), ("prod", prod), ("sum", s)):
            assert (got == z[f"{f.name}_{key}"]).all(), (f.name, key)


@pytest.mark.gpu
def test_files_have_dumptables_layout(tmp_path):
    from drift_b200 import Formats, dump_tables

    assert dump_tables.main([str(tmp_path)]) == 0
    for f in Formats.ALL:
        v = (tmp_path / f"values_{f.name}.csv").read_text().splitlines()
        assert v[0].startswith(f"# format={f.name} expBits={f.exp_bits} mantBits={f.mant_bits}")
        assert v[0].endswith(f"overflow=SATURATE codes={f.code_count()}")
        assert v[1] == "code,double_bits_hex,value" and len(v) == 2 + f.code_count()
        c, h, text = v[3].split(",")   # code 1: the smallest positive subnormal
        assert c == "1" and float(text) == f.min_subnormal
        assert np.uint64(int(h, 16)).view(np.float64) == f.min_subnormal
        p = (tmp_path / f"pairs_{f.name}.csv").read_text().splitlines()
        rows = f.code_count() ** 2 if f.width <= 8 else 200_000
        mode = "exhaustive" if f.width <= 8 else "sampled seed=0x51ED1EA5"
        assert p[0] == f"# format={f.name} mode={mode} pairs={rows}"
        assert p[1] == "a,b,prod_code,sum_code" and len(p) == 2 + rows


@pytest.mark.gpu
def test_bad_arguments():
    from drift_b200 import DriftError, Formats
    from drift_b200.dump_tables import PAIRS_EXHAUSTIVE, pair_codes

    with pytest.raises(DriftError):
        pair_codes(Formats.E2M1, PAIRS_EXHAUSTIVE, 257)   # 16 codes: 256 pairs
    with pytest.raises(DriftError):
        pair_codes(Formats.E2M1, 7, 1)
