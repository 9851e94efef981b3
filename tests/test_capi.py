"""The C ABI without a GPU: the library loads, exports every symbol the
header declares with the struct layout the header gives, and its host-only
entry points agree with the oracle. No compute call is made here."""
import ctypes
import re
from pathlib import Path

import pytest

from drift_b200 import _lib
from oracle import oracle as O

HEADER = Path(__file__).resolve().parent.parent / "include" / "drift_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"DRIFT_API\s+[\w\s\*]+?\b(drift_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = declared_symbols()
    assert len(names) >= 16
    for n in names:
        assert hasattr(lib, n), n


def test_binding_covers_the_header():
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_policy_struct_layout():
    assert ctypes.sizeof(_lib.DriftPolicy) == 64
    assert ctypes.sizeof(_lib.DriftPolicy) == ctypes.sizeof(O.OraclePolicy)


def test_version_string():
    assert b"sm_100a" in _lib.load().drift_version()


@pytest.mark.parametrize("fid", range(7))
def test_format_info_matches_oracle(fid):
    mx, mn, ms, w = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int32()
    _lib.check(_lib.load().drift_format_info(fid, mx, mn, ms, w))
    assert (mx.value, mn.value, ms.value, w.value) == O.format_info(fid)


@pytest.mark.parametrize("fid", range(7))
@pytest.mark.parametrize("amax", [0.0, 1e-300, 0.37, 3.0, 448.0, 1e300, float("inf"), float("nan")])
def test_per_tensor_scale_matches_oracle(fid, amax):
    out = ctypes.c_double()
    _lib.check(_lib.load().drift_per_tensor_scale(fid, amax, ctypes.byref(out)))
    assert out.value == O.per_tensor_scale(fid, amax)


def test_bad_format_is_einval():
    out = ctypes.c_double()
    assert _lib.load().drift_per_tensor_scale(9, 1.0, ctypes.byref(out)) == _lib.EINVAL
    assert "format" in _lib.last_error()
