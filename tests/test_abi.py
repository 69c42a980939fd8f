"""The C-ABI library loads without a GPU, exports every symbol the header
declares, and rejects invalid calls before touching the device."""
from __future__ import annotations

import ctypes

import pytest

from spark_b200 import _lib


def test_library_exports_every_header_symbol():
    syms = _lib.header_symbols()
    assert len(syms) >= 20
    L = _lib.lib()
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert set(syms) == set(_lib._SIGNATURES), "ctypes signatures out of sync with the header"


def test_version():
    assert _lib.lib().spark_version() >= 100


@pytest.mark.parametrize("call,args", [
    ("spark_spfp2_pack", (None, 0, 16, None, None, None)),
    ("spark_spfp2_pack", (ctypes.c_void_p(16), 0, 12, ctypes.c_void_p(16), None, None)),   # numel % 8
    ("spark_spfp2_pack", (ctypes.c_void_p(16), 7, 16, ctypes.c_void_p(16), None, None)),   # bad dtype
    ("spark_fp3_pack", (None, 0, 4, 16, None, None, None)),
    ("spark_twofour_fake_quant", (ctypes.c_void_p(16), 0, 20, ctypes.c_void_p(16), 0, None)),
])
def test_invalid_calls_are_rejected(call, args):
    with pytest.raises(_lib.SparkError) as e:
        _lib.call(call, *args)
    assert e.value.code == _lib.ERR_INVALID
    assert call in _lib.last_error() or "numel" in _lib.last_error() or "dtype" in _lib.last_error()


def test_linear_argument_validation():
    p = ctypes.c_void_p(256)
    base = dict(fmt=0, wq=p, sc=None, x=p, xd=1, M=1, oc=16, ic=256, ldx=256, b=None, bd=0, y=p, yd=0, ldy=16,
                ws=None, wsb=0, st=None)

    def run(**kw):
        a = {**base, **kw}
        return _lib.lib().spark_linear(a["fmt"], a["wq"], a["sc"], a["x"], a["xd"], a["M"], a["oc"], a["ic"],
                                       a["ldx"], a["b"], a["bd"], a["y"], a["yd"], a["ldy"], a["ws"], a["wsb"],
                                       a["st"])

    assert run(fmt=9) == _lib.ERR_INVALID
    assert run(wq=None) == _lib.ERR_INVALID
    assert run(ldx=100) == _lib.ERR_INVALID
    assert run(fmt=2) == _lib.ERR_INVALID          # FP3 without scales
    assert run(xd=5) == _lib.ERR_INVALID
    assert run(M=0) == _lib.OK                      # nothing to do
