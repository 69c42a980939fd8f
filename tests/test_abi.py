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


def test_batch_allreduce_argument_validation():
    """spark_linear_batch_ar rejects bad all-reduce arguments on the host,
    before it plans the launch (no device needed)."""
    P = ctypes.c_void_p
    ops = (_lib.SparkChainOp * 2)()
    for k in range(2):
        c = ops[k]
        c.kind, c.fmt, c.wq, c.x, c.ic, c.ldx = _lib.CHAIN_LINEAR, _lib.FMT_SPFP2 | _lib.LAYOUT_TILED, 256, 256, 512, 512
        c.oc, c.y, c.y_dtype, c.ldy = 256, 256, _lib.DTYPE_BF16, 256
        c.dep[0] = c.dep[1] = -1
    ops[1].dep[0] = 0
    L = _lib.lib()

    def run(op, world, rank):
        ar = _lib.SparkBatchAllReduce(op, world, rank, None, None)
        rc = L.spark_linear_batch_ar(ctypes.cast(ops, P), 2, 1, ctypes.byref(ar), P(256), 1 << 20, None)
        ws = L.spark_linear_batch_ar_workspace_size(ctypes.cast(ops, P), 2, 1, ctypes.byref(ar))
        return rc, ws

    assert run(1, 9, 0) == (_lib.ERR_INVALID, 0)             # more ranks than peers
    assert run(1, 2, 2) == (_lib.ERR_INVALID, 0)             # rank out of range
    assert run(2, 2, 0) == (_lib.ERR_INVALID, 0)             # op not in the batch
    assert run(0, 2, 0) == (_lib.ERR_UNSUPPORTED, 0)         # a later op reads the summed output
    assert "later launch" in _lib.last_error()
    assert L.spark_linear_batch_ar(ctypes.cast(ops, P), 2, 1, None, P(256), 1 << 20, None) == _lib.ERR_INVALID
    # 2 call parities x 2 ranks x 160 row groups x 16 tokens x 16 rows, 8-byte words
    assert L.spark_batch_ar_recv_bytes(2, 16, 2560) == 2 * 2 * 160 * 16 * 16 * 8
    assert L.spark_batch_ar_recv_bytes(0, 16, 2560) == 0 and L.spark_batch_ar_recv_bytes(9, 1, 16) == 0
    assert L.spark_batch_ar_recv_bytes(2, 17, 16) == 0


def test_tensor_core_modes_validate_arguments_on_the_host():
    """The sparse 2:4 and the native NVFP4 entry points reject bad shapes and
    null pointers before they touch the device."""
    L = _lib.lib()
    P = ctypes.c_void_p
    p = P(256)
    err = P(256)
    # 2:4 sparse: oc must be a multiple of 128, ic of 128
    assert L.spark_twofour_sparse_linear(p, p, 4, 100, 256, None, 0, p, 1, 100, err, None) == _lib.ERR_INVALID
    assert L.spark_twofour_sparse_linear(p, p, 4, 128, 96, None, 0, p, 1, 128, err, None) == _lib.ERR_INVALID
    assert L.spark_twofour_sparse_linear(None, p, 4, 128, 128, None, 0, p, 1, 128, err, None) == _lib.ERR_INVALID
    assert "multiple of 128" in _lib.last_error() or "null" in _lib.last_error()
    assert L.spark_twofour_sparse_linear(p, P(258), 4, 128, 128, None, 0, p, 1, 128, err, None) == _lib.ERR_ALIGNMENT
    # native NVFP4: oc a multiple of 128, ic of 256
    assert L.spark_nvfp4_native_linear(p, p, p, p, 4, 100, 256, p, 1, 100, err, None) == _lib.ERR_INVALID
    assert L.spark_nvfp4_native_linear(p, p, p, p, 4, 128, 128, p, 1, 128, err, None) == _lib.ERR_INVALID
    assert L.spark_nvfp4_native_linear(p, p, None, p, 4, 128, 256, p, 1, 128, err, None) == _lib.ERR_INVALID
    assert L.spark_nvfp4_native_linear(P(264), p, p, p, 4, 128, 256, p, 1, 128, err, None) == _lib.ERR_ALIGNMENT
