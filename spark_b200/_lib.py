"""ctypes binding of libspark_b200.so (the C ABI in include/spark_b200.h).

The shared library is built ahead of time (``__graft_entry__.build()`` or
``python -m spark_b200._build``) and loaded from this directory.  A missing
library is an error: there is no CPU fallback for any operation.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libspark_b200.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "spark_b200.h")

OK = 0
ERR_INVALID = -1
ERR_ALIGNMENT = -2
ERR_UNSUPPORTED = -3
ERR_WORKSPACE = -4
ERR_DEVICE = -5

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
FMT_SPFP2, FMT_SPFP2_V1, FMT_FP3, FMT_NVFP4, FMT_TWOFOUR = 0, 1, 2, 3, 4
LAYOUT_TILED = 0x100
PATH_TCGEN05 = 0x200
EPILOGUE_SILU = 0x400


CHAIN_LINEAR, CHAIN_SILU_MUL = 0, 1


class SparkChainOp(ctypes.Structure):
    """struct SparkChainOp of include/spark_b200.h."""
    _fields_ = [("kind", ctypes.c_int), ("fmt", ctypes.c_int), ("wq", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("x", ctypes.c_void_p), ("x2", ctypes.c_void_p), ("ic", ctypes.c_int64), ("ldx", ctypes.c_int64),
                ("oc", ctypes.c_int64), ("bias", ctypes.c_void_p), ("bias_dtype", ctypes.c_int),
                ("y", ctypes.c_void_p), ("y_dtype", ctypes.c_int), ("ldy", ctypes.c_int64), ("dep", ctypes.c_int * 2)]


class SparkBatchAllReduce(ctypes.Structure):
    """struct SparkBatchAllReduce of include/spark_b200.h."""
    _fields_ = [("op", ctypes.c_int), ("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("recv", ctypes.c_void_p), ("counter", ctypes.c_void_p)]


class SparkError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t

_SIGNATURES = {
    "spark_last_error": (ctypes.c_char_p, []),
    "spark_version": (_i, []),
    "spark_spfp2_pack": (_i, [_p, _i, _i64, _p, _p, _p]),
    "spark_spfp2_pack_v1": (_i, [_p, _i, _i64, _p, _p, _p]),
    "spark_spfp2_unpack": (_i, [_p, _i64, _p, _i, _p]),
    "spark_spfp2_legacy_decode": (_i, [_p, _i64, _p, _i, _p]),
    "spark_spfp2_unpack_v1": (_i, [_p, _i64, _p, _i, _p]),
    "spark_spfp2_fake_quant": (_i, [_p, _i, _i64, _p, _i, _p]),
    "spark_fp3_pack": (_i, [_p, _i, _i64, _i64, _p, _p, _p]),
    "spark_fp3_pack_nibble": (_i, [_p, _i, _i64, _i64, _p, _p, _p]),
    "spark_fp3_unpack": (_i, [_p, _p, _i64, _i64, _p, _i, _p]),
    "spark_fp3_unpack_nibble": (_i, [_p, _p, _i64, _i64, _p, _i, _p]),
    "spark_fp3_fake_quant": (_i, [_p, _i, _i64, _i64, _p, _i, _p]),
    "spark_nvfp4_pack": (_i, [_p, _i, _i64, _i64, _p, _p, _p]),
    "spark_nvfp4_unpack": (_i, [_p, _p, _i64, _i64, _p, _i, _p]),
    "spark_nvfp4_fake_quant": (_i, [_p, _i, _i64, _i64, _p, _i, _p]),
    "spark_twofour_pack": (_i, [_p, _i, _i64, _i64, _p, _p]),
    "spark_twofour_unpack": (_i, [_p, _i64, _p, _i, _p]),
    "spark_twofour_fake_quant": (_i, [_p, _i, _i64, _p, _i, _p]),
    "spark_int8_fake_quant": (_i, [_p, _i, _i64, _i64, _p, _i, _p]),
    "spark_int8_pack": (_i, [_p, _i, _i64, _i64, _p, _p, _p]),
    "spark_int8_unpack": (_i, [_p, _p, _i64, _i64, _p, _i, _p]),
    "spark_linear_workspace_size": (_sz, [_i, _i64, _i64, _i64]),
    "spark_linear": (_i, [_i, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _p, _i, _p, _i, _i64, _p, _sz, _p]),
    "spark_linear_prefetch": (_i, [_i, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _p, _i, _p, _i, _i64, _p, _sz, _p,
                                   _i64, _p]),
    "spark_linear_batch_workspace_size": (_sz, [_p, _i, _i64]),
    "spark_linear_batch": (_i, [_p, _i, _i64, _p, _sz, _p]),
    "spark_linear_batch_ar_workspace_size": (_sz, [_p, _i, _i64, _p]),
    "spark_batch_ar_recv_bytes": (_i64, [_i, _i64, _i64]),
    "spark_linear_batch_ar": (_i, [_p, _i, _i64, _p, _p, _sz, _p]),
    "spark_linear_chain_workspace_size": (_sz, [_i]),
    "spark_linear_chain": (_i, [_p, _i, _i64, _p, _sz, _p]),
    "spark_linear_noalloc": (_i, [_i, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _p, _i, _p, _i, _i64, _p]),
    "spark_workspace_check": (_i, [_p, _p]),
    "spark_tiled_bytes": (_sz, [_i, _i64, _i64]),
    "spark_tile_weights": (_i, [_i, _p, _p, _i64, _i64, _p, _p]),
    "spark_silu_mul": (_i, [_p, _p, _p, _i, _i64, _p]),
    "spark_silu_mul_rows": (_i, [_p, _p, _i64, _p, _i64, _i, _i64, _i64, _p]),
    "spark_nvfp4_embedding": (_i, [_p, _p, _i64, _i64, _p, _i64, _p, _i, _p, _p]),
    "spark_nvfp4_native_linear": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _p, _i, _i64, _p, _p]),
    "spark_twofour_sparse_linear": (_i, [_p, _p, _i64, _i64, _i64, _p, _i, _p, _i, _i64, _p, _p]),
    "spark_peer_flags_count": (_i, [_i]),
    "spark_peer_allreduce": (_i, [_p, _p, _i, _i, _i64, _i, _p, _i, _p, _p, _p]),
    "spark_ipc_handle": (_i, [_p, _p, ctypes.POINTER(ctypes.c_int64)]),
    "spark_ipc_open": (_i, [_p, _i64, ctypes.POINTER(ctypes.c_void_p)]),
    "spark_ipc_close": (_i, [_p, _i64]),
}

_lib = None


def header_symbols() -> list[str]:
    """Names of every function include/spark_b200.h declares."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"SPARK_API\s+[\w\s\*]*?\b(spark_\w+)\s*\(", txt)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(spark_b200 has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().spark_last_error().decode(errors="replace")


def call(name: str, *args) -> None:
    """Invoke a C-ABI function and raise SparkError on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        raise SparkError(name, rc, last_error())
