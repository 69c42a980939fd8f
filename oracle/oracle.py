"""numpy front end for the C oracle (oracle/spark_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` use this module as the checker.  The product
(``spark_b200``) never imports it.

Each function mirrors one reference emulator function of DJAzzs/SPARK
(``01_core/block_fp2_emu.py``, ``fp3_emu.py``, ``nvfp4_emu.py``,
``two_four.py``) and returns numpy arrays with the reference's layout.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, strict fp32)."""
    src = os.path.join(_HERE, "spark_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "-B" if force else "all"], check=True,
                       stdout=subprocess.DEVNULL)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "spo_spfp2_center": (ctypes.c_int, [ctypes.c_float]),
            "spo_spfp2_search": (ctypes.c_int, [_f32p]),
            "spo_spfp2_pack3": (None, [_f32p, _i64, _u8p, _u8p]),
            "spo_spfp2_pack_paired": (None, [_f32p, _i64, _u8p, _u8p]),
            "spo_spfp2_unpack3": (None, [_u8p, _i64, _f32p]),
            "spo_spfp2_unpack_paired": (None, [_u8p, _i64, _i64, _f32p]),
            "spo_spfp2_fake_quant": (None, [_f32p, _i64, _f32p]),
            "spo_f32_to_e4m3": (ctypes.c_uint8, [ctypes.c_float]),
            "spo_e4m3_to_f32": (ctypes.c_float, [ctypes.c_uint8]),
            "spo_fp3_pack3bit": (None, [_f32p, _i64, _i64, _u8p, _u8p]),
            "spo_fp3_pack_nibble": (None, [_f32p, _i64, _i64, _u8p, _u8p]),
            "spo_fp3_unpack3bit": (None, [_u8p, _u8p, _i64, _i64, _f32p]),
            "spo_fp3_unpack_nibble": (None, [_u8p, _u8p, _i64, _i64, _f32p]),
            "spo_fp3_fake_quant": (None, [_f32p, _i64, _i64, _f32p]),
            "spo_nvfp4_pack": (None, [_f32p, _i64, _i64, _u8p, _u8p]),
            "spo_nvfp4_unpack": (None, [_u8p, _u8p, _i64, _i64, _f32p]),
            "spo_nvfp4_fake_quant": (None, [_f32p, _i64, _i64, _f32p]),
            "spo_twofour_search": (ctypes.c_int, [_f32p]),
            "spo_twofour_pack": (None, [_f32p, _i64, _i64, _u8p]),
            "spo_twofour_unpack": (None, [_u8p, _i64, _i64, _f32p]),
            "spo_twofour_fake_quant": (None, [_f32p, _i64, _f32p]),
            "spo_linear_f64": (None, [_f32p, _i64, _i64, _f32p, _i64, _f32p, _f64p]),
            "spo_num_threads": (ctypes.c_int, []),
            "spo_spfp2_legacy_decode": (None, [_u8p, _i64, _f32p]),
            "spo_set_num_threads": (None, [ctypes.c_int]),
            "spo_cpu_spfp2_linear": (None, [_u8p, _f32p, _i64, _i64, _i64, _f32p]),
            "spo_cpu_fp3_linear": (None, [_u8p, _u8p, _f32p, _i64, _i64, _i64, _f32p]),
            "spo_cpu_nvfp4_linear": (None, [_u8p, _u8p, _f32p, _i64, _i64, _i64, _f32p]),
            "spo_center_thresholds": (ctypes.POINTER(ctypes.c_uint32), []),
            "spo_int8_fake_quant": (None, [_f32p, _i64, _i64, _f32p]),
            "spo_int8_pack": (None, [_f32p, _i64, _i64, ctypes.POINTER(ctypes.c_int8), _f32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint8))


def _p(a, t):
    return a.ctypes.data_as(t)


# ---------------------------------------------------------------- SPFP2
def center_thresholds() -> np.ndarray:
    ptr = lib().spo_center_thresholds()
    return np.array([ptr[i] for i in range(15)], dtype=np.uint32)


def spfp2_center(maxv: float) -> int:
    return lib().spo_spfp2_center(float(maxv))


def pack_blockwise_search(w) -> tuple[np.ndarray, np.ndarray]:
    """block_fp2_emu.pack_blockwise_search(w, window=2) -> (packed3, expv)."""
    w = _f32(w).reshape(-1)
    nb = w.size // 8
    out = np.zeros(nb * 3, np.uint8)
    expv = np.zeros(nb, np.uint8)
    lib().spo_spfp2_pack3(_p(w, _f32p), w.size, _p(out, _u8p), _p(expv, _u8p))
    return out, expv


def pack_blockwise_paired(w) -> tuple[np.ndarray, np.ndarray]:
    """block_fp2_emu.pack_blockwise_paired(w) -> (packed5, expv)."""
    w = _f32(w).reshape(-1)
    nb = w.size // 8
    out = np.zeros(((nb + 1) // 2) * 5, np.uint8)
    expv = np.zeros(nb, np.uint8)
    lib().spo_spfp2_pack_paired(_p(w, _f32p), w.size, _p(out, _u8p), _p(expv, _u8p))
    return out, expv


def unpack_blockwise(packed3) -> np.ndarray:
    p = _u8(packed3)
    nb = p.size // 3
    out = np.zeros(nb * 8, np.float32)
    lib().spo_spfp2_unpack3(_p(p, _u8p), nb, _p(out, _f32p))
    return out


def unpack_blockwise_paired(packed5, n_elements: int) -> np.ndarray:
    p = _u8(packed5)
    npairs = p.size // 5
    out = np.zeros(n_elements, np.float32)
    lib().spo_spfp2_unpack_paired(_p(p, _u8p), npairs, n_elements, _p(out, _f32p))
    return out


def spfp2_legacy_decode(packed5) -> np.ndarray:
    """block_fp2_kernel.cu's 16-weight single-exponent blocks (decode_fp32 / decode_fp16)."""
    p = _u8(packed5)
    nb = p.size // 5
    out = np.zeros(nb * 16, np.float32)
    lib().spo_spfp2_legacy_decode(_p(p, _u8p), nb, _p(out, _f32p))
    return out


def channel_fake_quantize(w) -> np.ndarray:
    w = _f32(w)
    out = np.zeros_like(w)
    lib().spo_spfp2_fake_quant(_p(w, _f32p), w.size, _p(out, _f32p))
    return out


# ---------------------------------------------------------------- FP8 / FP3 / NVFP4
def f32_to_e4m3(x) -> np.ndarray:
    x = _f32(x).reshape(-1)
    L = lib()
    return np.array([L.spo_f32_to_e4m3(float(v)) for v in x], dtype=np.uint8)


def e4m3_to_f32(b) -> np.ndarray:
    b = _u8(b).reshape(-1)
    L = lib()
    return np.array([L.spo_e4m3_to_f32(int(v)) for v in b], dtype=np.float32)


def _nb(ic):
    return (ic + 15) // 16


def fp3_pack_3bit(w) -> tuple[np.ndarray, np.ndarray]:
    w = _f32(w)
    oc, ic = w.shape
    n = oc * _nb(ic) * 16
    packed = np.zeros(((n + 7) // 8) * 3, np.uint8)
    scales = np.zeros(oc * _nb(ic), np.uint8)
    lib().spo_fp3_pack3bit(_p(w, _f32p), oc, ic, _p(packed, _u8p), _p(scales, _u8p))
    return packed, scales


def fp3_pack(w) -> tuple[np.ndarray, np.ndarray]:
    w = _f32(w)
    oc, ic = w.shape
    n = oc * _nb(ic) * 16
    packed = np.zeros((n + 1) // 2, np.uint8)
    scales = np.zeros(oc * _nb(ic), np.uint8)
    lib().spo_fp3_pack_nibble(_p(w, _f32p), oc, ic, _p(packed, _u8p), _p(scales, _u8p))
    return packed, scales


def fp3_unpack_3bit(packed, scales, oc, ic) -> np.ndarray:
    p, s = _u8(packed), _u8(scales)
    out = np.zeros((oc, ic), np.float32)
    lib().spo_fp3_unpack3bit(_p(p, _u8p), _p(s, _u8p), oc, ic, _p(out, _f32p))
    return out


def fp3_unpack(packed, scales, oc, ic) -> np.ndarray:
    p, s = _u8(packed), _u8(scales)
    out = np.zeros((oc, ic), np.float32)
    lib().spo_fp3_unpack_nibble(_p(p, _u8p), _p(s, _u8p), oc, ic, _p(out, _f32p))
    return out


def fp3_fake_quant(w) -> np.ndarray:
    w = _f32(w)
    oc, ic = w.shape
    out = np.zeros((oc, ic), np.float32)
    lib().spo_fp3_fake_quant(_p(w, _f32p), oc, ic, _p(out, _f32p))
    return out


def nvfp4_pack(w) -> tuple[np.ndarray, np.ndarray]:
    w = _f32(w)
    oc, ic = w.shape
    n = oc * _nb(ic) * 16
    packed = np.zeros((n + 1) // 2, np.uint8)
    scales = np.zeros(oc * _nb(ic), np.uint8)
    lib().spo_nvfp4_pack(_p(w, _f32p), oc, ic, _p(packed, _u8p), _p(scales, _u8p))
    return packed, scales


def nvfp4_unpack(packed, scales, oc, ic) -> np.ndarray:
    p, s = _u8(packed), _u8(scales)
    out = np.zeros((oc, ic), np.float32)
    lib().spo_nvfp4_unpack(_p(p, _u8p), _p(s, _u8p), oc, ic, _p(out, _f32p))
    return out


def nvfp4_fake_quant(w) -> np.ndarray:
    w = _f32(w)
    oc, ic = w.shape
    out = np.zeros((oc, ic), np.float32)
    lib().spo_nvfp4_fake_quant(_p(w, _f32p), oc, ic, _p(out, _f32p))
    return out


# ---------------------------------------------------------------- INT8
def int8_fake_quant(w) -> np.ndarray:
    """int8_emu.py:12-18 (per-row symmetric INT8 round trip)."""
    w = _f32(w)
    oc, ic = w.shape
    out = np.zeros((oc, ic), np.float32)
    lib().spo_int8_fake_quant(_p(w, _f32p), oc, ic, _p(out, _f32p))
    return out


def ptq_int8_pack(w) -> tuple[np.ndarray, np.ndarray]:
    """int8_emu.py:37-46: (q int8 [oc, ic], scale fp32 [oc])."""
    w = _f32(w)
    oc, ic = w.shape
    q = np.zeros((oc, ic), np.int8)
    scale = np.zeros(oc, np.float32)
    lib().spo_int8_pack(_p(w, _f32p), oc, ic, _p(q, ctypes.POINTER(ctypes.c_int8)), _p(scale, _f32p))
    return q, scale


# ---------------------------------------------------------------- 2:4
def two_four_pack(w) -> np.ndarray:
    w = _f32(w)
    oc, ic = w.shape
    nb = oc * _nb(ic)
    out = np.zeros(((nb + 1) // 2) * 7, np.uint8)
    lib().spo_twofour_pack(_p(w, _f32p), oc, ic, _p(out, _u8p))
    return out


def two_four_unpack(packed, n_elements: int) -> np.ndarray:
    p = _u8(packed)
    npairs = p.size // 7
    out = np.zeros(n_elements, np.float32)
    lib().spo_twofour_unpack(_p(p, _u8p), npairs, n_elements, _p(out, _f32p))
    return out


def two_four_fake_quant(w) -> np.ndarray:
    w = _f32(w)
    out = np.zeros_like(w)
    lib().spo_twofour_fake_quant(_p(w, _f32p), w.size, _p(out, _f32p))
    return out


# ---------------------------------------------------------------- linear
def linear_f64(x, W, bias=None) -> np.ndarray:
    """y = x @ W.T (+ bias) with fp64 accumulation."""
    x = _f32(x)
    W = _f32(W)
    M, ic = x.shape
    oc = W.shape[0]
    y = np.zeros((M, oc), np.float64)
    b = _f32(bias) if bias is not None else None
    lib().spo_linear_f64(_p(x, _f32p), M, ic, _p(W, _f32p), oc,
                         _p(b, _f32p) if b is not None else None, _p(y, _f64p))
    return y


def num_threads() -> int:
    return lib().spo_num_threads()


def set_num_threads(n: int) -> None:
    lib().spo_set_num_threads(int(n))


def cpu_spfp2_linear(packed5, x, oc, ic) -> np.ndarray:
    p = _u8(packed5)
    x = _f32(x)
    y = np.zeros((x.shape[0], oc), np.float32)
    lib().spo_cpu_spfp2_linear(_p(p, _u8p), _p(x, _f32p), x.shape[0], oc, ic, _p(y, _f32p))
    return y


def cpu_fp3_linear(codes, scales, x, oc, ic) -> np.ndarray:
    c, s = _u8(codes), _u8(scales)
    x = _f32(x)
    y = np.zeros((x.shape[0], oc), np.float32)
    lib().spo_cpu_fp3_linear(_p(c, _u8p), _p(s, _u8p), _p(x, _f32p), x.shape[0], oc, ic, _p(y, _f32p))
    return y


def cpu_nvfp4_linear(codes, scales, x, oc, ic) -> np.ndarray:
    c, s = _u8(codes), _u8(scales)
    x = _f32(x)
    y = np.zeros((x.shape[0], oc), np.float32)
    lib().spo_cpu_nvfp4_linear(_p(c, _u8p), _p(s, _u8p), _p(x, _f32p), x.shape[0], oc, ic, _p(y, _f32p))
    return y
