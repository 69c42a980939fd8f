"""torch-facing wrappers of the C ABI: allocate outputs, pass raw pointers and
the current CUDA stream, raise on a non-zero status.

Every function runs the sm_100a kernels; tensors on the CPU are copied to the
current CUDA device first and results are returned on the input's device, so
the functions can stand in for the reference emulators that take CPU tensors.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from ._lib import (DTYPE_BF16, DTYPE_F16, DTYPE_F32, FMT_FP3, FMT_NVFP4, FMT_SPFP2, FMT_SPFP2_V1,
                   FMT_TWOFOUR, LAYOUT_TILED, PATH_TCGEN05, EPILOGUE_SILU, call)

_DT = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}

FORMATS = {"spfp2": FMT_SPFP2, "spfp2_v1": FMT_SPFP2_V1, "fp3": FMT_FP3, "nvfp4": FMT_NVFP4,
           "twofour": FMT_TWOFOUR}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def _cuda(t: torch.Tensor) -> torch.Tensor:
    if not torch.cuda.is_available():
        raise RuntimeError("spark_b200 needs a CUDA device (no CPU fallback)")
    if not t.is_cuda:
        t = t.to(torch.device("cuda", torch.cuda.current_device()))
    return t.contiguous()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _bytes(t: torch.Tensor) -> torch.Tensor:
    """uint8 view of a packed buffer (uint8 or float8_e4m3fn)."""
    t = _cuda(t)
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


def _home(out: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return out if like.is_cuda else out.to(like.device)


# ------------------------------------------------------------------ SPFP2
def spfp2_pack(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """pack_blockwise_paired: (packed uint8[ceil(nb/2)*5], expv uint8[nb])."""
    x = _cuda(w.detach())
    n = x.numel()
    nb = n // 8
    packed = torch.empty(((nb + 1) // 2) * 5, dtype=torch.uint8, device=x.device)
    expv = torch.empty(nb, dtype=torch.uint8, device=x.device)
    call("spark_spfp2_pack", _p(x), _dt(x), n, _p(packed), _p(expv), _stream(x))
    return _home(packed, w), _home(expv, w)


def spfp2_pack_v1(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """pack_blockwise_search(window=2): (packed uint8[nb*3], expv uint8[nb])."""
    x = _cuda(w.detach())
    n = x.numel()
    nb = n // 8
    packed = torch.empty(nb * 3, dtype=torch.uint8, device=x.device)
    expv = torch.empty(nb, dtype=torch.uint8, device=x.device)
    call("spark_spfp2_pack_v1", _p(x), _dt(x), n, _p(packed), _p(expv), _stream(x))
    return _home(packed, w), _home(expv, w)


def spfp2_unpack(packed: torch.Tensor, n_elements: int, dtype=torch.float32) -> torch.Tensor:
    """unpack_blockwise_paired."""
    p = _bytes(packed)
    out = torch.empty(n_elements, dtype=dtype, device=p.device)
    if p.numel() < (n_elements + 15) // 16 * 5:
        raise ValueError(f"packed has {p.numel()} bytes, {n_elements} elements need {(n_elements + 15) // 16 * 5}")
    call("spark_spfp2_unpack", _p(p), n_elements, _p(out), _DT[dtype], _stream(p))
    return _home(out, packed)


def spfp2_unpack_v1(packed: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """unpack_blockwise (3-byte blocks)."""
    p = _bytes(packed)
    nb = p.numel() // 3
    out = torch.empty(nb * 8, dtype=dtype, device=p.device)
    call("spark_spfp2_unpack_v1", _p(p), nb, _p(out), _DT[dtype], _stream(p))
    return _home(out, packed)


def spfp2_fake_quant(w: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """channel_fake_quantize forward over the flattened tensor's 8-blocks."""
    x = _cuda(w.detach())
    out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    call("spark_spfp2_fake_quant", _p(x), _dt(x), x.numel(), _p(out), _dt(out), _stream(x))
    return _home(out, w)


# ------------------------------------------------------------------ FP3 / NVFP4
def _codes_shapes(oc: int, ic: int):
    nb = (ic + 15) // 16
    return oc * nb, oc * nb * 16


def fp3_pack(w: torch.Tensor, nibble: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """fp3_pack_3bit (nibble=False) or fp3_pack (nibble=True): (codes, scales e4m3fn)."""
    x = _cuda(w.detach())
    oc, ic = x.shape
    nblk, n = _codes_shapes(oc, ic)
    codes = torch.empty((n + 1) // 2 if nibble else (n + 7) // 8 * 3, dtype=torch.uint8, device=x.device)
    scales = torch.empty(nblk, dtype=torch.uint8, device=x.device)
    call("spark_fp3_pack_nibble" if nibble else "spark_fp3_pack", _p(x), _dt(x), oc, ic, _p(codes), _p(scales),
         _stream(x))
    return _home(codes, w), _home(scales.view(torch.float8_e4m3fn), w)


def fp3_unpack(codes: torch.Tensor, scales: torch.Tensor, oc: int, ic: int, nibble: bool = False,
               dtype=torch.float32) -> torch.Tensor:
    c, s = _bytes(codes), _bytes(scales)
    out = torch.empty(oc, ic, dtype=dtype, device=c.device)
    call("spark_fp3_unpack_nibble" if nibble else "spark_fp3_unpack", _p(c), _p(s), oc, ic, _p(out), _DT[dtype],
         _stream(c))
    return _home(out, codes)


def fp3_fake_quant(w: torch.Tensor, out_dtype=None) -> torch.Tensor:
    x = _cuda(w.detach())
    oc, ic = x.shape
    out = torch.empty(oc, ic, dtype=out_dtype or torch.float32, device=x.device)
    call("spark_fp3_fake_quant", _p(x), _dt(x), oc, ic, _p(out), _dt(out), _stream(x))
    return _home(out, w)


def nvfp4_pack(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    x = _cuda(w.detach())
    oc, ic = x.shape
    nblk, n = _codes_shapes(oc, ic)
    codes = torch.empty((n + 1) // 2, dtype=torch.uint8, device=x.device)
    scales = torch.empty(nblk, dtype=torch.uint8, device=x.device)
    call("spark_nvfp4_pack", _p(x), _dt(x), oc, ic, _p(codes), _p(scales), _stream(x))
    return _home(codes, w), _home(scales.view(torch.float8_e4m3fn), w)


def nvfp4_unpack(codes: torch.Tensor, scales: torch.Tensor, oc: int, ic: int, dtype=torch.float32) -> torch.Tensor:
    c, s = _bytes(codes), _bytes(scales)
    out = torch.empty(oc, ic, dtype=dtype, device=c.device)
    call("spark_nvfp4_unpack", _p(c), _p(s), oc, ic, _p(out), _DT[dtype], _stream(c))
    return _home(out, codes)


def nvfp4_native_linear(codes: torch.Tensor, scales: torch.Tensor, x: torch.Tensor, oc: int, ic: int,
                        out_dtype=torch.bfloat16, xq=None) -> torch.Tensor:
    """Native NVFP4 x NVFP4 linear (spark_nvfp4_native_linear, a reported mode:
    the activations are quantised to NVFP4 by the weights' own quantiser, so
    the result differs from the parity path `linear("nvfp4", ...)` by the
    activations' FP4 rounding).  codes / scales: nvfp4_pack of the weight;
    x: [M, ic]; xq: an already packed (codes, scales) of x, to skip that step."""
    xc, xs = nvfp4_pack(x) if xq is None else xq
    M = x.shape[0]
    y = torch.empty(M, oc, dtype=out_dtype, device=x.device)
    ws = workspace(x.device, 1 << 20)
    call("spark_nvfp4_native_linear", _p(_bytes(codes)), _p(_bytes(scales)), _p(_bytes(xc)), _p(_bytes(xs)), M, oc,
         ic, _p(y), _dt(y), oc, _p(ws), _stream(x))
    return y


def twofour_sparse_linear(packed: torch.Tensor, x: torch.Tensor, oc: int, ic: int, bias=None,
                          out_dtype=torch.bfloat16) -> torch.Tensor:
    """2:4 linear on the sparse tensor cores (spark_twofour_sparse_linear):
    the kept values of every group of four with their positions as the MMA's
    sparsity metadata.  x: bf16 [M, ic]; packed: twofour_pack of [oc, ic]."""
    x2 = _cuda(x).contiguous()
    if x2.dtype != torch.bfloat16:
        raise TypeError("twofour_sparse_linear: bf16 activations")
    M = x2.shape[0]
    y = torch.empty(M, oc, dtype=out_dtype, device=x2.device)
    ws = workspace(x2.device, 1 << 20)
    b = _cuda(bias) if bias is not None else None
    call("spark_twofour_sparse_linear", _p(_bytes(packed)), _p(x2), M, oc, ic, _p(b), _dt(b) if b is not None else 0,
         _p(y), _dt(y), oc, _p(ws), _stream(x2))
    return y


def nvfp4_fake_quant(w: torch.Tensor, out_dtype=None) -> torch.Tensor:
    x = _cuda(w.detach())
    oc, ic = x.shape
    out = torch.empty(oc, ic, dtype=out_dtype or torch.float32, device=x.device)
    call("spark_nvfp4_fake_quant", _p(x), _dt(x), oc, ic, _p(out), _dt(out), _stream(x))
    return _home(out, w)


# ------------------------------------------------------------------ 2:4
def nvfp4_embedding(codes: torch.Tensor, scales: torch.Tensor, num_embeddings: int, dim: int,
                    ids: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """Rows `ids` of a packed NVFP4 [num_embeddings, dim] table, decoded:
    F.embedding(ids, nvfp4_unpack(table)) without unpacking the table.  Out-of-
    range ids give zero rows and an error that check_device_errors() raises."""
    if not ids.is_cuda:
        raise RuntimeError("spark_b200.nvfp4_embedding: ids must be a CUDA tensor")
    flat = ids.reshape(-1).to(torch.int64).contiguous()
    out = torch.empty(flat.numel(), dim, dtype=dtype, device=ids.device)
    if out.numel() == 0:
        return out.reshape(*ids.shape, dim)
    ws = workspace(ids.device, 1 << 20)
    call("spark_nvfp4_embedding", _p(_bytes(codes)), _p(_bytes(scales)), num_embeddings, dim, _p(flat), flat.numel(),
         _p(out), _dt(out), _p(ws), _stream(ids))
    return out.reshape(*ids.shape, dim)


def twofour_pack(w: torch.Tensor) -> torch.Tensor:
    x = _cuda(w.detach())
    oc, ic = x.shape
    nblk, _ = _codes_shapes(oc, ic)
    packed = torch.empty((nblk + 1) // 2 * 7, dtype=torch.uint8, device=x.device)
    call("spark_twofour_pack", _p(x), _dt(x), oc, ic, _p(packed), _stream(x))
    return _home(packed, w)


def twofour_unpack(packed: torch.Tensor, n_elements: int, dtype=torch.float32) -> torch.Tensor:
    p = _bytes(packed)
    out = torch.empty(n_elements, dtype=dtype, device=p.device)
    call("spark_twofour_unpack", _p(p), n_elements, _p(out), _DT[dtype], _stream(p))
    return _home(out, packed)


def twofour_fake_quant(w: torch.Tensor, out_dtype=None) -> torch.Tensor:
    x = _cuda(w.detach())
    out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    call("spark_twofour_fake_quant", _p(x), _dt(x), x.numel(), _p(out), _dt(out), _stream(x))
    return _home(out, w)


# ------------------------------------------------------------------ INT8
def int8_fake_quant(w: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """int8_fake_quant: per-row symmetric INT8 round trip (fp32 out by default)."""
    x = _cuda(w.detach())
    oc, ic = x.shape
    out = torch.empty(oc, ic, dtype=out_dtype or torch.float32, device=x.device)
    call("spark_int8_fake_quant", _p(x), _dt(x), oc, ic, _p(out), _dt(out), _stream(x))
    return _home(out, w)


def int8_pack(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """ptq_int8_pack: (q int8 [oc, ic], scale fp32 [oc])."""
    x = _cuda(w.detach())
    oc, ic = x.shape
    q = torch.empty(oc, ic, dtype=torch.int8, device=x.device)
    scale = torch.empty(oc, dtype=torch.float32, device=x.device)
    call("spark_int8_pack", _p(x), _dt(x), oc, ic, _p(q), _p(scale), _stream(x))
    return _home(q, w), _home(scale, w)


def int8_unpack(q: torch.Tensor, scale: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """ptq_int8_unpack: q * scale[row]."""
    qq, s = _cuda(q), _cuda(scale.float())
    oc, ic = qq.shape
    out = torch.empty(oc, ic, dtype=dtype, device=qq.device)
    call("spark_int8_unpack", _p(qq), _p(s), oc, ic, _p(out), _DT[dtype], _stream(qq))
    return _home(out, q)


# ------------------------------------------------------------------ linear
_ws_lock = threading.Lock()
_ws: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int, stream=None) -> torch.Tensor:
    """Zero-initialised scratch for spark_linear, one per (device, stream)."""
    s = stream if stream is not None else torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), s.cuda_stream)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws[key] = buf
    return buf


def workspace_size(fmt: int, M: int, oc: int, ic: int) -> int:
    return int(_lib.lib().spark_linear_workspace_size(fmt, M, oc, ic))


def tiled_bytes(fmt, oc: int, ic: int) -> int:
    f = FORMATS[fmt] if isinstance(fmt, str) else int(fmt)
    return int(_lib.lib().spark_tiled_bytes(f, oc, ic))


def tile_weights(fmt, wq: torch.Tensor, scales, oc: int, ic: int) -> torch.Tensor | None:
    """Fragment-major copy of a packed weight for the decode GEMV (None when the
    shape has no tiled layout).  Same bytes, permuted; scales embedded."""
    f = FORMATS[fmt] if isinstance(fmt, str) else int(fmt)
    n = tiled_bytes(f, oc, ic)
    if n == 0:
        return None
    w = _bytes(wq)
    s = _bytes(scales) if scales is not None else None
    out = torch.empty(n, dtype=torch.uint8, device=w.device)
    call("spark_tile_weights", f, _p(w), _p(s), oc, ic, _p(out), _stream(w))
    return out


def linear(fmt, wq: torch.Tensor, scales, x: torch.Tensor, oc: int, ic: int, bias=None, out_dtype=None,
           out: torch.Tensor | None = None, tiled: bool = False, tcgen05: bool = False,
           prefetch: torch.Tensor | None = None, silu: bool = False) -> torch.Tensor:
    """y[..., oc] = x[..., ic] . decode(W)^T (+ bias) with W packed in `fmt`
    (reference layout, or the tile_weights copy with tiled=True).  tcgen05=True
    runs the tensor-memory kernel (SPFP2 reference layout, bf16 x).  prefetch:
    a tensor (typically the next layer's weight) the decode GEMV pulls into L2
    while it runs.  silu: the weight holds gate/up rows in groups of 8 + 8
    (V3GateUpSiLU) and the result is SiLU(gate) * up, oc // 2 wide (decode
    GEMV paths)."""
    f = FORMATS[fmt] if isinstance(fmt, str) else int(fmt)
    if tcgen05:
        f |= PATH_TCGEN05
    if tiled:
        f |= LAYOUT_TILED
        scales = None
    if silu:
        f |= EPILOGUE_SILU
    if not x.is_cuda:
        raise RuntimeError("spark_b200.linear: x must be a CUDA tensor")
    lead = x.shape[:-1]
    if x.shape[-1] != ic:
        raise ValueError(f"x has {x.shape[-1]} features, the weight has {ic}")
    x2 = x.reshape(-1, ic)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    w = _bytes(wq)
    s = _bytes(scales) if scales is not None else None
    b = bias.contiguous() if bias is not None else None
    width = oc // 2 if silu else oc
    y = out if out is not None else torch.empty(M, width, dtype=out_dtype or x.dtype, device=x.device)
    nbytes = workspace_size(f & 0xff, M, oc, ic)
    ws = workspace(x.device, nbytes)
    if prefetch is None:
        call("spark_linear", f, _p(w), _p(s), _p(x2), _dt(x2), M, oc, ic, x2.stride(0), _p(b),
             _dt(b) if b is not None else DTYPE_F32, _p(y), _dt(y), y.stride(0), _p(ws), ws.numel(), _stream(x))
    else:
        call("spark_linear_prefetch", f, _p(w), _p(s), _p(x2), _dt(x2), M, oc, ic, x2.stride(0), _p(b),
             _dt(b) if b is not None else DTYPE_F32, _p(y), _dt(y), y.stride(0), _p(ws), ws.numel(),
             _p(prefetch), prefetch.numel() * prefetch.element_size(), _stream(x))
    return y.reshape(*lead, width)


class ChainOp:
    """One op of linear_chain: a dequant linear or SiLU(gate) * up.

    Linear: ChainOp("linear", fmt=, wq=, scales=, x=, y=, bias=, deps=[...]).
    SiLU:   ChainOp("silu_mul", x=gate, x2=up, y=out, deps=[gate op, up op]).
    deps: indices of earlier ops whose output this op reads."""

    def __init__(self, kind, x, y, fmt="spfp2", wq=None, scales=None, x2=None, bias=None, deps=()):
        self.kind, self.fmt, self.wq, self.scales, self.x, self.x2, self.y = kind, fmt, wq, scales, x, x2, y
        self.bias, self.deps = bias, list(deps)


_chain_ws: dict[tuple[int, int], torch.Tensor] = {}


def linear_chain(chain: list[ChainOp], stream=None) -> None:
    """Run the ops in one persistent launch (spark_linear_chain).  Outputs are
    the caller's preallocated y tensors; every activation is bf16 [M, n]."""
    if not chain:
        return
    x0 = chain[0].x
    M = x0.shape[0]
    arr = (_lib.SparkChainOp * len(chain))()
    keep = []
    for k, op in enumerate(chain):
        c = arr[k]
        deps = op.deps + [-1] * (2 - len(op.deps))
        c.dep[0], c.dep[1] = deps[0], deps[1]
        c.x, c.y = op.x.data_ptr(), op.y.data_ptr()
        if op.kind == "silu_mul":
            c.kind, c.x2, c.ic = _lib.CHAIN_SILU_MUL, op.x2.data_ptr(), op.x.shape[1]
            continue
        f = FORMATS[op.fmt] if isinstance(op.fmt, str) else int(op.fmt)
        w = _bytes(op.wq)
        s = _bytes(op.scales) if op.scales is not None else None
        keep += [w, s]
        oc = op.y.shape[1]
        c.kind, c.fmt, c.wq, c.scales = _lib.CHAIN_LINEAR, f, w.data_ptr(), (s.data_ptr() if s is not None else None)
        c.ic, c.ldx, c.oc, c.ldy, c.y_dtype = op.x.shape[1], op.x.stride(0), oc, op.y.stride(0), _dt(op.y)
        if op.bias is not None:
            c.bias, c.bias_dtype = op.bias.data_ptr(), _dt(op.bias)
    n = int(_lib.lib().spark_linear_chain_workspace_size(len(chain)))
    st = stream if stream is not None else torch.cuda.current_stream(x0.device)
    key = (x0.device.index, st.cuda_stream)
    ws = _chain_ws.get(key)
    if ws is None or ws.numel() < n:
        ws = torch.zeros(n, dtype=torch.uint8, device=x0.device)
        _chain_ws[key] = ws
    call("spark_linear_chain", ctypes.cast(arr, ctypes.c_void_p), len(chain), M, _p(ws), ws.numel(),
         ctypes.c_void_p(st.cuda_stream))


class BatchOp:
    """One linear of linear_batch: y = x . decode(W)^T (+ bias) on tiled weights
    (tile_weights), bf16 x [M, ic]; silu: the weight holds gate/up rows in
    groups of 8 + 8 and y = SiLU(gate) * up, oc // 2 wide.  deps: indices of
    earlier ops of the batch whose output this op reads."""

    def __init__(self, fmt, wq_tiled: torch.Tensor, x: torch.Tensor, y: torch.Tensor, bias=None,
                 silu: bool = False, deps=()):
        self.fmt, self.wq, self.x, self.y, self.bias, self.silu, self.deps = fmt, wq_tiled, x, y, bias, silu, list(deps)


def _batch_array(batch: list[BatchOp]):
    arr = (_lib.SparkChainOp * len(batch))()
    for k, op in enumerate(batch):
        c = arr[k]
        if op.x.dtype != torch.bfloat16:
            raise TypeError("linear_batch: activations must be bfloat16")
        if op.x.dim() != 2 or op.x.stride(1) != 1 or op.y.dim() != 2 or op.y.stride(1) != 1:
            raise ValueError("linear_batch: x and y must be 2-D with unit column stride")
        deps = op.deps + [-1] * (2 - len(op.deps))
        if len(deps) > 2:
            raise ValueError("linear_batch: at most two deps per op")
        f = FORMATS[op.fmt] if isinstance(op.fmt, str) else int(op.fmt)
        c.kind, c.fmt = _lib.CHAIN_LINEAR, f | LAYOUT_TILED | (EPILOGUE_SILU if op.silu else 0)
        c.wq, c.scales = _bytes(op.wq).data_ptr(), None
        c.x, c.ic, c.ldx = op.x.data_ptr(), op.x.shape[1], op.x.stride(0)
        c.oc = op.y.shape[1] * (2 if op.silu else 1)
        c.y, c.y_dtype, c.ldy = op.y.data_ptr(), _dt(op.y), op.y.stride(0)
        if op.bias is not None:
            c.bias, c.bias_dtype = op.bias.data_ptr(), _dt(op.bias)
        c.dep[0], c.dep[1] = deps[0], deps[1]
    return arr


def linear_batch(batch: list[BatchOp], stream=None) -> None:
    """Run the linears in one persistent launch (spark_linear_batch).  Every op
    shares the token count M (rows of x); outputs are the ops' preallocated y."""
    if not batch:
        return
    x0 = batch[0].x
    M = x0.shape[0]
    arr = _batch_array(batch)
    st = stream if stream is not None else torch.cuda.current_stream(x0.device)
    n = int(_lib.lib().spark_linear_batch_workspace_size(ctypes.cast(arr, ctypes.c_void_p), len(batch), M))
    if n == 0:
        # an invalid batch: let the call itself report why
        n = 1 << 20
    ws = workspace(x0.device, n, stream=st)
    call("spark_linear_batch", ctypes.cast(arr, ctypes.c_void_p), len(batch), M, _p(ws), ws.numel(),
         ctypes.c_void_p(st.cuda_stream))


def linear_batch_allreduce(batch: list[BatchOp], op: int, world: int, rank: int, recv_ptrs, counter: torch.Tensor,
                           stream=None) -> None:
    """linear_batch whose op `op` is all-reduced over `world` ranks inside the
    same launch (spark_linear_batch_ar): every rank runs the same batch on its
    own shard (e.g. the K-sharded down projection of a tensor-parallel MLP)
    and gets the rank-order sum of the ranks' fp32 results (+ bias) in that
    op's y.  recv_ptrs: device addresses of every rank's receive buffer, as
    this process maps them; counter: this rank's call counter (one int32).
    tp.BatchAllReduce shares and owns both."""
    if not batch:
        raise ValueError("linear_batch_allreduce: empty batch")
    x0 = batch[0].x
    M = x0.shape[0]
    arr = _batch_array(batch)
    recv = (ctypes.c_void_p * world)(*recv_ptrs)
    ar = _lib.SparkBatchAllReduce(op, world, rank, ctypes.cast(recv, ctypes.c_void_p), counter.data_ptr())
    st = stream if stream is not None else torch.cuda.current_stream(x0.device)
    n = int(_lib.lib().spark_linear_batch_ar_workspace_size(ctypes.cast(arr, ctypes.c_void_p), len(batch), M,
                                                             ctypes.byref(ar)))
    ws = workspace(x0.device, n if n else 1 << 20, stream=st)
    call("spark_linear_batch_ar", ctypes.cast(arr, ctypes.c_void_p), len(batch), M, ctypes.byref(ar), _p(ws),
         ws.numel(), ctypes.c_void_p(st.cuda_stream))


def check_device_errors(device=None) -> None:
    """Raise if a kernel left an error in a workspace (synchronises)."""
    for (dev, sh), buf in list(_ws.items()) + list(_chain_ws.items()):
        if device is not None and dev != device:
            continue
        call("spark_workspace_check", _p(buf), ctypes.c_void_p(sh))


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """SiLU(gate) * up.  2-D views with unit column stride and a common row
    stride (the two halves of a row-merged gate|up output) are read in place."""
    if gate.shape != up.shape:
        raise ValueError("silu_mul: gate and up shapes differ")
    if (gate.dim() == 2 and gate.stride(1) == 1 and up.stride(1) == 1 and gate.stride(0) == up.stride(0)
            and gate.dtype == up.dtype):
        rows, cols = gate.shape
        out = torch.empty(rows, cols, dtype=gate.dtype, device=gate.device)
        call("spark_silu_mul_rows", _p(gate), _p(up), gate.stride(0), _p(out), cols, _dt(gate), rows, cols,
             _stream(gate))
        return out
    g, u = gate.contiguous(), up.contiguous()
    out = torch.empty_like(g)
    call("spark_silu_mul", _p(g), _p(u), _p(out), _dt(g), g.numel(), _stream(g))
    return out
