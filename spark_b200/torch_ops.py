"""torch.library ops with the call shapes of the reference's CUDA extensions,
so code that calls those ops through torch keeps working on this library.

  torch.ops.spark.decode_fp32(packed, rows) -> Tensor      (01_core/build_spark_fp2.py:28-54)
  torch.ops.spark.decode_fp16(packed, rows) -> Tensor
  torch.ops.spark.spark_v3_spfp2_forward(w, x, y, bias, oc, ic)    (01_core/spark_v3_kernel.cu:195-214)
  torch.ops.spark.spark_v3_twofour_forward(w, x, y, bias, oc, ic)  (01_core/spark_v3_twofour.cu:162-181)

decode_* read the legacy single-exponent blocks (5 bytes per 16 weights) that
the reference's decode kernels read (01_core/block_fp2_kernel.cu:3-62).  The
forward ops write y in place (y preallocated by the caller, as in
04_scripts/inference_v3.py:52-56); an empty bias tensor means no bias.  The
weight layouts are the ones those kernels index: per output row, 3-byte 8-weight
blocks (SPFP2 "v1") or 7-byte pairs of 16-weight blocks (2:4).  Unlike the
reference forwards, every op validates its arguments and raises on a bad call
or a failed launch; the activations may be fp16 (the reference's type), bf16
or fp32, and y fp16, bf16 or fp32.
"""
from __future__ import annotations

import torch

from . import _lib, ops

__all__ = ["decode_fp32", "decode_fp16", "spark_v3_spfp2_forward", "spark_v3_twofour_forward"]


def _check_packed(packed: torch.Tensor, what: str) -> None:
    if not packed.is_cuda:
        raise RuntimeError(f"{what}: packed must be a CUDA tensor")
    if packed.dtype != torch.uint8:
        raise RuntimeError(f"{what}: expected uint8 bytes, got {packed.dtype}")
    if not packed.is_contiguous():
        raise RuntimeError(f"{what}: packed must be contiguous")


def _legacy_decode(packed: torch.Tensor, rows: int, dtype: torch.dtype, what: str) -> torch.Tensor:
    _check_packed(packed, what)
    nb = packed.numel() // 5
    if nb * 16 != rows:
        raise RuntimeError(f"{what}: decode size mismatch ({packed.numel()} bytes hold {nb * 16} values, "
                           f"rows = {rows})")
    out = torch.empty(rows, dtype=dtype, device=packed.device)
    _lib.call("spark_spfp2_legacy_decode", ops._p(packed), nb, ops._p(out), ops._DT[dtype], ops._stream(packed))
    return out


@torch.library.custom_op("spark::decode_fp32", mutates_args=())
def decode_fp32(packed: torch.Tensor, rows: int) -> torch.Tensor:
    return _legacy_decode(packed, rows, torch.float32, "spark::decode_fp32")


@decode_fp32.register_fake
def _decode_fp32_fake(packed, rows):
    return packed.new_empty(rows, dtype=torch.float32)


@torch.library.custom_op("spark::decode_fp16", mutates_args=())
def decode_fp16(packed: torch.Tensor, rows: int) -> torch.Tensor:
    return _legacy_decode(packed, rows, torch.float16, "spark::decode_fp16")


@decode_fp16.register_fake
def _decode_fp16_fake(packed, rows):
    return packed.new_empty(rows, dtype=torch.float16)


def _forward(fmt: str, pad: int, row_bytes, w: torch.Tensor, x: torch.Tensor, y: torch.Tensor,
             bias: torch.Tensor, oc: int, ic: int, what: str) -> None:
    _check_packed(w, what)
    if oc <= 0 or ic <= 0:
        raise RuntimeError(f"{what}: oc and ic must be positive")
    if not (x.is_cuda and y.is_cuda):
        raise RuntimeError(f"{what}: x and y must be CUDA tensors")
    if x.dim() != 2 or x.shape[1] != ic:
        raise RuntimeError(f"{what}: x must be [M, {ic}], got {list(x.shape)}")
    if y.dim() != 2 or y.shape[0] != x.shape[0] or y.shape[1] != oc or not y.is_contiguous():
        raise RuntimeError(f"{what}: y must be a contiguous [{x.shape[0]}, {oc}] tensor")
    if x.dtype not in ops._DT or y.dtype not in ops._DT:
        raise RuntimeError(f"{what}: x and y must be float16, bfloat16 or float32")
    icp = (ic + pad - 1) // pad * pad
    need = oc * row_bytes(icp)
    if w.numel() < need:
        raise RuntimeError(f"{what}: {w.numel()} weight bytes, [{oc}, {ic}] needs {need}")
    b = None
    if bias.numel() > 0:
        if bias.numel() != oc or not bias.is_cuda:
            raise RuntimeError(f"{what}: bias must be empty or a CUDA tensor of {oc} values")
        b = bias.contiguous()
    xin = x if icp == ic else torch.nn.functional.pad(x, (0, icp - ic))
    # rows padded to whole blocks (the reference kernels index rows of
    # ceil(ic / block) blocks); the padded columns meet zero activations
    ops.linear(fmt, w, None, xin.contiguous(), oc, icp, bias=b, out=y)


@torch.library.custom_op("spark::spark_v3_spfp2_forward", mutates_args=("y",))
def spark_v3_spfp2_forward(w_packed: torch.Tensor, x: torch.Tensor, y: torch.Tensor, bias: torch.Tensor, oc: int,
                           ic: int) -> None:
    _forward("spfp2_v1", 8, lambda n: n // 8 * 3, w_packed, x, y, bias, oc, ic, "spark::spark_v3_spfp2_forward")


@torch.library.custom_op("spark::spark_v3_twofour_forward", mutates_args=("y",))
def spark_v3_twofour_forward(w_packed: torch.Tensor, x: torch.Tensor, y: torch.Tensor, bias: torch.Tensor, oc: int,
                             ic: int) -> None:
    _forward("twofour", 32, lambda n: n // 32 * 7, w_packed, x, y, bias, oc, ic,
             "spark::spark_v3_twofour_forward")
