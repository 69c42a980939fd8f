"""GPU stand-in for 01_core/fp3_emu.py (FP3 E1M1: 3-bit codes
+-{0, .5, 1, 1.5} with an e4m3 scale per 16 weights): same names, arguments
and results, computed by the sm_100a kernels."""
from __future__ import annotations

import torch

from . import ops

ELEMS_PER_BLOCK = 16         # fp3_emu.py:19


def fp3_fake_quant(w: torch.Tensor) -> torch.Tensor:
    """fp3_emu.py:24: (oc, ic) round trip, fp32."""
    return ops.fp3_fake_quant(w, out_dtype=torch.float32)


def fp3_pack(w: torch.Tensor):
    """fp3_emu.py:50: nibble codes (4 bits per weight) + e4m3 scales."""
    return ops.fp3_pack(w, nibble=True)


def fp3_unpack(codes: torch.Tensor, scales: torch.Tensor, oc: int, ic: int) -> torch.Tensor:
    """fp3_emu.py:77."""
    return ops.fp3_unpack(codes, scales, oc, ic, nibble=True)


def fp3_pack_3bit(w: torch.Tensor):
    """fp3_emu.py:107: 8 codes in 3 bytes + e4m3 scales."""
    return ops.fp3_pack(w, nibble=False)


def fp3_unpack_3bit(packed: torch.Tensor, scales: torch.Tensor, oc: int, ic: int) -> torch.Tensor:
    """fp3_emu.py:142."""
    return ops.fp3_unpack(packed, scales, oc, ic, nibble=False)


class FP3STE(torch.autograd.Function):
    """fp3_emu.py:89-96: forward = fp3_fake_quant, backward = identity."""

    @staticmethod
    def forward(ctx, x):
        return fp3_fake_quant(x)

    @staticmethod
    def backward(ctx, grad_output):
        return grad_output.clone()


def fp3_fake_quant_ste(x: torch.Tensor) -> torch.Tensor:
    if x.requires_grad:
        return FP3STE.apply(x)
    return fp3_fake_quant(x)
