"""GPU stand-in for 01_core/nvfp4_emu.py (e2m1 codes with an e4m3 scale per
16 weights): same names, arguments and results, computed by the sm_100a
kernels."""
from __future__ import annotations

import torch

from . import ops

ELEMS_PER_BLOCK = 16         # nvfp4_emu.py:15
E2M1_MAX = 6.0


def nvfp4_fake_quant(w: torch.Tensor) -> torch.Tensor:
    """nvfp4_emu.py:37: (oc, ic) round trip, fp32."""
    return ops.nvfp4_fake_quant(w, out_dtype=torch.float32)


def nvfp4_pack(w: torch.Tensor):
    """nvfp4_emu.py:81: (codes uint8, two per byte, scales e4m3)."""
    return ops.nvfp4_pack(w)


def nvfp4_unpack(codes: torch.Tensor, scales: torch.Tensor, oc: int, ic: int) -> torch.Tensor:
    """nvfp4_emu.py:109."""
    return ops.nvfp4_unpack(codes, scales, oc, ic)


class NVFP4STE(torch.autograd.Function):
    """nvfp4_emu.py:60-69: forward = nvfp4_fake_quant, backward = identity."""

    @staticmethod
    def forward(ctx, x: torch.Tensor) -> torch.Tensor:
        return nvfp4_fake_quant(x)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        return grad_output.clone()


def nvfp4_fake_quant_ste(x: torch.Tensor) -> torch.Tensor:
    if x.requires_grad:
        return NVFP4STE.apply(x)
    return nvfp4_fake_quant(x)
