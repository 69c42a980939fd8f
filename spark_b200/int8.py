"""GPU stand-in for 01_core/int8_emu.py (per-output-channel symmetric INT8,
the lm_head tier): same names, arguments and results, computed by the
sm_100a kernels."""
from __future__ import annotations

import torch

from . import ops


def int8_fake_quant(w: torch.Tensor) -> torch.Tensor:
    """int8_emu.py:12: (oc, ic) round trip, fp32."""
    return ops.int8_fake_quant(w, out_dtype=torch.float32)


class INT8STE(torch.autograd.Function):
    """int8_emu.py:20-27: forward = int8_fake_quant, backward = identity."""

    @staticmethod
    def forward(ctx, x):
        return int8_fake_quant(x)

    @staticmethod
    def backward(ctx, grad_output):
        return grad_output.clone()


def int8_fake_quant_ste(x: torch.Tensor) -> torch.Tensor:
    if x.requires_grad:
        return INT8STE.apply(x)
    return int8_fake_quant(x)


def ptq_int8_pack(w: torch.Tensor):
    """int8_emu.py:37: (q int8 [oc, ic], scale fp32 [oc])."""
    return ops.int8_pack(w)


def ptq_int8_unpack(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """int8_emu.py:49."""
    return ops.int8_unpack(q, scale)
