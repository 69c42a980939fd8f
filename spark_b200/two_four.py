"""GPU stand-in for 01_core/two_four.py (2:4-sparse SPFP2, 7 bytes per 32
weights): same names, arguments and results, computed by the sm_100a
kernels."""
from __future__ import annotations

import torch

from . import ops

BYTES_PER_PAIR = 7           # two_four.py:29


def two_four_pack(w: torch.Tensor) -> torch.Tensor:
    """two_four.py:112."""
    return ops.twofour_pack(w)


def two_four_unpack(packed: torch.Tensor, n_elements: int, dtype=torch.float32) -> torch.Tensor:
    """two_four.py:158."""
    return ops.twofour_unpack(packed, n_elements, dtype=dtype)


class TwoFourSTE(torch.autograd.Function):
    """two_four.py:57-67: forward = SPFP2 round trip then the 2:4 mask (first
    two nonzeros of every group of four), backward = identity."""

    @staticmethod
    def forward(ctx, x):
        return ops.twofour_fake_quant(x, out_dtype=x.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        return grad_output.clone()


def two_four_fake_quant(x: torch.Tensor) -> torch.Tensor:
    """two_four.py:70: x.dtype when differentiable, fp32 otherwise (as the reference)."""
    if x.requires_grad:
        return TwoFourSTE.apply(x)
    return ops.twofour_fake_quant(x, out_dtype=torch.float32)
