"""GPU stand-in for 01_core/block_fp2_emu.py (SPFP2): the same names,
arguments and results, computed by the sm_100a kernels.  CPU tensors are moved
to the current CUDA device and results come back on the caller's device.

Bit-exact with the reference emulator (pinned by tests/golden).  The legacy
search-free ``pack_blockwise`` / ``decode`` / ``BlockFP2STE`` path (no layer
of the reference uses it) is not provided.
"""
from __future__ import annotations

import torch

from . import ops

ELEMS_PER_BLOCK = 8          # block_fp2_emu.py:20
BYTES_PER_BLOCK = 3          # :23, 3-byte block layout
BYTES_PER_PAIR = 5           # :31, paired layout (16 weights in 5 bytes)
BIAS = 10                    # scale = 2 ** (e - BIAS)
DEFAULT_CANDIDATES = tuple(range(16))


def _check_window(window):
    if window != 2:
        raise NotImplementedError("spark_b200 implements the reference's window=2 exponent search only")


def pack_blockwise_search(w: torch.Tensor, candidates=DEFAULT_CANDIDATES, window: int = 2):
    """block_fp2_emu.py:86: 3 bytes per 8-weight block -> (packed uint8, expv uint8)."""
    _check_window(window)
    return ops.spfp2_pack_v1(w.detach().reshape(-1))


def pack_blockwise_paired(w: torch.Tensor, window: int = 2):
    """block_fp2_emu.py:231: two blocks in 5 bytes -> (packed uint8, expv uint8)."""
    _check_window(window)
    return ops.spfp2_pack(w.detach().reshape(-1))


def unpack_blockwise(packed: torch.Tensor, n_elements: int, dtype=torch.float32) -> torch.Tensor:
    """block_fp2_emu.py:204: every block of the buffer, like the reference
    (n_elements is accepted for the same call shape)."""
    return ops.spfp2_unpack_v1(packed, dtype=dtype)


def unpack_blockwise_paired(packed: torch.Tensor, n_elements: int, dtype=torch.float32) -> torch.Tensor:
    """block_fp2_emu.py:270."""
    return ops.spfp2_unpack(packed, n_elements, dtype=dtype)


class ChannelFP2STE(torch.autograd.Function):
    """block_fp2_emu.py:334-362: forward = the SPFP2 round trip of the weight
    (window search, 8-blocks over the flattened tensor), backward = identity."""

    @staticmethod
    def forward(ctx, x: torch.Tensor) -> torch.Tensor:
        return ops.spfp2_fake_quant(x, out_dtype=x.dtype)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        return grad_output.clone()


def channel_fake_quantize(x: torch.Tensor) -> torch.Tensor:
    """block_fp2_emu.py:365: differentiable when x requires grad (x.dtype out);
    otherwise the plain round trip in fp32, as the reference returns."""
    if x.requires_grad:
        return ChannelFP2STE.apply(x)
    return ops.spfp2_fake_quant(x, out_dtype=torch.float32)
