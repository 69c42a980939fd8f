"""Tensor-parallel MLP and layer-split packing over one node.

The path shards the way the model does (no collective is invented):
* gate_proj / up_proj are column-parallel: rank r keeps output rows
  [r*I/W, (r+1)*I/W) -- a contiguous byte range of the packed weight;
* down_proj is row-parallel: rank r keeps input columns [r*I/W, (r+1)*I/W),
  cut on 16-weight boundaries so SPFP2 block pairs never straddle it; each
  rank's partial [M, H] sums meet in one all-reduce (NCCL over NVLink on the
  GPUs, gloo in the CPU tests);
* whole-model pack / quantize is independent per layer: layers go to ranks
  round-robin and the packed bytes are gathered on the host.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

ALIGN = 16      # SPFP2 pairs, FP3 groups and 2:4 pairs of 16-blocks stay whole


def shard_bounds(n: int, rank: int, world: int, align: int = ALIGN) -> tuple[int, int]:
    """[lo, hi) of rank's share of n rows or columns, cut on `align` boundaries."""
    if n % (world * align):
        raise ValueError(f"{n} does not split into {world} shards of whole {align}-blocks")
    step = n // world
    return rank * step, (rank + 1) * step


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Column-parallel share (gate / up): output rows of rank."""
    lo, hi = shard_bounds(w.shape[0], rank, world)
    return w[lo:hi]


def shard_cols(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Row-parallel share (down): input columns of rank."""
    lo, hi = shard_bounds(w.shape[1], rank, world)
    return w[:, lo:hi]


class TPMLP(torch.nn.Module):
    """One SPFP2 MLP layer, tensor-parallel over the default process group:
    y = all_reduce( down_r( silu(gate_r x) * up_r x ) ).

    The shares are packed on this rank's GPU from the full fp32 weights (or
    given already packed via from_packed)."""

    def __init__(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, rank: int = 0, world: int = 1,
                 group=None):
        super().__init__()
        from .inference_v3 import V3MergedLinear, V3PackedLinear
        from . import ops
        self.world, self.group = world, group
        g, u, d = shard_rows(gate, rank, world), shard_rows(up, rank, world), shard_cols(down, rank, world)
        gate_l = V3PackedLinear("spfp2", ops.spfp2_pack(g.contiguous())[0], g.shape[0], g.shape[1])
        up_l = V3PackedLinear("spfp2", ops.spfp2_pack(u.contiguous())[0], u.shape[0], u.shape[1])
        # gate and up read the same x: one row-merged weight, one launch
        self.gate_up = V3MergedLinear([gate_l, up_l])
        self.down = V3PackedLinear("spfp2", ops.spfp2_pack(d.contiguous())[0], d.shape[0], d.shape[1])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from . import ops
        g, u = self.gate_up(x)
        y = self.down(ops.silu_mul(g, u))
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        return y


def pack_layers_split(weights: list[torch.Tensor], pack: Callable[[torch.Tensor], torch.Tensor], rank: int,
                      world: int, group=None) -> list[torch.Tensor]:
    """Pack layer l on rank l % world, then gather every layer's bytes to every
    rank (host memory).  `pack` maps a weight to its packed uint8 tensor."""
    mine = {l: pack(w).detach().cpu() for l, w in enumerate(weights) if l % world == rank}
    if world == 1:
        return [mine[l] for l in range(len(weights))]
    gathered: list = [None] * world
    dist.all_gather_object(gathered, mine, group=group)
    out = {}
    for part in gathered:
        out.update(part)
    return [out[l] for l in range(len(weights))]
