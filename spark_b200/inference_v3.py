"""Packed-weight-resident inference layers (mirror of 04_scripts/inference_v3.py).

The reference's ``V3SPFP2Layer`` (inference_v3.py:33-57) keeps the SPFP2 bytes
on the GPU and calls a JIT-built kernel on fp16 activations; its kernel reads
the 3-byte block layout although containers hold the paired 5-byte layout
(quant_linear.py:258-271 -> block_fp2_emu.py:231-267).  Here the layer reads
the container's paired bytes, takes bf16/fp16/fp32 activations, returns
x.dtype, and dispatches to the sm_100a decode GEMV / GEMM.  ``V3PackedLinear``
extends the same idea to the FP3, NVFP4 and 2:4 tiers.
"""
from __future__ import annotations

import torch
from torch import nn

from . import ops

_FMT_KEYS = {
    "spfp2": ("_packed", None),
    "fp3": ("_fp3_codes", "_fp3_scales"),
    "nvfp4": ("_nvfp4_codes", "_nvfp4_scales"),
    "twofour": ("_packed", None),
}


def fp3_nibbles_to_3bit(codes: torch.Tensor, n: int) -> torch.Tensor:
    """FP3 nibble codes (fp3_emu.fp3_pack, element 2j in the low nibble) to the
    3-bit layout (fp3_emu.fp3_pack_3bit: 8 codes in 3 bytes, code i at bit 3i),
    once at load time."""
    c = codes.view(torch.uint8).to(torch.int32)
    flat = torch.stack([c & 7, (c >> 4) & 7], dim=1).reshape(-1)[:n]
    if n % 8:
        flat = torch.nn.functional.pad(flat, (0, 8 - n % 8))
    g = flat.view(-1, 8)
    word = (g << torch.arange(0, 24, 3, device=g.device, dtype=torch.int32)).sum(dim=1)
    return torch.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], dim=1).reshape(-1).to(torch.uint8)


class V3PackedLinear(nn.Module):
    """y = x . decode(W)^T + bias with W kept packed in HBM.

    fmt: "spfp2" (paired 5 B / 16 w), "spfp2_v1" (3 B / 8 w), "fp3" (3-bit codes +
    e4m3 scales), "nvfp4" (e2m1 nibbles + e4m3 scales) or "twofour" (7 B / 32 w).
    prefetch_next: a tensor (the next layer's weight, see chain_prefetch) the
    decode GEMV pulls into L2 while it runs.
    """

    prefetch_next: torch.Tensor | None = None

    def __init__(self, fmt: str, packed: torch.Tensor, out_features: int, in_features: int,
                 scales: torch.Tensor | None = None, bias: torch.Tensor | None = None):
        super().__init__()
        if fmt not in ops.FORMATS:
            raise ValueError(f"unknown format {fmt!r}")
        self.fmt = fmt
        self.out_features = out_features
        self.in_features = in_features
        self.register_buffer("w_packed", packed)
        self.register_buffer("w_scales", scales.view(torch.uint8) if scales is not None else None)
        self.register_buffer("bias", bias)
        # fragment-major copy for the decode GEMV when the shape allows it; the
        # reference-layout bytes are kept for export and for the other paths
        # (2:4 always runs the tcgen05 kernel on the reference layout)
        self.register_buffer("w_tiled", ops.tile_weights(fmt, packed, scales, out_features, in_features)
                             if packed.is_cuda and fmt in ("spfp2", "fp3", "nvfp4") else None,
                             persistent=False)

    @classmethod
    def from_packed(cls, fmt, packed, scales, out_features, in_features, bias=None):
        return cls(fmt, packed, out_features, in_features, scales=scales, bias=bias)

    @classmethod
    def from_state(cls, state: dict, name: str, fmt: str, device="cuda"):
        """Build from a SPARK state dict entry (<name>_packed / _fp3_codes / ... + _meta)."""
        codes_key, scales_key = _FMT_KEYS[fmt]
        oc, ic = (int(v) for v in state[name + "_meta"][:2])
        packed = state[name + codes_key].to(device)
        scales = state[name + scales_key].to(device) if scales_key else None
        n = oc * ((ic + 15) // 16) * 16
        if fmt == "fp3" and packed.numel() == (n + 1) // 2:
            packed = fp3_nibbles_to_3bit(packed, n)
        b = state.get(f"param::{name}.bias")
        return cls(fmt, packed, oc, ic, scales=scales, bias=b.to(device) if b is not None else None)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """out: optional preallocated [M, out_features] result (its dtype is the
        output dtype; x.dtype otherwise)."""
        ic = self.in_features
        if self.fmt in ("spfp2", "spfp2_v1") and ic % 8:
            # the layer classes pack rows padded to whole 8-blocks (quant_linear.py:183-192)
            pad = (ic + 7) // 8 * 8
            x = torch.nn.functional.pad(x, (0, pad - ic))
            ic = pad
        # up to 16 tokens: the decode GEMV on the tiled copy; more: the tcgen05
        # GEMM, which reads the reference-layout bytes
        if self.tiled_ok(x) and ic == self.in_features:
            return ops.linear(self.fmt, self.w_tiled, None, x, self.out_features, ic, bias=self.bias,
                              out_dtype=x.dtype, out=out, tiled=True, prefetch=self.prefetch_next)
        return ops.linear(self.fmt, self.w_packed, self.w_scales, x, self.out_features, ic,
                          bias=self.bias, out_dtype=x.dtype, out=out)

    def tiled_ok(self, x: torch.Tensor) -> bool:
        """True when x (up to 16 tokens) can run on the tiled copy: any
        activation dtype for FP3 / NVFP4; bf16 rows on 16 bytes for SPFP2,
        whose tiled layout feeds the fp8 / bf16 tensor path of the batched
        decode kernel.  Other activations read the reference-layout bytes."""
        if self.w_tiled is None or x.shape[-1] != self.in_features or x.numel() > 16 * self.in_features:
            return False
        if self.fmt != "spfp2":
            return True
        return (x.dtype == torch.bfloat16 and x.stride(-1) == 1 and x.data_ptr() % 16 == 0
                and (x.dim() == 1 or x.reshape(-1, x.shape[-1]).stride(0) % 8 == 0))

    def extra_repr(self) -> str:
        return f"fmt={self.fmt}, in_features={self.in_features}, out_features={self.out_features}"


def _row_aligned(fmt: str, ic: int) -> bool:
    """True when every output row of a packed weight is a whole number of bytes,
    so row-concatenating packed buffers equals packing the stacked matrix."""
    if fmt == "spfp2":
        return ic % 16 == 0          # 5-byte block pairs never straddle rows
    if fmt == "twofour":
        return ic % 32 == 0          # 7-byte pairs of 16-blocks
    return fmt in ("fp3", "nvfp4")   # rows padded to whole 16-blocks


class V3MergedLinear(nn.Module):
    """Projections that read the same input (q/k/v, gate/up) kept as ONE
    packed weight, their rows stacked in order: one launch streams all of
    them.  forward(x) returns one output per part, views of the stacked
    [..., sum(out_features)] result; each equals the part's own layer output
    up to fp32 summation order."""

    def __init__(self, parts: list[V3PackedLinear]):
        super().__init__()
        if not parts:
            raise ValueError("V3MergedLinear needs at least one part")
        fmt, ic = parts[0].fmt, parts[0].in_features
        for p in parts:
            if p.fmt != fmt or p.in_features != ic:
                raise ValueError("merged parts must share the format and in_features")
        if not _row_aligned(fmt, ic):
            raise ValueError(f"{fmt} rows of {ic} weights are not byte-aligned; cannot merge")
        self.splits = [p.out_features for p in parts]
        packed = torch.cat([p.w_packed.reshape(-1) for p in parts])
        scales = None
        if parts[0].w_scales is not None:
            scales = torch.cat([p.w_scales.reshape(-1) for p in parts])
        bias = None
        if any(p.bias is not None for p in parts):
            ref = next(p.bias for p in parts if p.bias is not None)
            bias = torch.cat([p.bias if p.bias is not None else
                              torch.zeros(p.out_features, dtype=ref.dtype, device=ref.device) for p in parts])
        self.merged = V3PackedLinear(fmt, packed, sum(self.splits), ic, scales=scales, bias=bias)

    @property
    def in_features(self) -> int:
        return self.merged.in_features

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> tuple[torch.Tensor, ...]:
        """out: optional preallocated [M, sum(out_features)] result."""
        return self.merged(x, out=out).split(self.splits, dim=-1)

    def extra_repr(self) -> str:
        return f"fmt={self.merged.fmt}, in_features={self.in_features}, splits={self.splits}"


class V3GateUpSiLU(nn.Module):
    """SiLU(gate(x)) * up(x) of an MLP as one launch: gate and up are kept as
    one packed weight whose rows come in 16-row groups -- 8 gate rows, then the
    same 8 up rows -- so each thread of the decode GEMV holds a gate value and
    its up value and writes SiLU(gate) * up straight from the accumulators (no
    [M, 2I] intermediate, no separate SiLU launch).  Above 16 tokens the stacked
    linear runs on the tcgen05 GEMM and spark_silu_mul pairs the halves."""

    def __init__(self, gate: V3PackedLinear, up: V3PackedLinear):
        super().__init__()
        if (gate.fmt != up.fmt or gate.in_features != up.in_features or gate.out_features != up.out_features
                or gate.out_features % 8):
            raise ValueError("V3GateUpSiLU: gate and up must share format and shape, out_features % 8 == 0")
        fmt, ic, inter = gate.fmt, gate.in_features, gate.out_features
        if not _row_aligned(fmt, ic):
            raise ValueError(f"{fmt} rows of {ic} weights are not byte-aligned; cannot interleave")
        self.out_features = inter
        # row order: gate 8k..8k+7, up 8k..8k+7 for every k
        k = torch.arange(inter // 8, device=gate.w_packed.device)
        order = torch.stack([k * 8, k * 8 + inter], dim=1).repeat_interleave(8, dim=1)
        order = (order + torch.arange(8, device=order.device).repeat(2)).reshape(-1)

        def interleave(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
            both = torch.cat([a.reshape(inter, -1), b.reshape(inter, -1)])
            return both[order].reshape(-1)

        scales = interleave(gate.w_scales, up.w_scales) if gate.w_scales is not None else None
        bias = None
        if gate.bias is not None or up.bias is not None:
            ref = gate.bias if gate.bias is not None else up.bias
            zero = torch.zeros(inter, dtype=ref.dtype, device=ref.device)
            bias = interleave(gate.bias if gate.bias is not None else zero, up.bias if up.bias is not None else zero)
        self.merged = V3PackedLinear(fmt, interleave(gate.w_packed, up.w_packed), 2 * inter, ic, scales=scales,
                                     bias=bias)

    @property
    def in_features(self) -> int:
        return self.merged.in_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        m = self.merged
        if m.tiled_ok(x):
            return ops.linear(m.fmt, m.w_tiled, None, x, m.out_features, m.in_features, bias=m.bias,
                              out_dtype=x.dtype, tiled=True, prefetch=m.prefetch_next, silu=True)
        y = m(x).reshape(-1, self.out_features // 8, 2, 8)
        h = ops.silu_mul(y[:, :, 0, :].reshape(-1, self.out_features), y[:, :, 1, :].reshape(-1, self.out_features))
        return h.reshape(*x.shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"fmt={self.merged.fmt}, in_features={self.in_features}, out_features={self.out_features}, silu"


class V3LinearBatch:
    """The forwards of several packed layers (V3PackedLinear, V3MergedLinear,
    V3GateUpSiLU) in ONE launch of the batched decode kernel
    (spark_linear_batch): a decode step's projections stream their weights
    back to back instead of paying a kernel ramp and tail each.

    deps[i]: indices of earlier layers whose OUTPUT layer i reads as its input
    (at most two); the kernel then waits for them on the device.  Calls take
    bf16 activations, one [M, in_features] tensor per layer (M <= 16, the
    same M for all), and return one [M, width] tensor per layer: the stacked
    output of a V3MergedLinear (split it with .split(layer.splits, -1)),
    SiLU(gate) * up for a V3GateUpSiLU.  Layers must hold tiled weights."""

    def __init__(self, layers: list, deps: list | None = None):
        self.layers = list(layers)
        self.deps = [list(d) for d in deps] if deps is not None else [[] for _ in self.layers]
        if len(self.deps) != len(self.layers):
            raise ValueError("V3LinearBatch: one deps entry per layer")
        self._spec = []
        for m in self.layers:
            silu = isinstance(m, V3GateUpSiLU)
            lin = m.merged if isinstance(m, (V3MergedLinear, V3GateUpSiLU)) else m
            if lin.w_tiled is None:
                raise ValueError(f"V3LinearBatch: {lin.fmt} [{lin.out_features}, {lin.in_features}] has no tiled copy")
            width = lin.out_features // 2 if silu else lin.out_features
            self._spec.append((lin, silu, width))

    def __call__(self, inputs: list, outs: list | None = None) -> list:
        if len(inputs) != len(self.layers):
            raise ValueError("V3LinearBatch: one input per layer")
        if outs is None:
            outs = [torch.empty(x.shape[0], w, dtype=x.dtype, device=x.device)
                    for x, (_, _, w) in zip(inputs, self._spec)]
        batch = [ops.BatchOp(lin.fmt, lin.w_tiled, x, y, bias=lin.bias, silu=silu, deps=d)
                 for (lin, silu, _), x, y, d in zip(self._spec, inputs, outs, self.deps)]
        ops.linear_batch(batch)
        return outs


def chain_prefetch(modules: list) -> None:
    """Layers in call order (V3PackedLinear or V3MergedLinear): each one's decode
    GEMV pulls the next one's weight into L2 while it runs, the last one the
    first's (a decode loop starts over).  Only a hint: results do not change."""
    lin = [m.merged if isinstance(m, (V3MergedLinear, V3GateUpSiLU)) else m for m in modules]
    for i, m in enumerate(lin):
        nxt = lin[(i + 1) % len(lin)]
        m.prefetch_next = nxt.w_tiled if nxt.w_tiled is not None else nxt.w_packed


class V3SPFP2Layer(V3PackedLinear):
    """Drop-in for inference_v3.V3SPFP2Layer(packed_weight, out_features, in_features, bias)."""

    def __init__(self, packed_weight, out_features, in_features, bias=None):
        if bias is not None and bias.numel() == 0:
            bias = None
        super().__init__("spfp2", packed_weight, out_features, in_features, bias=bias)


class V3NVFP4Embedding(nn.Module):
    """Packed-resident NVFP4 embedding table: the inference form of
    quant_linear.NVFP4EmbeddingQAT (quant_linear.py:507-537), whose forward is
    F.embedding of the NVFP4-quantised table.  Codes [rows, pad16(dim)/2] and
    e4m3 scales [rows, pad16(dim)/16] stay on the GPU; a lookup decodes only
    the rows it reads.  padding_idx only affects gradients, as in
    F.embedding, so the forward ignores it."""

    def __init__(self, codes: torch.Tensor, scales: torch.Tensor, num_embeddings: int, embedding_dim: int,
                 padding_idx=None, dtype=torch.bfloat16):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.padding_idx = padding_idx
        self.dtype = dtype
        self.register_buffer("codes", codes.view(torch.uint8))
        self.register_buffer("scales", scales.view(torch.uint8))

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return ops.nvfp4_embedding(self.codes, self.scales, self.num_embeddings, self.embedding_dim, input_ids,
                                   dtype=self.dtype)

    def extra_repr(self) -> str:
        return f"{self.num_embeddings}, {self.embedding_dim}, nvfp4"


def build_v3_layers(model: nn.Module, state: dict, device="cuda") -> int:
    """Replace every nn.Linear that has packed weights in `state` by a packed-
    resident layer (the reference's build_v3_model, inference_v3.py:60-105,
    extended from MLP SPFP2 to every tier), and every nn.Embedding with NVFP4
    codes by a V3NVFP4Embedding.  Returns the number replaced."""
    n = 0
    for name, module in list(model.named_modules()):
        if isinstance(module, nn.Embedding) and name + "_nvfp4_codes" in state and name + "_meta" in state:
            rows, dim = (int(v) for v in state[name + "_meta"][:2])
            emb = V3NVFP4Embedding(state[name + "_nvfp4_codes"].to(device), state[name + "_nvfp4_scales"].to(device),
                                   rows, dim, padding_idx=module.padding_idx, dtype=module.weight.dtype)
            parent = model.get_submodule(".".join(name.split(".")[:-1])) if "." in name else model
            setattr(parent, name.split(".")[-1], emb)
            n += 1
            continue
        if not isinstance(module, nn.Linear):
            continue
        fmt = None
        if name + "_fp3_codes" in state:
            fmt = "fp3"
        elif name + "_nvfp4_codes" in state:
            fmt = "nvfp4"
        elif name + "_packed" in state:
            meta = state.get(name + "_meta")
            if meta is None:
                continue
            oc, ic = int(meta[0]), int(meta[1])
            nb = oc * ((ic + 7) // 8)
            fmt = "spfp2" if state[name + "_packed"].numel() == (nb + 1) // 2 * 5 else "spfp2_v1"
        if fmt is None or name + "_meta" not in state:
            continue
        layer = V3PackedLinear.from_state(state, name, fmt, device=device)
        parent = model.get_submodule(".".join(name.split(".")[:-1])) if "." in name else model
        setattr(parent, name.split(".")[-1], layer)
        n += 1
    return n
