"""Drop-in for 02_model/quant_linear.py: the SPFP2 / NVFP4 / 2:4 / INT8 layer
classes and the model-rewriting helpers, with the same names, arguments,
buffers (``_packed_weight``, ``_channel_scale_index`` / ``_scale_index``,
``_packed_format``) and training semantics.  Differences:

* packing, decoding and every fake-quant run on the sm_100a kernels;
* a quantized layer's CUDA forward does not decode the weight and call
  F.linear: it runs the dequant linear (decode GEMV for up to 16 tokens,
  tcgen05 GEMM above) on the packed bytes, returning x.dtype;
* one fake-quant cache version for every QAT layer, FP3 included.
On CPU the inference layers keep the reference's behaviour (F.linear on the
unquantized ``weight``, quant_linear.py:150-155).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from . import ops
from .block_fp2 import (BYTES_PER_BLOCK, BYTES_PER_PAIR, ELEMS_PER_BLOCK, channel_fake_quantize,
                        pack_blockwise_paired, unpack_blockwise, unpack_blockwise_paired)
from .fp3_linear import _WQ_VERSION, FP3QATLinear
from .int8 import int8_fake_quant
from .nvfp4 import nvfp4_fake_quant
from .two_four import two_four_fake_quant, two_four_pack

__all__ = [
    "quantize_tensor_blockwise", "FP2Linear", "ChannelFP2Linear", "ChannelFP2QATLinear", "NVFP4QATLinear",
    "TwoFourQATLinear", "INT8QATLinear", "NVFP4EmbeddingQAT", "FP3QATLinear", "apply_channel_fp2_qat",
    "apply_channel_fp2_quant", "apply_mixed_quant", "decode_layer_weight", "set_force_fake_quant",
    "bump_wq_version", "ELEMS_PER_BLOCK", "BYTES_PER_BLOCK", "BYTES_PER_PAIR",
]


def quantize_tensor_blockwise(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quant_linear.py:66: paired SPFP2 bytes and block exponents of w."""
    return pack_blockwise_paired(w.detach().contiguous().float())


def _detect_format(packed_numel: int, n_elements: int) -> str:
    """quant_linear.py:77: "v1" = 3-byte blocks, "v2" = 5-byte block pairs."""
    nb = (n_elements + ELEMS_PER_BLOCK - 1) // ELEMS_PER_BLOCK
    if packed_numel == nb * BYTES_PER_BLOCK:
        return "v1"
    if packed_numel == ((nb + 1) // 2) * BYTES_PER_PAIR:
        return "v2"
    raise ValueError(f"packed size {packed_numel} does not match n_elements {n_elements} "
                     f"(v1 expects {nb * BYTES_PER_BLOCK} B, v2 expects {((nb + 1) // 2) * BYTES_PER_PAIR} B)")


def _unpack_weight(packed: torch.Tensor, n_elements: int, device: str | torch.device = "cpu") -> torch.Tensor:
    """quant_linear.py:89: decode either layout to fp32 on `device`."""
    if _detect_format(packed.numel(), n_elements) == "v1":
        out = unpack_blockwise(packed, n_elements)[:n_elements]
    else:
        out = unpack_blockwise_paired(packed, n_elements)
    return out.to(device)


def _packed_linear(layer: nn.Module, x: torch.Tensor, rows_padded: bool) -> torch.Tensor:
    """y = x . decode(_packed_weight)^T + bias on the packed bytes.

    rows_padded: the layer packed each row padded to whole 8-blocks
    (ChannelFP2Linear); otherwise the weight was packed flattened, which is the
    same layout when ic is a multiple of 8."""
    oc, ic = layer.out_features, layer.in_features
    ic_p = (ic + ELEMS_PER_BLOCK - 1) // ELEMS_PER_BLOCK * ELEMS_PER_BLOCK
    packed = layer._packed_weight
    n_el = oc * (ic_p if rows_padded else ic)
    fmt = "spfp2_v1" if _detect_format(packed.numel(), n_el) == "v1" else "spfp2"
    if packed.device != x.device:
        packed = packed.to(x.device)
        layer._packed_weight = packed
    if ic_p != ic and not rows_padded:
        # blocks straddle rows: decode, then a plain GEMM
        w = _unpack_weight(packed, oc * ic, device=x.device).view(oc, ic).to(x.dtype)
        return nn.functional.linear(x, w, layer.bias)
    if ic_p != ic:
        x = nn.functional.pad(x, (0, ic_p - ic))
    return ops.linear(fmt, packed, None, x, oc, ic_p, bias=layer.bias, out_dtype=x.dtype)


class _LinearBase(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=dtype))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, device=device, dtype=dtype))
        else:
            self.register_parameter("bias", None)

    def _use_kernel_for(self, x: torch.Tensor) -> bool:
        return x.is_cuda


class FP2Linear(_LinearBase):
    """quant_linear.py:111-155: the whole weight packed as one flattened tensor."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device, dtype)
        self._packed_weight: Optional[torch.Tensor] = None
        self._scale_index: Optional[torch.Tensor] = None

    def quantize(self):
        self._packed_weight, self._scale_index = quantize_tensor_blockwise(self.weight.data.detach())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._packed_weight is not None and self._use_kernel_for(x):
            return _packed_linear(self, x, rows_padded=False)
        return nn.functional.linear(x, self.weight, self.bias)


class ChannelFP2Linear(_LinearBase):
    """quant_linear.py:158-219: rows padded to whole 8-blocks, then packed."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device, dtype)
        self._packed_weight: Optional[torch.Tensor] = None
        self._channel_scale_index: Optional[torch.Tensor] = None

    def quantize(self):
        self._packed_weight, self._channel_scale_index = _pack_rows(self.weight.data)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._packed_weight is not None and self._use_kernel_for(x):
            return _packed_linear(self, x, rows_padded=True)
        return nn.functional.linear(x, self.weight, self.bias)


def _pack_rows(w: torch.Tensor):
    """Paired SPFP2 of a (oc, ic) weight with each row zero-padded to whole
    8-blocks (quant_linear.py:173-195)."""
    w = w.detach().float()
    oc, ic = w.shape
    ic_p = (ic + ELEMS_PER_BLOCK - 1) // ELEMS_PER_BLOCK * ELEMS_PER_BLOCK
    if ic_p != ic:
        w = nn.functional.pad(w, (0, ic_p - ic))
    return pack_blockwise_paired(w)


def bump_wq_version():
    """quant_linear.py:228: after optimizer.step(): every QAT layer (FP3
    included) recomputes its fake-quant weight at its next forward."""
    _WQ_VERSION[0] += 1


class _QATBase(_LinearBase):
    force_fake_quant: bool = False
    _fake_quant = None       # set by subclasses: weight -> quantized weight

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device, dtype)
        self._wq_cache: Optional[torch.Tensor] = None
        self._wq_ver: int = -1

    def _effective_weight(self) -> torch.Tensor:
        """weight + (Wq - weight).detach(): forward value Wq, gradient straight
        through to weight (quant_linear.py:279-284); Wq cached per version."""
        if self._wq_cache is None or self._wq_ver != _WQ_VERSION[0]:
            with torch.no_grad():
                self._wq_cache = type(self)._fake_quant(self.weight.detach()).to(self.weight.dtype)
            self._wq_ver = _WQ_VERSION[0]
        return self.weight + (self._wq_cache - self.weight).detach()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.training or self.force_fake_quant:
            return nn.functional.linear(x, self._effective_weight(), self.bias)
        return nn.functional.linear(x, self.weight, self.bias)


class ChannelFP2QATLinear(_QATBase):
    """quant_linear.py:233-306: SPFP2 QAT; after quantize() the eval forward
    runs on the packed bytes like ChannelFP2Linear."""
    _fake_quant = staticmethod(channel_fake_quantize)

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device, dtype)
        self._packed_weight: Optional[torch.Tensor] = None
        self._channel_scale_index: Optional[torch.Tensor] = None

    def quantize(self):
        self._packed_weight, self._channel_scale_index = _pack_rows(self.weight.data)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.training or self.force_fake_quant:
            return nn.functional.linear(x, self._effective_weight(), self.bias)
        if self._packed_weight is not None and self._use_kernel_for(x):
            return _packed_linear(self, x, rows_padded=True)
        return nn.functional.linear(x, self.weight, self.bias)


class NVFP4QATLinear(_QATBase):
    """quant_linear.py:385-422."""
    _fake_quant = staticmethod(nvfp4_fake_quant)


class TwoFourQATLinear(_QATBase):
    """quant_linear.py:425-462: SPFP2 round trip then the 2:4 mask."""
    _fake_quant = staticmethod(two_four_fake_quant)

    def quantize(self):
        self._packed_weight = two_four_pack(self.weight.data.detach())
        self._packed_format = "v3-24"


class INT8QATLinear(_QATBase):
    """quant_linear.py:476-504: per-channel symmetric INT8."""
    _fake_quant = staticmethod(int8_fake_quant)


class NVFP4EmbeddingQAT(nn.Module):
    """quant_linear.py:507-537: NVFP4 fake-quant embedding table."""
    force_fake_quant: bool = False

    def __init__(self, num_embeddings: int, embedding_dim: int, padding_idx=None, device=None, dtype=None):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.padding_idx = padding_idx
        self.weight = nn.Parameter(torch.empty(num_embeddings, embedding_dim, device=device, dtype=dtype))
        self._wq_cache: Optional[torch.Tensor] = None
        self._wq_ver: int = -1

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        w = self.weight
        if self.training or self.force_fake_quant:
            if self._wq_cache is None or self._wq_ver != _WQ_VERSION[0]:
                with torch.no_grad():
                    self._wq_cache = nvfp4_fake_quant(w.detach()).to(self.weight.dtype)
                self._wq_ver = _WQ_VERSION[0]
            w = self.weight + (self._wq_cache - self.weight).detach()
        return nn.functional.embedding(input_ids, w, padding_idx=self.padding_idx)


def _replace(cls, old: nn.Module):
    q = cls(old.in_features, old.out_features, old.bias is not None, device=old.weight.device,
            dtype=old.weight.dtype)
    with torch.no_grad():
        q.weight.copy_(old.weight)
        if old.bias is not None:
            q.bias.copy_(old.bias)
    return q


def _skip_name(name: str) -> bool:
    return "lm_head" in name or "embed" in name.lower()


def apply_channel_fp2_qat(model: nn.Module) -> nn.Module:
    """quant_linear.py:309: every nn.Linear except lm_head / embeddings ->
    ChannelFP2QATLinear (weights and bias copied)."""
    for name, module in model.named_children():
        if isinstance(module, nn.Linear):
            if not _skip_name(name):
                setattr(model, name, _replace(ChannelFP2QATLinear, module))
        else:
            apply_channel_fp2_qat(module)
    return model


def apply_channel_fp2_quant(model: nn.Module) -> nn.Module:
    """quant_linear.py:352: the same replacement with ChannelFP2Linear."""
    for name, module in model.named_children():
        if isinstance(module, nn.Linear):
            if not _skip_name(name):
                setattr(model, name, _replace(ChannelFP2Linear, module))
        else:
            apply_channel_fp2_quant(module)
    return model


def decode_layer_weight(layer: nn.Module, device: str | torch.device = "cpu"):
    """quant_linear.py:333: the layer's packed weight decoded to fp32 (oc, ic),
    or a copy of its weight when it has not been quantized."""
    w = layer.weight.data.detach()
    packed = getattr(layer, "_packed_weight", None)
    if packed is None:
        return w.clone()
    oc, ic = w.shape
    nb_ic = (ic + ELEMS_PER_BLOCK - 1) // ELEMS_PER_BLOCK
    n_total = oc * nb_ic * ELEMS_PER_BLOCK
    if n_total != oc * ic:
        try:
            _detect_format(packed.numel(), n_total)
        except ValueError:
            # FP2Linear packs the weight flattened, without row padding
            return _unpack_weight(packed, oc * ic, device=device).reshape_as(w)
    dec = _unpack_weight(packed, n_total, device=device).reshape(oc, -1)
    return dec[:, :ic].reshape_as(w)


def set_force_fake_quant(model: nn.Module, flag: bool):
    """quant_linear.py:371: returns how many layers were switched."""
    n = 0
    for m in model.modules():
        if hasattr(m, "force_fake_quant"):
            m.force_fake_quant = flag
            n += 1
    return n


def _tier(path: str, v3: bool, fp3_tier: bool, fp3_aggressive: bool) -> str:
    """Tier of a Linear under apply_mixed_quant (quant_linear.py:622-657)."""
    if "mlp" in path:
        return "twofour" if v3 else "spfp2"
    if fp3_tier and fp3_aggressive:
        if "o_proj" in path:
            return "fp3"
        if "out_proj" not in path:
            return "spfp2"
    elif fp3_tier:
        if "in_proj_ba" in path:
            return "spfp2"
        if "out_proj" not in path:
            return "fp3"
    return "nvfp4"


def apply_mixed_quant(model: nn.Module, quantize_head: bool = False, v3: bool = False, fp3_tier: bool = False,
                      fp3_aggressive: bool = False) -> nn.Module:
    """quant_linear.py:551-729: the mixed tiers.  MLP projections SPFP2 (2:4
    with v3), attention / DeltaNet projections NVFP4 (or FP3 / SPFP2 with the
    fp3 options), embed / lm_head BF16 -- or, with quantize_head, the embedding
    NVFP4 and a tied lm_head sharing its weight.  Prints per-tier counts."""
    stats = {k: [0, 0] for k in ("nvfp4", "spfp2", "fp3", "int8", "bf16")}
    embed_ref, embed_path = None, None
    for path, module in model.named_modules():
        if isinstance(module, nn.Embedding):
            embed_ref, embed_path = module.weight, path
            break
    tied_head_path = None
    plan = []
    for path, module in model.named_modules():
        if isinstance(module, nn.Embedding):
            key = "nvfp4" if quantize_head else "bf16"
            if quantize_head:
                plan.append((path, "nvfp4_embed"))
            stats[key][0] += 1
            stats[key][1] += module.weight.numel()
            continue
        if not isinstance(module, nn.Linear):
            for pn, prm in module.named_parameters(recurse=False):
                if "A_log" in pn or "dt_bias" in pn:
                    stats["bf16"][1] += prm.numel()
            continue
        if "lm_head" in path:
            if quantize_head and embed_ref is not None and module.weight is embed_ref:
                tied_head_path = path
                stats["nvfp4"][0] += 1
                stats["nvfp4"][1] += module.weight.numel()
            else:
                stats["bf16"][0] += 1
                stats["bf16"][1] += module.weight.numel()
            continue
        if "embed" in path.lower():
            stats["bf16"][0] += 1
            stats["bf16"][1] += module.weight.numel()
            continue
        kind = _tier(path, v3, fp3_tier, fp3_aggressive)
        plan.append((path, kind))
        key = "spfp2" if kind == "twofour" else kind
        stats[key][0] += 1
        stats[key][1] += module.weight.numel()

    classes = {"spfp2": ChannelFP2QATLinear, "fp3": FP3QATLinear, "twofour": TwoFourQATLinear,
               "nvfp4": NVFP4QATLinear, "int8": INT8QATLinear}
    qat_embed = None
    for path, kind in plan:
        parent = model.get_submodule(".".join(path.split(".")[:-1]))
        leaf = path.split(".")[-1]
        old = getattr(parent, leaf)
        if kind == "nvfp4_embed":
            qe = NVFP4EmbeddingQAT(old.num_embeddings, old.embedding_dim, padding_idx=old.padding_idx,
                                   device=old.weight.device, dtype=old.weight.dtype)
            with torch.no_grad():
                qe.weight.copy_(old.weight)
            setattr(parent, leaf, qe)
            if path == embed_path:
                qat_embed = qe
        else:
            setattr(parent, leaf, _replace(classes[kind], old))
    if tied_head_path is not None and qat_embed is not None:
        parent = model.get_submodule(".".join(tied_head_path.split(".")[:-1]))
        leaf = tied_head_path.split(".")[-1]
        old = getattr(parent, leaf)
        head = NVFP4QATLinear(old.in_features, old.out_features, old.bias is not None,
                              device=qat_embed.weight.device, dtype=qat_embed.weight.dtype)
        head.weight = qat_embed.weight            # the tie is kept: one Parameter
        if old.bias is not None:
            with torch.no_grad():
                head.bias.copy_(old.bias)
        setattr(parent, leaf, head)

    total = sum(v[1] for v in stats.values()) or 1
    for k, (n, prm) in stats.items():
        if n or prm:
            print(f"[spark_b200 mixed] {k.upper():5s}: {n:4d} layers  {prm / 1e9:.2f}B ({prm / total * 100:.1f}%)")
    bits = (stats["spfp2"][1] * 2.5 + stats["fp3"][1] * 3.5 + stats["nvfp4"][1] * 4.5 + stats["int8"][1] * 8
            + stats["bf16"][1] * 16)
    print(f"[spark_b200 mixed] {bits / total:.2f} bit/weight, ~{bits / 8 / 1e9:.2f} GB of weights")
    return model
