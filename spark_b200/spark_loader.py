"""Drop-in for 02_model/spark_loader.py: read a SPARK checkpoint and apply it
to a model, decoding on the GPU.  Adds a packed-resident variant that keeps
the codes on the device and serves the layers from them.

State-dict keys (as the reference exporter writes them):
  <layer>_packed (+ <layer>_meta = (oc, ic))   SPFP2, paired or 3-byte blocks
  <layer>_fp3_codes / _fp3_scales (+ _meta)    FP3 (3-bit codes or nibbles)
  <layer>_nvfp4_codes / _nvfp4_scales (+ _meta) NVFP4
  <layer>_nvfp4_weight                         NVFP4 values stored unpacked
  param::<name>                                any other parameter
"""
from __future__ import annotations

import os

import torch

from . import ops
from .block_fp2 import ELEMS_PER_BLOCK
from .quant_linear import _unpack_weight


def _meta(state: dict, layer: str):
    meta = state.get(layer + "_meta")
    return None if meta is None else (int(meta[0]), int(meta[1]))


def _fp3_nibble(codes: torch.Tensor, oc: int, ic: int) -> bool:
    """FP3 codes: nibbles (fp3_emu.fp3_pack, 4 bits a weight) or 3-bit groups
    (fp3_pack_3bit); the byte count tells them apart."""
    n = oc * ((ic + 15) // 16) * 16
    return codes.numel() == (n + 1) // 2


def decode_spfp2(packed: torch.Tensor, oc: int, ic: int, device="cpu") -> torch.Tensor:
    """(oc, ic) fp32 from a row-padded SPFP2 weight (either block layout)."""
    nb_ic = (ic + ELEMS_PER_BLOCK - 1) // ELEMS_PER_BLOCK
    dec = _unpack_weight(packed, oc * nb_ic * ELEMS_PER_BLOCK, device=device)
    return dec.reshape(oc, -1)[:, :ic]


class SparkWeightLoader:
    """spark_loader.py:13-64: a .spark directory's state_dict.pt, decoded."""

    def __init__(self, spark_dir: str):
        self.spark_dir = spark_dir
        pth = os.path.join(spark_dir, "state_dict.pt")
        if not os.path.exists(pth):
            raise FileNotFoundError(f"not found: {pth}")
        self.data = torch.load(pth, map_location="cpu", weights_only=False)

    def state_dict(self):
        """{<layer>.weight: fp16 (oc, ic)} for every SPFP2 layer (spark_loader.py:22-53)."""
        state = {}
        for pk in sorted(k for k in self.data if k.endswith("_packed")):
            layer = pk[: -len("_packed")]
            shape = _meta(self.data, layer)
            if shape is None:
                raise KeyError(f"missing '{layer}_meta' shape metadata (oc, ic) for layer '{layer}'")
            state[layer + ".weight"] = self._decode_weight(self.data[pk], *shape)
        return state

    def _decode_weight(self, packed: torch.Tensor, oc: int, ic: int) -> torch.Tensor:
        return decode_spfp2(packed, oc, ic).contiguous().to(torch.float16)


def load_spark_model(spark_dir: str, hf_base: str):
    """spark_loader.py:67-93: HF base model + decoded SPARK weights, eval mode."""
    from transformers import AutoModelForCausalLM, AutoTokenizer
    model = AutoModelForCausalLM.from_pretrained(hf_base, device_map="cpu", low_cpu_mem_usage=True,
                                                 torch_dtype=torch.float32)
    decoded = SparkWeightLoader(spark_dir).state_dict()
    msd = model.state_dict()
    with torch.no_grad():
        for name, w in decoded.items():
            if name in msd and msd[name].shape == w.shape:
                msd[name].copy_(w.to(msd[name].dtype))
    tok = AutoTokenizer.from_pretrained(hf_base, trust_remote_code=True)
    if tok.pad_token is None:
        tok.pad_token = tok.eos_token
    return model.eval(), tok


def apply_spark_state(model, state):
    """spark_loader.py:102-163: decode every packed entry into the model's
    weights; returns (n_spfp2, n_fp3_or_nvfp4, n_param)."""
    msd = model.state_dict()
    n1 = n2 = n3 = 0

    def put(name, w):
        if name in msd and msd[name].shape == w.shape:
            with torch.no_grad():
                msd[name].copy_(w.to(device=msd[name].device, dtype=msd[name].dtype))
            return 1
        return 0

    for key in list(state.keys()):
        if key.endswith("_packed"):
            layer = key[: -len("_packed")]
            shape = _meta(state, layer)
            if shape is not None:
                n1 += put(layer + ".weight", decode_spfp2(state[key], *shape))
        elif key.endswith("_fp3_codes"):
            layer = key[: -len("_fp3_codes")]
            shape = _meta(state, layer)
            if shape is None or layer + "_fp3_scales" not in state:
                continue
            codes = state[key]
            w = ops.fp3_unpack(codes, state[layer + "_fp3_scales"], *shape, nibble=_fp3_nibble(codes, *shape))
            n2 += put(layer + ".weight", w)
        elif key.endswith("_nvfp4_codes"):
            layer = key[: -len("_nvfp4_codes")]
            shape = _meta(state, layer)
            if shape is None or layer + "_nvfp4_scales" not in state:
                continue
            n2 += put(layer + ".weight", ops.nvfp4_unpack(state[key], state[layer + "_nvfp4_scales"], *shape))
        elif key.endswith("_nvfp4_weight"):
            n2 += put(key[: -len("_nvfp4_weight")] + ".weight", state[key].float())
        elif key.startswith("param::"):
            n3 += put(key[len("param::"):], state[key].float())
    return n1, n2, n3


def apply_spark_state_resident(model, state, device="cuda"):
    """Packed-resident variant (no counterpart in the reference loader): every
    nn.Linear with SPFP2 / FP3 / NVFP4 entries becomes a V3PackedLinear that
    keeps the codes on `device` and runs the dequant linear on them; the other
    parameters are copied in.  Returns (n_packed_layers, n_param)."""
    from .inference_v3 import build_v3_layers
    n_layers = build_v3_layers(model, state, device=device)
    msd = model.state_dict()
    n_param = 0
    with torch.no_grad():
        for key, val in state.items():
            if key.startswith("param::"):
                name = key[len("param::"):]
                if name in msd and msd[name].shape == val.shape:
                    msd[name].copy_(val.float().to(device=msd[name].device, dtype=msd[name].dtype))
                    n_param += 1
    return n_layers, n_param
