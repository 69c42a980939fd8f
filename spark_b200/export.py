"""Export of quantized models to SPARK states, on the GPU kernels.

  export_spark_model(model, out_dir, base_model_dir=None)
        mirror of 02_model/spark_exporter.py:16-48: <name>_packed,
        <name>_scale_index, <name>_meta of every packed SPFP2 layer (embeddings
        and lm_head excepted) into <out_dir>/state_dict.pt.
  save_quantized(model, outdir, tag="final")
        the state SPARKQATrainer._save_quantized writes (03_training/trainer.py:588-658):
        SPFP2 layers quantize() -> _packed / _scale_index / _meta; FP3 layers ->
        fp3_pack_3bit(weight) codes + scales; NVFP4 layers and embeddings ->
        nvfp4_pack(nvfp4_fake_quant(weight)); every other parameter as
        param::<name> in bf16.  Returns (state, path).
  export_spark(state, rank=0, world=1, group=None)
        steps 1-2 of 04_scripts/export_spark.py:36-100: SPFP2 _packed / _meta
        carried over; every 2-D param::*.weight outside the MLP gets PTQ --
        NVFP4 (out_proj / embed / lm_head names) as
        nvfp4_pack(nvfp4_fake_quant(w)), FP3 otherwise as
        fp3_pack_3bit(fp3_fake_quant(w)); other params carried over.  With
        world > 1 the PTQ layers are split round-robin over the ranks and the
        packed bytes gathered on the host (every rank returns the whole state).
"""
from __future__ import annotations

import os
import shutil

import torch
import torch.distributed as dist

from . import ops


def _is_spark_quant_layer(module) -> bool:
    return isinstance(module, torch.nn.Module) and hasattr(module, "_packed_weight")


def export_spark_model(model: torch.nn.Module, out_dir: str, base_model_dir: str | None = None) -> dict:
    os.makedirs(out_dir, exist_ok=True)
    state = {}
    for name, module in model.named_modules():
        if not _is_spark_quant_layer(module) or "embed" in name.lower() or "lm_head" in name:
            continue
        if module._packed_weight is None:
            continue
        n = name.replace(".weight", "")
        state[n + "_packed"] = module._packed_weight.cpu()
        idx = getattr(module, "_channel_scale_index", None)
        if idx is not None:
            state[n + "_scale_index"] = idx.cpu()
        oc, ic = module.weight.shape
        state[n + "_meta"] = torch.tensor([oc, ic], dtype=torch.long)
    if base_model_dir is not None:
        src = os.path.join(base_model_dir, "config.json")
        if os.path.exists(src):
            shutil.copy(src, os.path.join(out_dir, "config.json"))
    torch.save(state, os.path.join(out_dir, "state_dict.pt"))
    return state


def save_quantized(model: torch.nn.Module, outdir: str, tag="final") -> tuple[dict, str]:
    from .fp3_linear import FP3QATLinear
    from .quant_linear import ChannelFP2QATLinear, NVFP4EmbeddingQAT, NVFP4QATLinear
    state = {}
    quant_ids = set()
    with torch.no_grad():
        for name, module in model.named_modules():
            n = name.replace(".weight", "")
            if isinstance(module, ChannelFP2QATLinear):
                module.quantize()
                state[n + "_packed"] = module._packed_weight.cpu()
                if module._channel_scale_index is not None:
                    state[n + "_scale_index"] = module._channel_scale_index.cpu()
                state[n + "_meta"] = torch.tensor([module.out_features, module.in_features], dtype=torch.long)
                quant_ids.add(id(module.weight))
            elif isinstance(module, FP3QATLinear):
                codes, scales = ops.fp3_pack(module.weight.detach().float())
                state[n + "_fp3_codes"] = codes.cpu()
                state[n + "_fp3_scales"] = scales.cpu()
                state[n + "_meta"] = torch.tensor(list(module.weight.shape), dtype=torch.long)
                quant_ids.add(id(module.weight))
            elif isinstance(module, (NVFP4QATLinear, NVFP4EmbeddingQAT)):
                w = module.weight.detach().float()
                codes, scales = ops.nvfp4_pack(ops.nvfp4_fake_quant(w))
                state[n + "_nvfp4_codes"] = codes.cpu()
                state[n + "_nvfp4_scales"] = scales.cpu()
                state[n + "_meta"] = torch.tensor(list(module.weight.shape), dtype=torch.long)
                quant_ids.add(id(module.weight))
        for pname, p in model.named_parameters():
            if id(p) not in quant_ids:
                state["param::" + pname] = p.detach().float().bfloat16().cpu()
    os.makedirs(outdir, exist_ok=True)
    path = os.path.join(outdir, f"spark-qat-{tag}.pt")
    torch.save(state, path)
    return state, path


def _ptq(pname: str, w: torch.Tensor) -> dict:
    """PTQ of one trained 2-D weight (export_spark.py:79-96): double
    quantization pack(fake_quant(w)) on the GPU."""
    layer = pname[: -len(".weight")]
    wc = w.float().cuda() if torch.cuda.is_available() else w.float()
    meta = torch.tensor(list(w.shape[:2]))
    if "out_proj" in pname or "embed" in pname or "lm_head" in pname:
        codes, scales = ops.nvfp4_pack(ops.nvfp4_fake_quant(wc))
        return {layer + "_nvfp4_codes": codes.cpu(), layer + "_nvfp4_scales": scales.cpu(), layer + "_meta": meta}
    codes, scales = ops.fp3_pack(ops.fp3_fake_quant(wc))
    return {layer + "_fp3_codes": codes.cpu(), layer + "_fp3_scales": scales.cpu(), layer + "_meta": meta}


def export_spark(state: dict, rank: int = 0, world: int = 1, group=None) -> tuple[dict, dict]:
    """Returns (export_state, counts) with counts = {"spfp2", "fp3", "nvfp4"}."""
    out = {}
    for k, v in state.items():
        if k.endswith("_packed"):
            out[k] = v
            meta = state.get(k[: -len("_packed")] + "_meta")
            if meta is not None:
                out[k[: -len("_packed")] + "_meta"] = meta
    jobs = []
    for k, v in state.items():
        if not k.startswith("param::"):
            continue
        pname = k[len("param::"):]
        if not pname.endswith(".weight") or v.dim() != 2:
            out[k] = v                       # norms, A_log, conv1d (3-D) ... carried over
            continue
        if "mlp" in pname:
            continue                         # covered by the SPFP2 packed entries
        jobs.append((pname, v))
    mine = {}
    for i, (pname, v) in enumerate(jobs):
        if i % world == rank:
            mine.update(_ptq(pname, v))
    if world > 1:
        parts: list = [None] * world
        dist.all_gather_object(parts, mine, group=group)
        for p in parts:
            out.update(p)
    else:
        out.update(mine)
    counts = {"spfp2": sum(k.endswith("_packed") for k in out), "fp3": sum(k.endswith("_fp3_codes") for k in out),
              "nvfp4": sum(k.endswith("_nvfp4_codes") for k in out)}
    return out, counts
