"""SPARK v2 container (mirror of 02_model/spark_v2_container.py).

Directory layout, as the reference writes it:
  <out>/manifest.json   {"version": "2.0", "format": "spark-v2", "tensors": {key: entry}}
  <out>/tensors/*.zst   one zstd frame per tensor
  <out>/config.json     the base model's config (when given)

Entry kinds and what load_spark_v2 rebuilds (02_model/spark_v2_container.py:70-240):
  spfp2_packed   <layer>_packed (+ <layer>_meta from oc/ic)
  fp3_codes / fp3_scales       <layer>_fp3_codes, _fp3_scales, _meta
  nvfp4_codes / nvfp4_scales   <layer>_nvfp4_codes, _nvfp4_scales, _meta
                 (legacy <layer>_nvfp4_weight values are re-packed to codes on save)
  int8_head_q / int8_head_scale  param::*lm_head* stored per-row INT8, loaded
                 back as bf16 (ptq_int8_pack / ptq_int8_unpack)
  param_fp32     other param:: tensors, fp32 (bit-exact round trip)
  raw            anything else, bytes

The re-pack of legacy NVFP4 values and the INT8 head run on the GPU kernels.
Blobs are zstd frames: with the `zstandard` module installed they are
compressed as the reference does (level 19); without it, frames of raw zstd
blocks are written (valid zstd that any reader decodes, no size reduction) and
only such frames can be read back.
"""
from __future__ import annotations

import json
import os
import shutil
import struct

import torch

CONTAINER_VERSION = "2.0"

_ZSTD_MAGIC = 0xFD2FB528
_RAW_BLOCK = 128 * 1024


def _zstd():
    try:
        import zstandard
        return zstandard
    except ImportError:
        return None


def _frame_raw(raw: bytes) -> bytes:
    """One zstd frame of raw blocks (RFC 8878 3.1): single segment, 8-byte
    content size, no checksum."""
    out = bytearray(struct.pack("<IB", _ZSTD_MAGIC, 0xE0))
    out += struct.pack("<Q", len(raw))
    pos = 0
    while True:
        n = min(_RAW_BLOCK, len(raw) - pos)
        last = pos + n >= len(raw)
        out += (int(last) | (0 << 1) | (n << 3)).to_bytes(3, "little")
        out += raw[pos:pos + n]
        pos += n
        if last:
            return bytes(out)


def _unframe(buf: bytes) -> bytes:
    """Content of zstd frames made of raw / RLE blocks (skippable frames are
    skipped).  Compressed blocks need the zstandard module."""
    out = bytearray()
    pos = 0
    while pos < len(buf):
        magic = struct.unpack_from("<I", buf, pos)[0]
        if magic & 0xFFFFFFF0 == 0x184D2A50:
            size = struct.unpack_from("<I", buf, pos + 4)[0]
            pos += 8 + size
            continue
        if magic != _ZSTD_MAGIC:
            raise ValueError("not a zstd frame")
        fhd = buf[pos + 4]
        pos += 5
        fcs_flag, single, checksum, dict_flag = fhd >> 6, (fhd >> 5) & 1, (fhd >> 2) & 1, fhd & 3
        if not single:
            pos += 1
        pos += (0, 1, 2, 4)[dict_flag]
        pos += (1 if single else 0, 2, 4, 8)[fcs_flag]
        while True:
            hdr = int.from_bytes(buf[pos:pos + 3], "little")
            pos += 3
            last, btype, size = hdr & 1, (hdr >> 1) & 3, hdr >> 3
            if btype == 0:
                out += buf[pos:pos + size]
                pos += size
            elif btype == 1:
                out += bytes([buf[pos]]) * size
                pos += 1
            else:
                raise RuntimeError("this blob holds compressed zstd blocks: install the zstandard module to read it")
            if last:
                break
        if checksum:
            pos += 4
    return bytes(out)


def _raw_bytes(t: torch.Tensor) -> bytes:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bfloat16, torch.float16):
        t = t.view(torch.uint8 if t.dtype == torch.float8_e4m3fn else torch.int16)
    return t.numpy().tobytes()


def _compress(t: torch.Tensor) -> bytes:
    raw = _raw_bytes(t)
    z = _zstd()
    if z is not None:
        return z.ZstdCompressor(level=19, threads=-1).compress(raw)
    return _frame_raw(raw)


def _decompress(buf: bytes, dtype: torch.dtype) -> torch.Tensor:
    z = _zstd()
    raw = z.ZstdDecompressor().decompress(buf) if z is not None else _unframe(buf)
    if dtype == torch.float8_e4m3fn:
        return torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(torch.float8_e4m3fn).clone()
    if dtype == torch.bfloat16:
        return torch.frombuffer(bytearray(raw), dtype=torch.int16).view(torch.bfloat16).clone()
    if len(raw) == 0:
        return torch.empty(0, dtype=dtype)
    return torch.frombuffer(bytearray(raw), dtype=dtype).clone()


def _meta_of(state: dict, layer: str):
    meta = state.get(layer + "_meta")
    return (int(meta[0]), int(meta[1])) if meta is not None else (None, None)


def save_spark_v2(state: dict, out_dir: str, base_model_dir: str | None = None) -> dict:
    """Write a training / export state (v1 key layout) as a v2 container.
    Returns {"raw": bytes before compression, "comp": blob bytes}."""
    from . import ops
    os.makedirs(os.path.join(out_dir, "tensors"), exist_ok=True)
    manifest = {"version": CONTAINER_VERSION, "format": "spark-v2", "tensors": {}}
    stats = {"raw": 0, "comp": 0}

    def emit(name: str, kind: str, payload: bytes, **extra) -> None:
        fname = f"tensors/{name.replace('::', '_')}.zst"
        with open(os.path.join(out_dir, fname), "wb") as f:
            f.write(payload)
        manifest["tensors"][name] = dict(kind=kind, file=fname, bytes=len(payload), **extra)
        stats["comp"] += len(payload)

    # merged into their codes / packed entries
    merged = ("_meta", "_scale_index", "_nvfp4_scales", "_fp3_scales")
    for key, val in state.items():
        if any(key.endswith(sfx) for sfx in merged):
            continue
        stats["raw"] += val.numel() * val.element_size()
        if key.endswith("_fp3_codes"):
            layer = key[: -len("_fp3_codes")]
            oc, ic = _meta_of(state, layer)
            emit(key, "fp3_codes", _compress(val), oc=oc, ic=ic)
            sc = state.get(layer + "_fp3_scales")
            if sc is not None:
                emit(layer + "_fp3_scales", "fp3_scales", _compress(sc))
        elif key.endswith("_nvfp4_codes"):
            layer = key[: -len("_nvfp4_codes")]
            oc, ic = _meta_of(state, layer)
            emit(key, "nvfp4_codes", _compress(val), oc=oc, ic=ic)
            sc = state.get(layer + "_nvfp4_scales")
            if sc is not None:
                emit(layer + "_nvfp4_scales", "nvfp4_scales", _compress(sc))
        elif key.endswith("_nvfp4_weight"):
            # legacy entries hold NVFP4 values: re-pack them to codes + scales
            layer = key[: -len("_nvfp4_weight")]
            oc, ic = _meta_of(state, layer)
            if oc is None:
                oc, ic = tuple(val.shape[:2])
            codes, scales = ops.nvfp4_pack(val.float())
            emit(key, "nvfp4_codes", _compress(codes), oc=oc, ic=ic, codes_numel=codes.numel())
            emit(key + "::scales", "nvfp4_scales", _compress(scales), scales_numel=scales.numel())
        elif key.endswith("_packed"):
            layer = key[: -len("_packed")]
            oc, ic = _meta_of(state, layer)
            emit(key, "spfp2_packed", _compress(val), oc=oc, ic=ic)
        elif key.startswith("param::") and "lm_head" in key:
            q, scale = ops.int8_pack(val.float())
            emit(key, "int8_head_q", _compress(q), shape=list(val.shape))
            emit(key + "::scale", "int8_head_scale", _compress(scale))
        elif key.startswith("param::"):
            # fp32 keeps norms / A_log etc. bit-exact through the round trip
            emit(key, "param_fp32", _compress(val.float()), shape=list(val.shape))
        else:
            emit(key, "raw", _compress(val))

    if base_model_dir:
        src = os.path.join(base_model_dir, "config.json")
        if os.path.exists(src):
            shutil.copy(src, os.path.join(out_dir, "config.json"))
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return stats


def load_spark_v2(out_dir: str) -> dict:
    """Read a v2 container back into the v1 key layout (what apply_spark_state
    and apply_spark_state_resident take).  Tensors are on the CPU."""
    from . import ops
    with open(os.path.join(out_dir, "manifest.json")) as f:
        manifest = json.load(f)

    def blob(e: dict, dtype: torch.dtype) -> torch.Tensor:
        with open(os.path.join(out_dir, e["file"]), "rb") as f:
            return _decompress(f.read(), dtype)

    state, heads, coded = {}, {}, {}
    for key, e in manifest["tensors"].items():
        kind = e["kind"]
        if kind in ("fp3_codes", "nvfp4_codes"):
            c = coded.setdefault(key, {})
            c["codes"], c["oc"], c["ic"] = blob(e, torch.uint8), e.get("oc"), e.get("ic")
        elif kind == "fp3_scales":
            coded.setdefault(key.replace("_fp3_scales", "_fp3_codes"), {})["scales"] = blob(e, torch.float8_e4m3fn)
        elif kind == "nvfp4_scales":
            base = key.replace("::scales", "").replace("_nvfp4_scales", "_nvfp4_codes")
            coded.setdefault(base, {})["scales"] = blob(e, torch.float8_e4m3fn)
        elif kind == "spfp2_packed":
            state[key] = blob(e, torch.uint8)
            if e.get("oc"):
                state[key[: -len("_packed")] + "_meta"] = torch.tensor([e["oc"], e["ic"]], dtype=torch.long)
        elif kind == "int8_head_q":
            heads[key] = {"q": blob(e, torch.int8), "shape": e["shape"]}
        elif kind == "int8_head_scale":
            heads[key.replace("::scale", "")]["scale"] = blob(e, torch.float32)
        elif kind == "param_fp32":
            state[key] = blob(e, torch.float32).reshape(e["shape"]) if "shape" in e else blob(e, torch.float32)
        else:
            state[key] = blob(e, torch.uint8)

    for key, c in coded.items():
        if "codes" not in c or "scales" not in c:
            continue
        if key.endswith("_fp3_codes"):
            layer = key[: -len("_fp3_codes")]
            state[key], state[layer + "_fp3_scales"] = c["codes"], c["scales"]
        else:
            # a legacy "<layer>_nvfp4_weight" entry comes back as <layer>_nvfp4_codes /
            # _nvfp4_scales (the reference loader writes both under the legacy key,
            # so its scales replace its codes)
            layer = key[: -len("_nvfp4_weight")] if key.endswith("_nvfp4_weight") else key[: -len("_nvfp4_codes")]
            state[layer + "_nvfp4_codes"], state[layer + "_nvfp4_scales"] = c["codes"], c["scales"]
        if c.get("oc") is not None:
            state[layer + "_meta"] = torch.tensor([c["oc"], c["ic"]], dtype=torch.long)
    for key, h in heads.items():
        if "scale" in h:
            q = h["q"].reshape(h["shape"])
            state[key] = ops.int8_unpack(q, h["scale"]).bfloat16()
    return state


def container_size_gb(out_dir: str) -> float:
    total = 0
    for root, _, files in os.walk(out_dir):
        for f in files:
            total += os.path.getsize(os.path.join(root, f))
    return total / 1024 ** 3
