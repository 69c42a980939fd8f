"""CPU tests of the container, the registered torch ops' schemas and the
layer-split export (gloo, two ranks): host logic only, no kernel launches."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from spark_b200 import spark_v2_container as C


@pytest.mark.parametrize("n", [0, 1, 5, 128 * 1024, 128 * 1024 + 17, 300_000])
def test_raw_zstd_frame_round_trip(n):
    raw = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    frame = C._frame_raw(raw)
    assert frame[:4] == bytes.fromhex("28b52ffd")       # zstd magic number, little endian
    assert C._unframe(frame) == raw
    assert C._unframe(frame + frame) == raw + raw         # concatenated frames decode in order


def test_unframe_rle_and_skippable():
    # a skippable frame, then a frame with one RLE block of 1000 x 0xAB
    skip = (0x184D2A5A).to_bytes(4, "little") + (3).to_bytes(4, "little") + b"xyz"
    hdr = (0xFD2FB528).to_bytes(4, "little") + bytes([0x20, 0])     # single segment, 1-byte size (0: unused)
    blk = (1 | (1 << 1) | (1000 << 3)).to_bytes(3, "little") + b"\xab"
    assert C._unframe(skip + hdr + blk) == b"\xab" * 1000


def _state():
    g = torch.Generator().manual_seed(0)
    return {
        "model.layers.0.mlp.down_proj_packed": torch.randint(0, 256, (2560 * 128 // 16 * 5,), generator=g,
                                                            dtype=torch.uint8),
        "model.layers.0.mlp.down_proj_scale_index": torch.randint(0, 16, (2560 * 16,), generator=g,
                                                                  dtype=torch.uint8),
        "model.layers.0.mlp.down_proj_meta": torch.tensor([2560, 128]),
        "model.layers.0.self_attn.q_proj_fp3_codes": torch.randint(0, 256, (64 * 256 // 8 * 3,), generator=g,
                                                                   dtype=torch.uint8),
        "model.layers.0.self_attn.q_proj_fp3_scales": torch.randint(0, 120, (64 * 16,), generator=g,
                                                                    dtype=torch.uint8).view(torch.float8_e4m3fn),
        "model.layers.0.self_attn.q_proj_meta": torch.tensor([64, 256]),
        "model.layers.0.self_attn.o_proj_nvfp4_codes": torch.randint(0, 256, (32 * 128 // 2,), generator=g,
                                                                     dtype=torch.uint8),
        "model.layers.0.self_attn.o_proj_nvfp4_scales": torch.randint(0, 120, (32 * 8,), generator=g,
                                                                      dtype=torch.uint8).view(torch.float8_e4m3fn),
        "model.layers.0.self_attn.o_proj_meta": torch.tensor([32, 128]),
        "param::model.norm.weight": torch.randn(64, generator=g).bfloat16(),
        "param::model.layers.0.linear_attn.A_log": torch.randn(4, 8, generator=g),
        "extra_blob": torch.arange(10, dtype=torch.uint8),
    }


def test_container_round_trip(tmp_path):
    state = _state()
    cfg = tmp_path / "base"
    cfg.mkdir()
    (cfg / "config.json").write_text('{"model_type": "test"}')
    out = str(tmp_path / "c")
    stats = C.save_spark_v2(state, out, base_model_dir=str(cfg))
    assert stats["comp"] > 0 and stats["raw"] > 0
    man = json.load(open(os.path.join(out, "manifest.json")))
    assert man["version"] == "2.0" and man["format"] == "spark-v2"
    kinds = {k: e["kind"] for k, e in man["tensors"].items()}
    assert kinds["model.layers.0.mlp.down_proj_packed"] == "spfp2_packed"
    assert kinds["model.layers.0.self_attn.q_proj_fp3_codes"] == "fp3_codes"
    assert kinds["model.layers.0.self_attn.q_proj_fp3_scales"] == "fp3_scales"
    assert kinds["model.layers.0.self_attn.o_proj_nvfp4_codes"] == "nvfp4_codes"
    assert kinds["param::model.norm.weight"] == "param_fp32"
    assert kinds["extra_blob"] == "raw"
    # _meta / _scale_index are folded into their entries, as the reference does
    assert not any(k.endswith("_meta") or k.endswith("_scale_index") for k in kinds)
    assert man["tensors"]["model.layers.0.mlp.down_proj_packed"]["oc"] == 2560
    assert os.path.exists(os.path.join(out, "config.json"))
    for e in man["tensors"].values():
        assert e["file"].startswith("tensors/") and e["file"].endswith(".zst")

    back = C.load_spark_v2(out)
    for k in ("model.layers.0.mlp.down_proj_packed", "model.layers.0.self_attn.q_proj_fp3_codes",
              "model.layers.0.self_attn.o_proj_nvfp4_codes", "extra_blob"):
        assert torch.equal(back[k], state[k]), k
    for k in ("model.layers.0.self_attn.q_proj_fp3_scales", "model.layers.0.self_attn.o_proj_nvfp4_scales"):
        assert back[k].dtype == torch.float8_e4m3fn
        assert torch.equal(back[k].view(torch.uint8), state[k].view(torch.uint8)), k
    for layer in ("model.layers.0.mlp.down_proj", "model.layers.0.self_attn.q_proj", "model.layers.0.self_attn.o_proj"):
        assert torch.equal(back[layer + "_meta"], state[layer + "_meta"].long()), layer
    # params come back fp32 with their shape, bit-exact
    assert torch.equal(back["param::model.norm.weight"], state["param::model.norm.weight"].float())
    assert torch.equal(back["param::model.layers.0.linear_attn.A_log"], state["param::model.layers.0.linear_attn.A_log"])
    assert C.container_size_gb(out) > 0


def test_torch_ops_registered():
    import spark_b200  # noqa: F401  (registers the ops)
    s = str(torch.ops.spark.decode_fp32.default._schema)
    assert s.startswith("spark::decode_fp32(Tensor packed, SymInt rows) -> Tensor")
    s = str(torch.ops.spark.spark_v3_spfp2_forward.default._schema)
    assert "Tensor w_packed, Tensor x, Tensor(a2!) y, Tensor bias, SymInt oc, SymInt ic" in s
    assert "spark_v3_twofour_forward" in str(torch.ops.spark.spark_v3_twofour_forward.default._schema)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.spark.decode_fp32(torch.zeros(5, dtype=torch.uint8), 16)


def _export_rank(rank, world, port, state, q):
    import torch.distributed as dist
    from spark_b200 import export as E
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    calls = []

    def fake_ptq(pname, w):
        calls.append(pname)
        layer = pname[: -len(".weight")]
        kind = "_nvfp4_codes" if "out_proj" in pname else "_fp3_codes"
        return {layer + kind: (w.float().sum() * 0 + len(pname)).reshape(1), layer + "_meta": torch.tensor(list(w.shape))}

    E._ptq = fake_ptq
    out, counts = E.export_spark(state, rank, world)
    q.put((rank, sorted(calls), sorted(out.keys()), counts))
    dist.barrier()
    dist.destroy_process_group()


def test_export_split_by_layer_gloo():
    """PTQ layers are split round-robin over the ranks; every rank returns the
    complete export state (the packing itself runs on the GPU and is tested
    there; here a stand-in records which rank handled which layer)."""
    state = {f"param::model.layers.{i}.self_attn.{p}.weight": torch.randn(8, 16)
             for i in range(3) for p in ("q_proj", "out_proj")}
    state["param::model.layers.0.mlp.up_proj.weight"] = torch.randn(8, 16)   # skipped (SPFP2 covers the MLP)
    state["param::model.norm.weight"] = torch.randn(16)                       # carried over
    state["model.layers.0.mlp.up_proj_packed"] = torch.zeros(40, dtype=torch.uint8)
    state["model.layers.0.mlp.up_proj_meta"] = torch.tensor([8, 16])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_export_rank, args=(r, 2, port, state, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (c, k, n)) for r, c, k, n in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    calls0, keys0, n0 = res[0]
    calls1, keys1, n1 = res[1]
    assert keys0 == keys1 and n0 == n1 == {"spfp2": 1, "fp3": 3, "nvfp4": 3}
    assert not set(calls0) & set(calls1) and len(calls0) + len(calls1) == 6
    assert "param::model.norm.weight" in keys0 and "param::model.layers.0.mlp.up_proj.weight" not in keys0
