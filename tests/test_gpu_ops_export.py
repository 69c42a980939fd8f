"""The registered torch ops (torch.ops.spark.*) and the GPU export / container
paths against the oracle.

Bit-exact: decode_fp32 / decode_fp16 on arbitrary bytes (the legacy
single-exponent blocks), the PTQ bytes of export_spark (double quantization
pack(fake_quant(w)), 04_scripts/export_spark.py:79-90) and the INT8 head of the
container.  Forward ops: max |y - y_ref| within fp16 output rounding
(2^-11 relative) + 5e-4 against an fp64 accumulation of the oracle-decoded
weights, since the reference ops write fp16.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_decode_ops_bit_exact():
    import spark_b200  # noqa: F401
    rng = np.random.default_rng(1)
    raw = rng.integers(0, 256, 5 * 4099, dtype=np.uint8)
    ref = O.spfp2_legacy_decode(raw)
    p = torch.from_numpy(raw).cuda()
    y32 = torch.ops.spark.decode_fp32(p, 16 * 4099)
    y16 = torch.ops.spark.decode_fp16(p, 16 * 4099)
    assert y32.dtype == torch.float32 and y16.dtype == torch.float16
    assert np.array_equal(y32.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert torch.equal(y16.cpu(), torch.from_numpy(ref).half())
    with pytest.raises(RuntimeError, match="size mismatch"):
        torch.ops.spark.decode_fp32(p, 16)


@pytest.mark.parametrize("oc,ic,M", [(256, 512, 1), (100, 44, 3), (512, 1024, 20)])
def test_v3_spfp2_forward(oc, ic, M):
    import spark_b200  # noqa: F401
    from spark_b200 import ops
    g = torch.Generator().manual_seed(oc + ic)
    icp = (ic + 7) // 8 * 8
    W = torch.zeros(oc, icp)
    W[:, :ic] = torch.randn(oc, ic, generator=g) * 0.02
    packed, _ = O.pack_blockwise_search(W.numpy())          # the reference kernel's 3-byte rows
    dec = O.unpack_blockwise(packed).reshape(oc, icp)[:, :ic]
    x = torch.randn(M, ic, generator=g).half()
    bias = torch.randn(oc, generator=g) * 0.1
    y = torch.empty(M, oc, dtype=torch.float16, device="cuda")
    torch.ops.spark.spark_v3_spfp2_forward(torch.from_numpy(packed).cuda(), x.cuda(), y, bias.cuda(), oc, ic)
    y64 = O.linear_f64(x.float().numpy(), np.ascontiguousarray(dec), bias.numpy())
    err = np.abs(y.float().cpu().numpy() - y64)
    assert np.all(err <= 5e-4 + 2.0 ** -11 * np.abs(y64))
    # empty bias = none
    torch.ops.spark.spark_v3_spfp2_forward(torch.from_numpy(packed).cuda(), x.cuda(), y,
                                           torch.empty(0, device="cuda"), oc, ic)
    y64 = O.linear_f64(x.float().numpy(), np.ascontiguousarray(dec))
    assert np.all(np.abs(y.float().cpu().numpy() - y64) <= 5e-4 + 2.0 ** -11 * np.abs(y64))
    ops.check_device_errors()


@pytest.mark.parametrize("oc,ic,M", [(256, 512, 1), (64, 48, 2)])
def test_v3_twofour_forward(oc, ic, M):
    import spark_b200  # noqa: F401
    g = torch.Generator().manual_seed(7 + ic)
    icp = (ic + 31) // 32 * 32
    W = torch.zeros(oc, icp)
    W[:, :ic] = torch.randn(oc, ic, generator=g) * 0.02
    packed = O.two_four_pack(W.numpy())
    dec = O.two_four_unpack(packed, oc * icp).reshape(oc, icp)[:, :ic]
    x = torch.randn(M, ic, generator=g).half()
    y = torch.empty(M, oc, dtype=torch.float16, device="cuda")
    torch.ops.spark.spark_v3_twofour_forward(torch.from_numpy(packed).cuda(), x.cuda(), y,
                                             torch.empty(0, device="cuda"), oc, ic)
    y64 = O.linear_f64(x.float().numpy(), np.ascontiguousarray(dec))
    assert np.all(np.abs(y.float().cpu().numpy() - y64) <= 5e-4 + 2.0 ** -11 * np.abs(y64))


def test_forward_ops_validate():
    import spark_b200  # noqa: F401
    w = torch.zeros(30, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1, 16, dtype=torch.float16, device="cuda")
    y = torch.zeros(1, 4, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="weight bytes"):
        torch.ops.spark.spark_v3_spfp2_forward(w[:10], x, y, torch.empty(0, device="cuda"), 4, 16)
    with pytest.raises(RuntimeError, match=r"x must be \[M, 32\]"):
        torch.ops.spark.spark_v3_spfp2_forward(w, x, y, torch.empty(0, device="cuda"), 4, 32)
    with pytest.raises(RuntimeError, match="bias"):
        torch.ops.spark.spark_v3_spfp2_forward(w, x, y, torch.zeros(3, device="cuda"), 4, 16)


def test_export_spark_ptq_bit_exact():
    """FP3 / NVFP4 PTQ of trained weights = the reference's
    fp3_pack_3bit(fp3_fake_quant(w)) / nvfp4_pack(nvfp4_fake_quant(w))."""
    from spark_b200 import export as E
    g = torch.Generator().manual_seed(3)
    state = {"param::model.layers.0.self_attn.q_proj.weight": (torch.randn(64, 256, generator=g) * 0.02).bfloat16(),
             "param::model.layers.0.self_attn.out_proj.weight": (torch.randn(48, 128, generator=g) * 0.02).bfloat16(),
             "param::model.layers.0.mlp.gate_proj.weight": torch.randn(8, 16, generator=g).bfloat16(),
             "param::model.norm.weight": torch.randn(64, generator=g).bfloat16(),
             "model.layers.0.mlp.gate_proj_packed": torch.zeros(40, dtype=torch.uint8),
             "model.layers.0.mlp.gate_proj_meta": torch.tensor([8, 16])}
    out, counts = E.export_spark(state)
    assert counts == {"spfp2": 1, "fp3": 1, "nvfp4": 1}
    wq = state["param::model.layers.0.self_attn.q_proj.weight"].float().numpy()
    c, s = O.fp3_pack_3bit(O.fp3_fake_quant(wq))
    assert np.array_equal(out["model.layers.0.self_attn.q_proj_fp3_codes"].numpy(), c)
    assert np.array_equal(out["model.layers.0.self_attn.q_proj_fp3_scales"].view(torch.uint8).numpy(), s)
    wo = state["param::model.layers.0.self_attn.out_proj.weight"].float().numpy()
    c, s = O.nvfp4_pack(O.nvfp4_fake_quant(wo))
    assert np.array_equal(out["model.layers.0.self_attn.out_proj_nvfp4_codes"].numpy(), c)
    assert np.array_equal(out["model.layers.0.self_attn.out_proj_nvfp4_scales"].view(torch.uint8).numpy(), s)
    assert "param::model.layers.0.mlp.gate_proj.weight" not in out
    assert torch.equal(out["param::model.norm.weight"], state["param::model.norm.weight"])


def test_save_quantized_and_container_gpu(tmp_path):
    """save_quantized on a small QAT model, then the container round trip with
    the entries that run kernels (INT8 head, legacy NVFP4 values)."""
    from spark_b200 import quant_linear as ql
    from spark_b200 import export as E
    from spark_b200 import spark_v2_container as C
    from spark_b200.fp3_linear import FP3QATLinear
    torch.manual_seed(0)
    model = torch.nn.ModuleDict({
        "mlp": ql.ChannelFP2QATLinear(256, 128, bias=False),
        "attn": FP3QATLinear(256, 64, bias=False),
        "out_proj": ql.NVFP4QATLinear(64, 256, bias=False),
        "norm": torch.nn.LayerNorm(256),
    }).cuda()
    state, path = E.save_quantized(model, str(tmp_path), tag="t")
    assert state["mlp_meta"].tolist() == [128, 256]
    w = model["attn"].weight.detach().float().cpu().numpy()
    c, s = O.fp3_pack_3bit(w)
    assert np.array_equal(state["attn_fp3_codes"].numpy(), c)
    w = model["out_proj"].weight.detach().float().cpu().numpy()
    c, s = O.nvfp4_pack(O.nvfp4_fake_quant(w))
    assert np.array_equal(state["out_proj_nvfp4_codes"].numpy(), c)
    assert "param::norm.weight" in state and "param::mlp.weight" not in state
    # container: int8 head and a legacy NVFP4-values entry
    g = torch.Generator().manual_seed(5)
    head = torch.randn(32, 64, generator=g) * 0.05
    state["param::lm_head.weight"] = head.bfloat16()
    state["emb_nvfp4_weight"] = torch.from_numpy(O.nvfp4_fake_quant((torch.randn(16, 32, generator=g) * 0.02).numpy()))
    state["emb_meta"] = torch.tensor([16, 32])
    out = str(tmp_path / "c")
    C.save_spark_v2(state, out)
    back = C.load_spark_v2(out)
    q, sc = O.ptq_int8_pack(head.bfloat16().float().numpy())
    want = torch.from_numpy(q.astype(np.float32) * sc[:, None]).bfloat16()
    assert torch.equal(back["param::lm_head.weight"], want)
    c, s = O.nvfp4_pack(state["emb_nvfp4_weight"].numpy())
    assert np.array_equal(back["emb_nvfp4_codes"].numpy(), c)
    assert np.array_equal(back["emb_nvfp4_scales"].view(torch.uint8).numpy(), s)
    assert back["emb_meta"].tolist() == [16, 32]
    assert torch.equal(back["mlp_packed"], state["mlp_packed"])
