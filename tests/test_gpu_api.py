"""The drop-in Python API on the GPU: STE fake-quant forward/backward, the QAT
layer caches, the packed inference forwards, model rewriting and the
checkpoint loaders, against the oracle (bit-exact fake-quant / decode) and an
fp64 reference for the linears (5e-4 max-abs, fp32 activations)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
from torch import nn

from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = 5e-4


def mods():
    from spark_b200 import block_fp2, fp3, fp3_linear, int8, nvfp4, quant_linear, spark_loader, two_four
    return block_fp2, fp3, fp3_linear, int8, nvfp4, quant_linear, spark_loader, two_four


def rnd(*shape, seed=0, scale=0.02, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(device)


@pytest.mark.parametrize("name", ["channel", "fp3", "nvfp4", "two_four", "int8"])
def test_ste_forward_backward(name):
    block_fp2, fp3, _, int8, nvfp4, _, _, two_four = mods()
    fn, ref, dtype_out = {
        "channel": (block_fp2.channel_fake_quantize, O.channel_fake_quantize, "same"),
        "fp3": (fp3.fp3_fake_quant_ste, O.fp3_fake_quant, torch.float32),
        "nvfp4": (nvfp4.nvfp4_fake_quant_ste, O.nvfp4_fake_quant, torch.float32),
        "two_four": (two_four.two_four_fake_quant, O.two_four_fake_quant, "same"),
        "int8": (int8.int8_fake_quant_ste, O.int8_fake_quant, torch.float32),
    }[name]
    w = rnd(96, 256, seed=1).bfloat16().requires_grad_(True)
    y = fn(w)
    assert y.dtype == (w.dtype if dtype_out == "same" else dtype_out)
    want = ref(w.detach().float().cpu().numpy())
    assert np.array_equal(y.detach().float().cpu().numpy().view(np.uint32), want.astype(np.float32).view(np.uint32))
    g = torch.randn_like(y)
    y.backward(g)
    assert torch.equal(w.grad.float(), g.float().to(w.grad.dtype).float())      # straight through
    # without grad: fp32 round trip, as the reference
    y0 = fn(w.detach())
    assert y0.dtype == torch.float32


def test_qat_layers_forward_backward_and_cache():
    _, _, fp3_linear, _, _, ql, _, _ = mods()
    x = rnd(4, 128, seed=2, scale=1.0).requires_grad_(True)
    for cls, fq in [(ql.ChannelFP2QATLinear, O.channel_fake_quantize), (fp3_linear.FP3QATLinear, O.fp3_fake_quant),
                    (ql.NVFP4QATLinear, O.nvfp4_fake_quant), (ql.TwoFourQATLinear, O.two_four_fake_quant),
                    (ql.INT8QATLinear, O.int8_fake_quant)]:
        layer = cls(128, 64, bias=True, device="cuda")
        with torch.no_grad():
            layer.weight.copy_(rnd(64, 128, seed=3))
            layer.bias.copy_(rnd(64, seed=4, scale=0.1))
        layer.train()
        y = layer(x)
        wq = torch.from_numpy(fq(layer.weight.detach().cpu().numpy())).cuda()
        assert (y - (x @ wq.T + layer.bias)).abs().max().item() < 1e-5, cls.__name__
        y.sum().backward()
        assert torch.allclose(layer.weight.grad, torch.ones(4, 64, device="cuda").T @ x.detach()), cls.__name__
        # cached until the shared version moves (w + (Wq - w) equals Wq up to fp32 rounding)
        with torch.no_grad():
            layer.weight.add_(0.01)
        assert (layer(x) - y).abs().max().item() < 1e-5, cls.__name__
        ql.bump_wq_version()
        assert (layer(x) - y).abs().max().item() > 1e-3, cls.__name__
        x.grad = None


@pytest.mark.parametrize("ic", [256, 100])
def test_channel_fp2_linear_packed_forward(ic):
    _, _, _, _, _, ql, _, _ = mods()
    layer = ql.ChannelFP2Linear(ic, 96, bias=True, device="cuda")
    with torch.no_grad():
        layer.weight.copy_(rnd(96, ic, seed=5))
        layer.bias.copy_(rnd(96, seed=6, scale=0.1))
    layer.quantize()
    ic_p = (ic + 7) // 8 * 8
    w_pad = np.zeros((96, ic_p), np.float32)
    w_pad[:, :ic] = layer.weight.detach().cpu().numpy()
    packed, _ = O.pack_blockwise_paired(w_pad)
    assert np.array_equal(layer._packed_weight.cpu().numpy(), packed)
    dec = O.unpack_blockwise_paired(packed, 96 * ic_p).reshape(96, ic_p)[:, :ic]
    assert np.array_equal(ql.decode_layer_weight(layer).numpy(), dec)
    for M in (1, 20):
        x = rnd(M, ic, seed=7 + M, scale=1.0)
        y = layer(x).double().cpu().numpy()
        y64 = O.linear_f64(x.cpu().numpy(), dec, layer.bias.detach().cpu().numpy())
        assert np.abs(y - y64).max() <= TOL


@pytest.mark.parametrize("ic", [256, 100])
def test_fp2_linear_packed_forward(ic):
    _, _, _, _, _, ql, _, _ = mods()
    layer = ql.FP2Linear(ic, 64, bias=False, device="cuda")
    with torch.no_grad():
        layer.weight.copy_(rnd(64, ic, seed=8))
    layer.quantize()
    dec = ql.decode_layer_weight(layer).numpy()
    x = rnd(3, ic, seed=9, scale=1.0)
    y = layer(x).double().cpu().numpy()
    assert np.abs(y - O.linear_f64(x.cpu().numpy(), dec)).max() <= TOL


def test_qat_quantize_then_eval_uses_packed_bytes():
    _, _, _, _, _, ql, _, _ = mods()
    layer = ql.ChannelFP2QATLinear(512, 256, bias=False, device="cuda")
    with torch.no_grad():
        layer.weight.copy_(rnd(256, 512, seed=10))
    layer.quantize()
    layer.eval()
    x = rnd(2, 512, seed=11, scale=1.0).bfloat16()
    y = layer(x)
    assert y.dtype == torch.bfloat16
    dec = ql.decode_layer_weight(layer).numpy()
    y64 = O.linear_f64(x.float().cpu().numpy(), dec)
    assert np.all(np.abs(y.float().cpu().numpy() - y64) <= TOL + 2.0 ** -8 * np.abs(y64))


class _Toy(nn.Module):
    def __init__(self):
        super().__init__()
        self.embed_tokens = nn.Embedding(64, 32)
        self.layers = nn.ModuleList([nn.ModuleDict({
            "mlp": nn.ModuleDict({"gate_proj": nn.Linear(32, 64), "down_proj": nn.Linear(64, 32)}),
            "self_attn": nn.ModuleDict({"q_proj": nn.Linear(32, 32), "o_proj": nn.Linear(32, 32)}),
        })])
        self.lm_head = nn.Linear(32, 64, bias=False)
        self.lm_head.weight = self.embed_tokens.weight


def test_apply_mixed_quant_tiers_and_tied_head():
    _, _, fp3_linear, _, _, ql, _, _ = mods()
    m = ql.apply_mixed_quant(_Toy().cuda(), quantize_head=True, fp3_tier=True)
    L = m.layers[0]
    assert isinstance(L["mlp"]["gate_proj"], ql.ChannelFP2QATLinear)
    assert isinstance(L["self_attn"]["q_proj"], fp3_linear.FP3QATLinear)
    assert isinstance(m.embed_tokens, ql.NVFP4EmbeddingQAT)
    assert isinstance(m.lm_head, ql.NVFP4QATLinear) and m.lm_head.weight is m.embed_tokens.weight
    m2 = ql.apply_mixed_quant(_Toy().cuda(), v3=True)
    assert isinstance(m2.layers[0]["mlp"]["down_proj"], ql.TwoFourQATLinear)
    assert isinstance(m2.layers[0]["self_attn"]["o_proj"], ql.NVFP4QATLinear)
    assert isinstance(m2.lm_head, nn.Linear)
    m.train()
    ids = torch.randint(0, 64, (2, 5), device="cuda")
    out = m.embed_tokens(ids)
    wq = torch.from_numpy(O.nvfp4_fake_quant(m.embed_tokens.weight.detach().cpu().numpy())).cuda()
    assert torch.equal(out, wq[ids])


def _state():
    """A SPARK-style state dict: SPFP2 (row-padded), FP3 3-bit and nibble,
    NVFP4, a param:: entry."""
    _, fp3, _, _, nvfp4, ql, _, _ = mods()
    st, w = {}, {}
    w["a"] = rnd(64, 100, seed=20)
    lay = ql.ChannelFP2Linear(100, 64, device="cuda")
    with torch.no_grad():
        lay.weight.copy_(w["a"])
    lay.quantize()
    st["a_packed"], st["a_meta"] = lay._packed_weight.cpu(), torch.tensor([64, 100])
    w["b"] = rnd(32, 256, seed=21)
    st["b_fp3_codes"], st["b_fp3_scales"] = [t.cpu() for t in fp3.fp3_pack_3bit(w["b"])]
    st["b_meta"] = torch.tensor([32, 256])
    w["c"] = rnd(48, 256, seed=22)
    st["c_fp3_codes"], st["c_fp3_scales"] = [t.cpu() for t in fp3.fp3_pack(w["c"])]
    st["c_meta"] = torch.tensor([48, 256])
    w["d"] = rnd(40, 512, seed=23)
    st["d_nvfp4_codes"], st["d_nvfp4_scales"] = [t.cpu() for t in nvfp4.nvfp4_pack(w["d"])]
    st["d_meta"] = torch.tensor([40, 512])
    st["param::norm.weight"] = torch.full((16,), 2.0)
    return st, w


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.a, self.b, self.c, self.d = nn.Linear(100, 64), nn.Linear(256, 32), nn.Linear(256, 48), nn.Linear(512, 40)
        self.norm = nn.LayerNorm(16)


def test_apply_spark_state_and_resident_variant(tmp_path):
    _, _, _, _, _, ql, spark_loader, _ = mods()
    st, w = _state()
    net = _Net()
    n1, n2, n3 = spark_loader.apply_spark_state(net, st)
    assert (n1, n2, n3) == (1, 3, 1)
    wa = np.zeros((64, 104), np.float32)
    wa[:, :100] = w["a"].cpu().numpy()
    assert np.array_equal(net.a.weight.detach().numpy(),
                          O.unpack_blockwise_paired(O.pack_blockwise_paired(wa)[0], 64 * 104).reshape(64, 104)[:, :100])
    assert np.array_equal(net.b.weight.detach().numpy(), O.fp3_unpack_3bit(*O.fp3_pack_3bit(w["b"].cpu().numpy()), 32, 256))
    assert np.array_equal(net.c.weight.detach().numpy(), O.fp3_unpack(*O.fp3_pack(w["c"].cpu().numpy()), 48, 256))
    assert np.array_equal(net.d.weight.detach().numpy(), O.nvfp4_unpack(*O.nvfp4_pack(w["d"].cpu().numpy()), 40, 512))
    assert torch.equal(net.norm.weight, torch.full((16,), 2.0))
    # packed-resident: same outputs from the codes kept on the GPU
    res = _Net().cuda()
    n_layers, n_param = spark_loader.apply_spark_state_resident(res, st)
    assert (n_layers, n_param) == (4, 1)
    for name, ic in (("a", 100), ("b", 256), ("c", 256), ("d", 512)):
        x = rnd(3, ic, seed=30, scale=1.0)
        y = getattr(res, name)(x).double().cpu().numpy()
        y64 = O.linear_f64(x.cpu().numpy(), getattr(net, name).weight.detach().numpy())
        assert np.abs(y - y64).max() <= TOL, name
    # SparkWeightLoader on a state_dict.pt directory
    torch.save(st, os.path.join(tmp_path, "state_dict.pt"))
    sd = spark_loader.SparkWeightLoader(str(tmp_path)).state_dict()
    assert list(sd) == ["a.weight"] and sd["a.weight"].dtype == torch.float16
    assert torch.equal(sd["a.weight"], net.a.weight.detach().half())
