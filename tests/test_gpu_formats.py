"""Pack / unpack / fake-quant kernels are bit-exact with the reference.

Golden vectors come from the reference emulators (tests/golden); larger
inputs are checked against the C oracle and, at BASELINE's full sizes,
against SHA-256 digests of the reference's own output bytes.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(G, name))


def ops():
    from spark_b200 import ops as _ops
    return _ops


def cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def host(t):
    t = t.detach().cpu()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    return t.numpy()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def same_bits(a, b):
    return np.array_equal(bits(a), bits(b))


def same_values(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return a.shape == b.shape and bool(np.all((a == b) | (np.isnan(a) & np.isnan(b))))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ----------------------------------------------------------------- SPFP2
def test_spfp2_golden_blocks():
    g = load("spfp2.npz")
    for w_key, p5_key, e_key, dec_key in (("adv_w", "adv_packed5", "adv_expv", "adv_dec"),
                                          ("odd_w", "odd_packed5", "odd_expv", "odd_dec")):
        w = cuda(g[w_key])
        p5, e = ops().spfp2_pack(w)
        assert np.array_equal(host(p5), g[p5_key]), w_key
        assert np.array_equal(host(e), g[e_key]), w_key
        assert same_bits(host(ops().spfp2_unpack(p5, w.numel())), g[dec_key]), w_key
    p3, _ = ops().spfp2_pack_v1(cuda(g["adv_w"]))
    assert np.array_equal(host(p3), g["adv_packed3"])
    assert same_bits(host(ops().spfp2_fake_quant(cuda(g["adv_w"]))), g["adv_fq"])
    assert same_bits(host(ops().spfp2_unpack(cuda(g["rnd5"]), 97 * 16)), g["rnd5_dec"])
    assert same_bits(host(ops().spfp2_unpack_v1(cuda(g["rnd3"]))), g["rnd3_dec"])


def test_spfp2_bf16_weights():
    g = load("spfp2.npz")
    wb = cuda(g["bf16_w"], torch.bfloat16)
    fq = ops().spfp2_fake_quant(wb, out_dtype=torch.float32)
    assert same_bits(host(fq), g["bf16_fq"])
    # bf16 output holds the same values exactly
    assert same_bits(host(ops().spfp2_fake_quant(wb).float()), g["bf16_fq"])


def test_spfp2_config1_full_size_matches_reference_digest():
    g = load("spfp2.npz")
    torch.manual_seed(0)
    W = torch.randn(9728, 2560) * 0.02
    Wc = W.cuda()
    p5, e = ops().spfp2_pack(Wc)
    assert sha(host(p5)) == str(g["cfg1_packed5_sha"])
    assert sha(host(e)) == str(g["cfg1_expv_sha"])
    assert sha(host(ops().spfp2_unpack(p5, W.numel()))) == str(g["cfg1_dec_sha"])
    p3, _ = ops().spfp2_pack_v1(Wc)
    assert sha(host(p3)) == str(g["cfg1_packed3_sha"])
    assert sha(host(ops().spfp2_fake_quant(Wc))) == str(g["cfg1_fq_sha"])


def test_spfp2_random_scales_vs_oracle():
    rng = np.random.default_rng(5)
    w = (rng.standard_normal(1 << 16) * np.exp(rng.standard_normal(1 << 16) * 3)).astype(np.float32)
    p5, e = ops().spfp2_pack(cuda(w))
    op5, oe = O.pack_blockwise_paired(w)
    assert np.array_equal(host(p5), op5) and np.array_equal(host(e), oe)
    assert same_bits(host(ops().spfp2_fake_quant(cuda(w))), O.channel_fake_quantize(w))


# ----------------------------------------------------------------- FP3 / NVFP4
@pytest.mark.parametrize("name", ["edge", "rnd", "rag"])
def test_fp3_golden(name):
    g = load("fp3_nvfp4.npz")
    w = cuda(g[f"fp3_{name}_w"])
    oc, ic = w.shape
    c3, s = ops().fp3_pack(w)
    assert np.array_equal(host(c3), g[f"fp3_{name}_c3"])
    assert np.array_equal(host(s), g[f"fp3_{name}_s"])
    cn, sn = ops().fp3_pack(w, nibble=True)
    assert np.array_equal(host(cn), g[f"fp3_{name}_cn"])
    assert same_bits(host(ops().fp3_unpack(c3, s, oc, ic)), g[f"fp3_{name}_dec3"])
    assert same_bits(host(ops().fp3_unpack(cn, sn, oc, ic, nibble=True)), g[f"fp3_{name}_decn"])
    assert same_values(host(ops().fp3_fake_quant(w)), g[f"fp3_{name}_fq"])


@pytest.mark.parametrize("name", ["edge", "rnd", "rag"])
def test_nvfp4_golden(name):
    g = load("fp3_nvfp4.npz")
    w = cuda(g[f"nvfp4_{name}_w"])
    oc, ic = w.shape
    c, s = ops().nvfp4_pack(w)
    assert np.array_equal(host(c), g[f"nvfp4_{name}_c"])
    assert np.array_equal(host(s), g[f"nvfp4_{name}_s"])
    assert same_bits(host(ops().nvfp4_unpack(c, s, oc, ic)), g[f"nvfp4_{name}_dec"])
    assert same_values(host(ops().nvfp4_fake_quant(w)), g[f"nvfp4_{name}_fq"])


def test_fp3_nvfp4_random_bytes_and_full_size():
    g = load("fp3_nvfp4.npz")
    assert same_bits(host(ops().fp3_unpack(cuda(g["rnd_fp3_c3"]), cuda(g["rnd_fp3_s"]), 5, 32)), g["rnd_fp3_dec3"])
    assert same_bits(host(ops().nvfp4_unpack(cuda(g["rnd_nvfp4_c"]), cuda(g["rnd_nvfp4_s"]), 5, 32)),
                     g["rnd_nvfp4_dec"])
    torch.manual_seed(1)
    Wq = (torch.randn(4096, 2560) * 0.02).cuda()
    Wo = (torch.randn(2560, 4096) * 0.02).cuda()
    c3, s3 = ops().fp3_pack(Wq)
    assert sha(host(c3)) == str(g["q_c3_sha"]) and sha(host(s3)) == str(g["q_s3_sha"])
    assert sha(host(ops().fp3_unpack(c3, s3, 4096, 2560))) == str(g["q_d3_sha"])
    c4, s4 = ops().nvfp4_pack(Wo)
    assert sha(host(c4)) == str(g["o_c4_sha"]) and sha(host(s4)) == str(g["o_s4_sha"])
    assert sha(host(ops().nvfp4_unpack(c4, s4, 2560, 4096))) == str(g["o_d4_sha"])


# ----------------------------------------------------------------- 2:4
@pytest.mark.parametrize("name", ["rnd", "rag", "edge"])
def test_two_four_golden(name):
    g = load("two_four.npz")
    w = cuda(g[f"{name}_w"])
    oc, ic = w.shape
    p = ops().twofour_pack(w)
    assert np.array_equal(host(p), g[f"{name}_packed"])
    n = oc * ((ic + 15) // 16) * 16
    assert same_bits(host(ops().twofour_unpack(p, n)), g[f"{name}_dec"])
    if f"{name}_fq" in g:
        assert same_bits(host(ops().twofour_fake_quant(w)), g[f"{name}_fq"])
    assert same_bits(host(ops().twofour_unpack(cuda(g["rnd_bytes"]), 33 * 32)), g["rnd_bytes_dec"])


def test_two_four_full_down_proj_vs_oracle():
    torch.manual_seed(5)
    W = torch.randn(2560, 9728) * 0.02
    p = ops().twofour_pack(W.cuda())
    assert np.array_equal(host(p), O.two_four_pack(W.numpy()))
    assert same_bits(host(ops().twofour_fake_quant(W.cuda())), O.two_four_fake_quant(W.numpy()))


# ----------------------------------------------------------------- INT8
def test_int8_golden_gpu():
    g = load("int8.npz")
    fq = host(ops().int8_fake_quant(cuda(g["w"])))
    assert same_values(fq, g["fq"])
    assert same_bits(fq[np.arange(24) != 6], g["fq"][np.arange(24) != 6])
    q, scale = ops().int8_pack(cuda(g["w_pack"]))
    assert np.array_equal(host(q), g["q"]) and same_bits(host(scale), g["scale"])
    assert same_bits(host(ops().int8_unpack(q, scale)), g["unpack"])
    wb = cuda(g["w_bf16_bits"]).view(torch.bfloat16)
    assert same_bits(host(ops().int8_fake_quant(wb)), g["fq_bf16_in"])


def test_int8_full_size_vs_oracle():
    gen = torch.Generator().manual_seed(12)
    w = torch.randn(2560, 4096, generator=gen) * 0.02
    fq = host(ops().int8_fake_quant(w.cuda()))
    assert same_bits(fq, O.int8_fake_quant(w.numpy()))
