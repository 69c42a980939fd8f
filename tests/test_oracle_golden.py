"""The C oracle reproduces the reference emulators bit for bit.

Golden vectors come from tests/golden/make_golden.py, which ran DJAzzs/SPARK's
own emulators (01_core/block_fp2_emu.py, fp3_emu.py, nvfp4_emu.py,
two_four.py).  Full-size configurations are checked through SHA-256 digests of
the reference's output bytes on regenerated seeded inputs.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

G = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(G, name))


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def same_bits(a, b):
    """Bitwise float equality (NaN payloads included, -0.0 != +0.0)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    assert a.shape == b.shape, (a.shape, b.shape)
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


def same_values(a, b):
    """torch.equal semantics extended to NaN == NaN (sign of zero ignored)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return a.shape == b.shape and bool(np.all((a == b) | (np.isnan(a) & np.isnan(b))))


# ----------------------------------------------------------------- thresholds
def test_center_thresholds_match_torch_log2():
    """The window centre boundaries equal torch.log2's rounding, re-derived live."""
    t = load("thresholds.npz")["center_t"]
    assert np.array_equal(t, O.center_thresholds())
    for k, tb in enumerate(t, start=1):
        bits = np.arange(int(tb) - 64, int(tb) + 64, dtype=np.uint32)
        m = torch.from_numpy(bits.view(np.float32).copy())
        c = (torch.log2(m) + 10.0 - 0.75).round().long().clamp(0, 15).numpy()
        want = np.where(bits >= tb, k, k - 1)
        assert np.array_equal(c, want), k
        assert all(O.spfp2_center(float(v)) == w for v, w in zip(m[::16].tolist(), want[::16]))


def test_center_specials():
    assert O.spfp2_center(float("inf")) == 0
    assert O.spfp2_center(float("nan")) == 0
    assert O.spfp2_center(1e-38) == 0
    assert O.spfp2_center(1e38) == 15


# ----------------------------------------------------------------- SPFP2
def test_spfp2_config1_full_size_digests():
    torch.manual_seed(0)
    W = (torch.randn(9728, 2560) * 0.02).numpy()
    g = load("spfp2.npz")
    p5, e = O.pack_blockwise_paired(W)
    assert sha(p5) == str(g["cfg1_packed5_sha"])
    assert sha(e) == str(g["cfg1_expv_sha"])
    dec = O.unpack_blockwise_paired(p5, W.size)
    assert sha(dec) == str(g["cfg1_dec_sha"])
    p3, _ = O.pack_blockwise_search(W)
    assert sha(p3) == str(g["cfg1_packed3_sha"])
    fq = O.channel_fake_quantize(W)
    assert sha(fq) == str(g["cfg1_fq_sha"])


def test_spfp2_config1_rows_and_gemv():
    g = load("spfp2.npz")
    w = g["cfg1_rows_w"]
    p5, _ = O.pack_blockwise_paired(w)
    assert np.array_equal(p5, g["cfg1_rows_packed5"])
    assert same_bits(O.unpack_blockwise_paired(p5, w.size), g["cfg1_rows_dec"])
    # the reference's CPU linear (x.float() @ Wdeq.T) against fp64 accumulation
    x = g["cfg1_x"]
    y64 = O.linear_f64(x, g["cfg1_rows_dec"].reshape(16, 2560))
    assert np.max(np.abs(y64 - g["cfg1_y"][:, :16])) < 5e-5


def test_spfp2_adversarial_blocks():
    g = load("spfp2.npz")
    w = g["adv_w"]
    p5, e = O.pack_blockwise_paired(w)
    assert np.array_equal(p5, g["adv_packed5"])
    assert np.array_equal(e, g["adv_expv"])
    p3, _ = O.pack_blockwise_search(w)
    assert np.array_equal(p3, g["adv_packed3"])
    assert same_bits(O.unpack_blockwise_paired(p5, w.size), g["adv_dec"])
    assert same_bits(O.channel_fake_quantize(w), g["adv_fq"])


def test_spfp2_odd_blocks_and_random_bytes():
    g = load("spfp2.npz")
    p5, e = O.pack_blockwise_paired(g["odd_w"])
    assert np.array_equal(p5, g["odd_packed5"]) and np.array_equal(e, g["odd_expv"])
    assert same_bits(O.unpack_blockwise_paired(p5, g["odd_w"].size), g["odd_dec"])
    assert same_bits(O.unpack_blockwise_paired(g["rnd5"], 97 * 16), g["rnd5_dec"])
    assert same_bits(O.unpack_blockwise(g["rnd3"]), g["rnd3_dec"])


def test_spfp2_fake_quant_bf16_weights():
    g = load("spfp2.npz")
    assert same_bits(O.channel_fake_quantize(g["bf16_w"]), g["bf16_fq"])


# ----------------------------------------------------------------- FP8 / FP3 / NVFP4
def test_e4m3_decode_all_bytes():
    g = load("fp3_nvfp4.npz")
    assert same_bits(O.e4m3_to_f32(np.arange(256)), g["e4m3_all_f32"])


def test_e4m3_encode_sweep():
    g = load("fp3_nvfp4.npz")
    assert np.array_equal(O.f32_to_e4m3(g["e4m3_sweep_x"]), g["e4m3_sweep_b"])


@pytest.mark.parametrize("name", ["edge", "rnd", "rag"])
def test_fp3_pack_unpack_fake_quant(name):
    g = load("fp3_nvfp4.npz")
    w = g[f"fp3_{name}_w"]
    oc, ic = w.shape
    c3, s = O.fp3_pack_3bit(w)
    assert np.array_equal(c3, g[f"fp3_{name}_c3"])
    assert np.array_equal(s, g[f"fp3_{name}_s"])
    cn, sn = O.fp3_pack(w)
    assert np.array_equal(cn, g[f"fp3_{name}_cn"])
    assert same_bits(O.fp3_unpack_3bit(c3, s, oc, ic), g[f"fp3_{name}_dec3"])
    assert same_bits(O.fp3_unpack(cn, sn, oc, ic), g[f"fp3_{name}_decn"])
    assert same_values(O.fp3_fake_quant(w), g[f"fp3_{name}_fq"])


@pytest.mark.parametrize("name", ["edge", "rnd", "rag"])
def test_nvfp4_pack_unpack_fake_quant(name):
    g = load("fp3_nvfp4.npz")
    w = g[f"nvfp4_{name}_w"]
    oc, ic = w.shape
    c, s = O.nvfp4_pack(w)
    assert np.array_equal(c, g[f"nvfp4_{name}_c"])
    assert np.array_equal(s, g[f"nvfp4_{name}_s"])
    assert same_bits(O.nvfp4_unpack(c, s, oc, ic), g[f"nvfp4_{name}_dec"])
    assert same_values(O.nvfp4_fake_quant(w), g[f"nvfp4_{name}_fq"])


def test_fp3_nvfp4_random_bytes():
    g = load("fp3_nvfp4.npz")
    assert same_bits(O.fp3_unpack_3bit(g["rnd_fp3_c3"], g["rnd_fp3_s"], 5, 32), g["rnd_fp3_dec3"])
    assert same_bits(O.nvfp4_unpack(g["rnd_nvfp4_c"], g["rnd_nvfp4_s"], 5, 32), g["rnd_nvfp4_dec"])


def test_fp3_nvfp4_config2_full_size_digests():
    g = load("fp3_nvfp4.npz")
    torch.manual_seed(1)
    Wq = (torch.randn(4096, 2560) * 0.02).numpy()
    Wo = (torch.randn(2560, 4096) * 0.02).numpy()
    c3, s3 = O.fp3_pack_3bit(Wq)
    assert sha(c3) == str(g["q_c3_sha"]) and sha(s3) == str(g["q_s3_sha"])
    assert sha(O.fp3_unpack_3bit(c3, s3, 4096, 2560)) == str(g["q_d3_sha"])
    c4, s4 = O.nvfp4_pack(Wo)
    assert sha(c4) == str(g["o_c4_sha"]) and sha(s4) == str(g["o_s4_sha"])
    assert sha(O.nvfp4_unpack(c4, s4, 2560, 4096)) == str(g["o_d4_sha"])


# ----------------------------------------------------------------- 2:4
@pytest.mark.parametrize("name", ["rnd", "rag", "edge"])
def test_two_four_pack_unpack(name):
    g = load("two_four.npz")
    w = g[f"{name}_w"]
    oc, ic = w.shape
    p = O.two_four_pack(w)
    assert np.array_equal(p, g[f"{name}_packed"])
    n = oc * ((ic + 15) // 16) * 16
    assert same_bits(O.two_four_unpack(p, n), g[f"{name}_dec"])
    if f"{name}_fq" in g:
        assert same_bits(O.two_four_fake_quant(w), g[f"{name}_fq"])


def test_two_four_random_bytes():
    g = load("two_four.npz")
    assert same_bits(O.two_four_unpack(g["rnd_bytes"], 33 * 32), g["rnd_bytes_dec"])


# ----------------------------------------------------------------- INT8
def test_int8_golden():
    """int8_emu (lm_head tier): fake-quant incl. a NaN row, PTQ pack / unpack."""
    g = load("int8.npz")
    assert same_values(O.int8_fake_quant(g["w"]), g["fq"])
    assert same_bits(O.int8_fake_quant(g["w"])[np.arange(24) != 6], g["fq"][np.arange(24) != 6])
    q, scale = O.ptq_int8_pack(g["w_pack"])
    assert np.array_equal(q, g["q"]) and same_bits(scale, g["scale"])
    assert same_bits(q.astype(np.float32) * scale[:, None], g["unpack"])
    wb = torch.from_numpy(g["w_bf16_bits"]).view(torch.bfloat16).float().numpy()
    assert same_bits(O.int8_fake_quant(wb), g["fq_bf16_in"])
