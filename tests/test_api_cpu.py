"""The drop-in Python API (mirrors of quant_linear.py, fp3_linear.py,
spark_loader.py and the four emulators): names, format detection, tier
assignment and the shared fake-quant version, without a GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from oracle import oracle as O
from spark_b200 import block_fp2, fp3, fp3_linear, int8, nvfp4, quant_linear as ql, spark_loader, two_four
from spark_b200.inference_v3 import fp3_nibbles_to_3bit

REFERENCE_NAMES = {
    ql: ["quantize_tensor_blockwise", "_detect_format", "_unpack_weight", "FP2Linear", "ChannelFP2Linear",
         "bump_wq_version", "ChannelFP2QATLinear", "apply_channel_fp2_qat", "decode_layer_weight",
         "apply_channel_fp2_quant", "set_force_fake_quant", "NVFP4QATLinear", "TwoFourQATLinear", "INT8QATLinear",
         "NVFP4EmbeddingQAT", "apply_mixed_quant", "FP3QATLinear", "ELEMS_PER_BLOCK"],
    fp3_linear: ["FP3QATLinear"],
    spark_loader: ["SparkWeightLoader", "load_spark_model", "apply_spark_state"],
    block_fp2: ["pack_blockwise_search", "pack_blockwise_paired", "unpack_blockwise", "unpack_blockwise_paired",
                "ChannelFP2STE", "channel_fake_quantize", "ELEMS_PER_BLOCK", "BYTES_PER_BLOCK", "BYTES_PER_PAIR"],
    fp3: ["fp3_fake_quant", "fp3_pack", "fp3_unpack", "fp3_pack_3bit", "fp3_unpack_3bit", "FP3STE",
          "fp3_fake_quant_ste"],
    nvfp4: ["nvfp4_fake_quant", "nvfp4_pack", "nvfp4_unpack", "NVFP4STE", "nvfp4_fake_quant_ste"],
    two_four: ["two_four_pack", "two_four_unpack", "two_four_fake_quant", "TwoFourSTE"],
    int8: ["int8_fake_quant", "INT8STE", "int8_fake_quant_ste", "ptq_int8_pack", "ptq_int8_unpack"],
}


@pytest.mark.parametrize("mod", list(REFERENCE_NAMES), ids=lambda m: m.__name__)
def test_reference_names_present(mod):
    missing = [n for n in REFERENCE_NAMES[mod] if not hasattr(mod, n)]
    assert not missing, missing


def test_constants():
    assert (block_fp2.ELEMS_PER_BLOCK, block_fp2.BYTES_PER_BLOCK, block_fp2.BYTES_PER_PAIR) == (8, 3, 5)
    assert two_four.BYTES_PER_PAIR == 7 and fp3.ELEMS_PER_BLOCK == 16 and nvfp4.ELEMS_PER_BLOCK == 16


def test_detect_format():
    assert ql._detect_format(3 * 4, 32) == "v1"
    assert ql._detect_format(5 * 2, 32) == "v2"
    assert ql._detect_format(5 * 4, 56) == "v2"        # odd block count: padded pair
    # 5 blocks take 15 bytes either way; like the reference, the 3-byte layout wins
    assert ql._detect_format(15, 40) == "v1"
    with pytest.raises(ValueError):
        ql._detect_format(7, 32)


def test_single_wq_version_counter():
    v = fp3_linear._WQ_VERSION[0]
    ql.bump_wq_version()
    assert fp3_linear._WQ_VERSION[0] == v + 1 and ql._WQ_VERSION is fp3_linear._WQ_VERSION


def test_mixed_quant_tiers():
    t = ql._tier
    assert t("model.layers.0.mlp.gate_proj", False, False, False) == "spfp2"
    assert t("model.layers.0.mlp.down_proj", True, False, False) == "twofour"
    assert t("model.layers.0.self_attn.q_proj", False, False, False) == "nvfp4"
    assert t("model.layers.0.self_attn.q_proj", False, True, False) == "fp3"
    assert t("model.layers.0.linear_attn.in_proj_ba", False, True, False) == "spfp2"
    assert t("model.layers.0.linear_attn.out_proj", False, True, False) == "nvfp4"
    assert t("model.layers.0.self_attn.o_proj", False, True, True) == "fp3"
    assert t("model.layers.0.self_attn.k_proj", False, True, True) == "spfp2"


def test_set_force_fake_quant_counts():
    m = nn.Sequential(fp3_linear.FP3QATLinear(16, 16), nn.Linear(16, 16))
    assert ql.set_force_fake_quant(m, True) == 1 and m[0].force_fake_quant


def test_fp3_nibbles_to_3bit_matches_oracle():
    w = np.random.RandomState(3).randn(6, 80).astype(np.float32) * 0.02   # ragged: ic % 16 != 0
    c3, _ = O.fp3_pack_3bit(w)
    cn, _ = O.fp3_pack(w)
    n = 6 * 96
    assert np.array_equal(fp3_nibbles_to_3bit(torch.from_numpy(cn), n).numpy(), c3)


def test_merged_linear_concatenates_rows_and_rejects_straddling_rows():
    from spark_b200.inference_v3 import V3MergedLinear, V3PackedLinear
    g = torch.Generator().manual_seed(0)
    a = torch.randint(0, 256, (64 * 512 // 16 * 5,), dtype=torch.uint8, generator=g)
    b = torch.randint(0, 256, (32 * 512 // 16 * 5,), dtype=torch.uint8, generator=g)
    m = V3MergedLinear([V3PackedLinear("spfp2", a, 64, 512), V3PackedLinear("spfp2", b, 32, 512)])
    assert m.splits == [64, 32] and m.merged.out_features == 96 and m.in_features == 512
    assert torch.equal(m.merged.w_packed, torch.cat([a, b]))
    c = torch.randint(0, 256, (16 * 104 // 16 * 5,), dtype=torch.uint8, generator=g)
    with pytest.raises(ValueError):
        V3MergedLinear([V3PackedLinear("spfp2", c, 16, 104), V3PackedLinear("spfp2", c, 16, 104)])
    with pytest.raises(ValueError):
        V3MergedLinear([V3PackedLinear("spfp2", a, 64, 512), V3PackedLinear("twofour", a, 64, 512)])


def test_chain_prefetch_links_layers_in_call_order():
    from spark_b200.inference_v3 import V3MergedLinear, V3NVFP4Embedding, V3PackedLinear, chain_prefetch
    g = torch.Generator().manual_seed(1)
    mk = lambda oc, ic: V3PackedLinear("spfp2", torch.randint(0, 256, (oc * ic // 16 * 5,), dtype=torch.uint8,
                                                              generator=g), oc, ic)
    a, b, c = mk(64, 256), mk(32, 256), mk(256, 64)
    m = V3MergedLinear([a, b])
    chain_prefetch([m, c])
    # CPU layers keep no tiled copy: the hint falls back to the packed bytes
    assert m.merged.prefetch_next is c.w_packed and c.prefetch_next is m.merged.w_packed
    emb = V3NVFP4Embedding(torch.zeros(10, 8, dtype=torch.uint8), torch.zeros(10, 1, dtype=torch.uint8), 10, 16,
                           padding_idx=3)
    assert emb.codes.dtype == torch.uint8 and emb.padding_idx == 3 and "nvfp4" in emb.extra_repr()


def test_gate_up_silu_interleaves_rows_in_groups_of_eight():
    from spark_b200.inference_v3 import V3GateUpSiLU, V3PackedLinear
    inter, ic = 24, 64
    rb, sb = ic // 2, ic // 16                                      # NVFP4 row bytes, scale bytes
    g = torch.Generator().manual_seed(3)
    gc, uc = (torch.randint(0, 256, (inter * rb,), dtype=torch.uint8, generator=g) for _ in range(2))
    gs, us = (torch.randint(0, 256, (inter * sb,), dtype=torch.uint8, generator=g) for _ in range(2))
    gb, ub = torch.randn(inter, generator=g), torch.randn(inter, generator=g)
    m = V3GateUpSiLU(V3PackedLinear("nvfp4", gc, inter, ic, scales=gs, bias=gb),
                     V3PackedLinear("nvfp4", uc, inter, ic, scales=us, bias=ub))
    assert m.out_features == inter and m.merged.out_features == 2 * inter
    rows = m.merged.w_packed.view(2 * inter, rb)
    srows = m.merged.w_scales.view(2 * inter, sb)
    for k in range(inter // 8):
        for i in range(8):
            assert torch.equal(rows[16 * k + i], gc.view(inter, rb)[8 * k + i])
            assert torch.equal(rows[16 * k + 8 + i], uc.view(inter, rb)[8 * k + i])
            assert torch.equal(srows[16 * k + 8 + i], us.view(inter, sb)[8 * k + i])
            assert m.merged.bias[16 * k + i] == gb[8 * k + i] and m.merged.bias[16 * k + 8 + i] == ub[8 * k + i]
    with pytest.raises(ValueError):
        V3GateUpSiLU(V3PackedLinear("nvfp4", gc[: 12 * rb], 12, ic, scales=gs[: 12 * sb]),
                     V3PackedLinear("nvfp4", uc[: 12 * rb], 12, ic, scales=us[: 12 * sb]))
