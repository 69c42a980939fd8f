"""Row-merged projections (V3MergedLinear): one packed weight for q/k/v or
gate/up, one launch; every part's output against an fp64 product with the
part's own decoded weight (5e-4 max-abs, fp32 activations) and against the
part's own layer."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 5e-4


def _part(fmt, oc, ic, seed):
    from spark_b200 import ops
    from spark_b200.inference_v3 import V3PackedLinear
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(oc, ic, device="cuda", generator=g) * 0.02
    b = torch.randn(oc, device="cuda", generator=g) * 0.1
    if fmt == "spfp2":
        wq, s = ops.spfp2_pack(w)[0], None
        deq = ops.spfp2_unpack(wq, oc * ic).view(oc, ic)
    elif fmt == "fp3":
        wq, s = ops.fp3_pack(w)
        deq = ops.fp3_unpack(wq, s, oc, ic)
    elif fmt == "nvfp4":
        wq, s = ops.nvfp4_pack(w)
        deq = ops.nvfp4_unpack(wq, s, oc, ic)
    else:
        wq, s = ops.twofour_pack(w), None
        deq = ops.twofour_unpack(wq, oc * ic).view(oc, ic)
    return V3PackedLinear(fmt, wq, oc, ic, scales=s, bias=b), deq, b


@pytest.mark.parametrize("fmt,ocs,ic", [("spfp2", (768, 768), 512), ("fp3", (512, 256, 256), 512),
                                        ("nvfp4", (256, 512), 512), ("twofour", (512, 256), 1024)])
@pytest.mark.parametrize("M", [1, 5, 300])
def test_merged_parts_match(fmt, ocs, ic, M):
    from spark_b200.inference_v3 import V3MergedLinear
    parts = [_part(fmt, oc, ic, seed=11 * k + 1) for k, oc in enumerate(ocs)]
    merged = V3MergedLinear([p for p, _, _ in parts])
    x = torch.randn(M, ic, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    outs = merged(x)
    assert len(outs) == len(ocs)
    for (layer, deq, b), y in zip(parts, outs):
        ref = x.double() @ deq.double().T + b.double()
        assert y.shape == (M, layer.out_features)
        assert (y.double() - ref).abs().max().item() <= TOL
        assert (y.double() - layer(x).double()).abs().max().item() <= TOL
    xb = x.bfloat16()
    for (layer, _, _), y in zip(parts, merged(xb)):
        assert y.dtype == torch.bfloat16
        assert torch.allclose(y.float(), layer(xb).float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_silu_mul_on_merged_halves(dtype):
    from spark_b200 import ops
    gu = torch.randn(37, 2 * 300, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3)).to(dtype)
    g, u = gu.split(300, dim=-1)
    out = ops.silu_mul(g, u)
    ref = torch.nn.functional.silu(g.float()) * u.float()
    assert out.shape == (37, 300) and out.is_contiguous()
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert torch.allclose(out.float(), ref, rtol=tol, atol=tol)
    assert torch.equal(out, ops.silu_mul(g.contiguous(), u.contiguous()))


def test_tp_mlp_single_rank_matches_fp64():
    from spark_b200 import ops
    from spark_b200.tp import TPMLP
    gen = torch.Generator(device="cuda").manual_seed(9)
    H, I = 512, 1024
    gate = torch.randn(I, H, device="cuda", generator=gen) * 0.05
    up = torch.randn(I, H, device="cuda", generator=gen) * 0.05
    down = torch.randn(H, I, device="cuda", generator=gen) * 0.05
    mlp = TPMLP(gate, up, down)
    x = torch.randn(64, H, device="cuda", generator=gen)
    dec = lambda w: ops.spfp2_unpack(ops.spfp2_pack(w)[0], w.numel()).view_as(w).double()
    h = torch.nn.functional.silu(x.double() @ dec(gate).T) * (x.double() @ dec(up).T)
    want = h @ dec(down).T
    got = mlp(x).double()
    assert (got - want).abs().max().item() <= 1e-3 * max(1.0, want.abs().max().item())


def test_prefetch_hint_changes_nothing():
    from spark_b200 import ops
    from spark_b200.inference_v3 import V3PackedLinear, chain_prefetch
    g = torch.Generator(device="cuda").manual_seed(2)
    a = V3PackedLinear("spfp2", ops.spfp2_pack(torch.randn(512, 768, device="cuda", generator=g) * 0.02)[0], 512, 768)
    b = V3PackedLinear("spfp2", ops.spfp2_pack(torch.randn(768, 512, device="cuda", generator=g) * 0.02)[0], 768, 512)
    x = torch.randn(3, 768, device="cuda", generator=g).bfloat16()
    want_a = a(x)
    want_b = b(want_a)
    chain_prefetch([a, b])
    assert a.prefetch_next is b.w_tiled and b.prefetch_next is a.w_tiled
    ya = a(x)
    assert torch.equal(ya, want_a) and torch.equal(b(ya), want_b)
    odd = torch.empty(1000, dtype=torch.uint8, device="cuda")      # length not a multiple of 16
    assert torch.equal(ops.linear("spfp2", a.w_tiled, None, x, 512, 768, tiled=True, prefetch=odd[:999]), want_a)


@pytest.mark.parametrize("fmt", ["spfp2", "fp3", "nvfp4"])
@pytest.mark.parametrize("M", [1, 7, 40])
def test_gate_up_silu_epilogue(fmt, M):
    from spark_b200.inference_v3 import V3GateUpSiLU
    (gate, _, _), (up, _, _) = _part(fmt, 512, 768, seed=3), _part(fmt, 512, 768, seed=4)
    fused = V3GateUpSiLU(gate, up)
    x = torch.randn(M, 768, device="cuda", generator=torch.Generator(device="cuda").manual_seed(8))
    want = torch.nn.functional.silu(gate(x).double()) * up(x).double()
    got = fused(x)
    assert got.shape == (M, 512) and got.dtype == torch.float32
    assert torch.allclose(got.double(), want, rtol=1e-4, atol=1e-5)
    xb = x.bfloat16()
    wb = torch.nn.functional.silu(gate(xb).float()) * up(xb).float()
    assert torch.allclose(fused(xb).float(), wb, rtol=3e-2, atol=3e-2)


def test_silu_epilogue_rejected_off_the_gemv():
    from spark_b200 import ops
    from spark_b200._lib import SparkError
    (gate, _, _) = _part("spfp2", 512, 768, seed=5)
    x = torch.randn(300, 768, device="cuda").bfloat16()
    with pytest.raises(SparkError):
        ops.linear("spfp2", gate.w_packed, None, x, 512, 768, silu=True)   # 300 tokens -> tcgen05 path
