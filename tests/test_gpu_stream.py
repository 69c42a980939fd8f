"""The batched decode kernel (spark_linear_batch, and spark_linear on tiled
weights with bf16 activations) against an fp64 accumulation of the
oracle-decoded weights.

Tolerance: max |y - y_ref| <= 5e-4 for fp32 output; for
activations scaled away from 1 the bound scales with max |y_ref| (relative
1e-5, the fp32 accumulation's own error at these sizes).  Up to 8 tokens every
format runs the f16 path (weights decoded to f16, activations converted once
per launch with a power-of-two scale per 256-column chunk); above 8 tokens and
for ops whose activations hold an inf or NaN, the bf16 path.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 5e-4


def ops():
    from spark_b200 import ops as _ops
    return _ops


def make(fmt, oc, ic, seed, std=0.02):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(oc, ic, generator=g) * std).cuda()
    if fmt == "spfp2":
        wq, s = ops().spfp2_pack(W)[0], None
        dec = O.unpack_blockwise_paired(wq.cpu().numpy(), oc * ic).reshape(oc, ic)
    elif fmt == "fp3":
        wq, s = ops().fp3_pack(W)
        dec = O.fp3_unpack_3bit(wq.cpu().numpy(), s.cpu().view(torch.uint8).numpy(), oc, ic)
    else:
        wq, s = ops().nvfp4_pack(W)
        dec = O.nvfp4_unpack(wq.cpu().numpy(), s.cpu().view(torch.uint8).numpy(), oc, ic)
    return wq, s, ops().tile_weights(fmt, wq, s, oc, ic), dec


def ref(x, dec, bias=None):
    return O.linear_f64(x.float().cpu().numpy(), dec, bias.float().cpu().numpy() if bias is not None else None)


SHAPES = [("spfp2", 9728, 2560), ("spfp2", 2560, 9728), ("fp3", 4096, 2560), ("nvfp4", 2560, 4096),
          ("spfp2", 1000, 768), ("fp3", 300, 512), ("nvfp4", 40, 2048)]


@pytest.mark.parametrize("fmt,oc,ic", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 16])
def test_single_linear(fmt, oc, ic, M):
    wq, s, wt, dec = make(fmt, oc, ic, seed=oc + ic + M)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, ic, generator=g).bfloat16().cuda()
    y = ops().linear(fmt, wt, None, x, oc, ic, out_dtype=torch.float32, tiled=True)
    torch.cuda.synchronize()
    err = np.abs(y.cpu().numpy() - ref(x, dec)).max()
    assert err <= TOL, (fmt, oc, ic, M, err)
    ops().check_device_errors()


@pytest.mark.parametrize("fmt", ["spfp2", "fp3", "nvfp4"])
def test_bias_and_output_dtypes(fmt):
    oc, ic = 1024, 1024
    wq, s, wt, dec = make(fmt, oc, ic, seed=5)
    g = torch.Generator().manual_seed(6)
    for M in (1, 4, 12):
        x = torch.randn(M, ic, generator=g).bfloat16().cuda()
        b = (torch.randn(oc, generator=g) * 0.1).cuda()
        y64 = ref(x, dec, b)
        for od in (torch.float32, torch.bfloat16, torch.float16):
            y = ops().linear(fmt, wt, None, x, oc, ic, bias=b, out_dtype=od, tiled=True).float().cpu().numpy()
            bound = TOL if od == torch.float32 else TOL + 2.0 ** -7 * np.abs(y64)
            assert np.all(np.abs(y - y64) <= bound), (fmt, M, od)


def test_spfp2_activation_range():
    """f16 path: the per-chunk power-of-two scale keeps the result at
    fp32-accumulation accuracy whatever the activations' magnitude, also with
    one large outlier per token."""
    oc, ic = 512, 2560
    wq, s, wt, dec = make("spfp2", oc, ic, seed=9)
    g = torch.Generator().manual_seed(10)
    for scale in (1e-6, 1e-2, 1.0, 3e4, 1e8):
        for M in (1, 3):
            x = torch.randn(M, ic, generator=g) * scale
            x[:, 7] = 1000.0 * scale                      # an outlier 3 decades above the rest
            x = x.bfloat16().cuda()
            y = ops().linear("spfp2", wt, None, x, oc, ic, out_dtype=torch.float32, tiled=True).cpu().numpy()
            y64 = ref(x, dec)
            rel = np.abs(y - y64).max() / max(np.abs(y64).max(), 1e-30)
            assert rel < 1e-5, (scale, M, rel)


def test_spfp2_nonfinite_activations():
    """A non-finite activation moves the op to the bf16 path: the result has the
    same NaN / inf pattern as the reference-layout linear, the rest matches."""
    oc, ic = 256, 1024
    wq, s, wt, dec = make("spfp2", oc, ic, seed=11)
    x = torch.randn(3, ic).bfloat16().cuda()
    x[0, 5] = float("inf")
    x[1, 9] = float("nan")              # token 2 stays finite
    y = ops().linear("spfp2", wt, None, x, oc, ic, out_dtype=torch.float32, tiled=True).cpu()
    y_ref = ops().linear("spfp2", wq, None, x, oc, ic, out_dtype=torch.float32).cpu()
    assert torch.equal(torch.isnan(y), torch.isnan(y_ref))
    assert torch.equal(torch.isinf(y), torch.isinf(y_ref))
    fin = torch.isfinite(y_ref)
    assert (y[fin] - y_ref[fin]).abs().max().item() <= TOL


def test_zero_activations():
    wq, s, wt, dec = make("spfp2", 256, 512, seed=12)
    x = torch.zeros(1, 512, dtype=torch.bfloat16, device="cuda")
    y = ops().linear("spfp2", wt, None, x, 256, 512, out_dtype=torch.float32, tiled=True)
    assert torch.count_nonzero(y).item() == 0


def test_repeat_calls_bit_identical():
    for fmt in ("spfp2", "fp3", "nvfp4"):
        wq, s, wt, dec = make(fmt, 2560, 9728 if fmt == "spfp2" else 4096, seed=13)
        ic = 9728 if fmt == "spfp2" else 4096
        x = torch.randn(2, ic).bfloat16().cuda()
        ys = [ops().linear(fmt, wt, None, x, 2560, ic, out_dtype=torch.float32, tiled=True) for _ in range(3)]
        assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2]), fmt


@pytest.mark.parametrize("M", [1, 4, 16])
def test_batch_independent_ops(M):
    """One launch over the projections of a config-2 layer (all formats), each
    op against its own fp64 reference."""
    specs = [("fp3", 12288, 2560), ("nvfp4", 2560, 4096), ("spfp2", 19456, 2560), ("spfp2", 2560, 9728)]
    g = torch.Generator().manual_seed(20 + M)
    batch, refs = [], []
    for i, (fmt, oc, ic) in enumerate(specs):
        wq, s, wt, dec = make(fmt, oc, ic, seed=100 + i)
        x = torch.randn(M, ic, generator=g).bfloat16().cuda()
        y = torch.empty(M, oc, dtype=torch.float32, device="cuda")
        batch.append(ops().BatchOp(fmt, wt, x, y))
        refs.append(ref(x, dec))
    ops().linear_batch(batch)
    torch.cuda.synchronize()
    for op, y64 in zip(batch, refs):
        assert np.abs(op.y.cpu().numpy() - y64).max() <= TOL
    ops().check_device_errors()


@pytest.mark.parametrize("M", [1, 3, 8])
def test_batch_dependent_chain(M):
    """gate|up (SiLU epilogue) -> down -> a second layer, each op reading the
    previous op's bf16 output; checked against the same sequence of separate
    spark_linear calls (identical kernels, identical results)."""
    H, I = 1024, 2048
    g = torch.Generator().manual_seed(30 + M)
    gate = (torch.randn(I, H, generator=g) * 0.02).cuda()
    up = (torch.randn(I, H, generator=g) * 0.02).cuda()
    down = (torch.randn(H, I, generator=g) * 0.02).cuda()
    w2 = (torch.randn(H, H, generator=g) * 0.02).cuda()
    from spark_b200.inference_v3 import V3GateUpSiLU, V3PackedLinear
    gu = V3GateUpSiLU(V3PackedLinear("spfp2", ops().spfp2_pack(gate)[0], I, H),
                      V3PackedLinear("spfp2", ops().spfp2_pack(up)[0], I, H))
    dn = V3PackedLinear("spfp2", ops().spfp2_pack(down)[0], H, I)
    c2, s2 = ops().nvfp4_pack(w2)
    l2 = V3PackedLinear("nvfp4", c2, H, H, scales=s2)
    x = torch.randn(M, H, generator=g).bfloat16().cuda()
    h = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
    z = torch.empty(M, H, dtype=torch.float32, device="cuda")
    batch = [ops().BatchOp("spfp2", gu.merged.w_tiled, x, h, silu=True),
             ops().BatchOp("spfp2", dn.w_tiled, h, y, deps=[0]),
             ops().BatchOp("nvfp4", l2.w_tiled, y, z, deps=[1])]
    for _ in range(2):                      # a repeated launch reuses the control block
        ops().linear_batch(batch)
    torch.cuda.synchronize()
    h_ref = gu(x)
    y_ref = dn(h_ref)
    z_ref = ops().linear("nvfp4", l2.w_tiled, None, y_ref, H, H, out_dtype=torch.float32, tiled=True)
    assert torch.equal(h, h_ref)
    assert torch.equal(y, y_ref)
    assert torch.equal(z, z_ref)
    ops().check_device_errors()


@pytest.mark.parametrize("M", [1, 5, 12])
def test_batch_fed_consumer(M):
    """An all-SPFP2 two-op batch (gate|up with the SiLU epilogue, then down
    reading its output) small enough to keep the bf16 path: the consumer waits
    only for the chunks of h it reads, as the producer's row groups complete.
    Checked bit for bit against the two ops as separate launches."""
    H, I = 1024, 4096
    g = torch.Generator().manual_seed(60 + M)
    from spark_b200.inference_v3 import V3GateUpSiLU, V3PackedLinear
    gate = (torch.randn(I, H, generator=g) * 0.02).cuda()
    up = (torch.randn(I, H, generator=g) * 0.02).cuda()
    down = (torch.randn(H, I, generator=g) * 0.02).cuda()
    gu = V3GateUpSiLU(V3PackedLinear("spfp2", ops().spfp2_pack(gate)[0], I, H),
                      V3PackedLinear("spfp2", ops().spfp2_pack(up)[0], I, H))
    dn = V3PackedLinear("spfp2", ops().spfp2_pack(down)[0], H, I)
    x = torch.randn(M, H, generator=g).bfloat16().cuda()
    h = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(M, H, dtype=torch.float32, device="cuda")
    batch = [ops().BatchOp("spfp2", gu.merged.w_tiled, x, h, silu=True),
             ops().BatchOp("spfp2", dn.w_tiled, h, y, deps=[0])]
    for _ in range(3):                      # the feed counters reset between launches
        ops().linear_batch(batch)
    torch.cuda.synchronize()
    h_ref = gu(x)
    y_ref = ops().linear("spfp2", dn.w_tiled, None, h_ref, H, I, out_dtype=torch.float32, tiled=True)
    assert torch.equal(h, h_ref)
    assert torch.equal(y, y_ref)
    ops().check_device_errors()


def test_batch_rejects_bad_ops():
    from spark_b200._lib import SparkError
    wq, s, wt, dec = make("spfp2", 256, 512, seed=40)
    x = torch.randn(1, 512).bfloat16().cuda()
    y = torch.empty(1, 256, dtype=torch.float32, device="cuda")
    with pytest.raises(SparkError, match="dep"):
        ops().linear_batch([ops().BatchOp("spfp2", wt, x, y, deps=[0])])
    with pytest.raises(TypeError):
        ops().linear_batch([ops().BatchOp("spfp2", wt, x.float(), y)])
    xm = torch.randn(17, 512).bfloat16().cuda()
    ym = torch.empty(17, 256, dtype=torch.float32, device="cuda")
    with pytest.raises(SparkError, match="M must be"):
        ops().linear_batch([ops().BatchOp("spfp2", wt, xm, ym)])


@pytest.mark.parametrize("M", [1, 8, 16])
def test_batch_long_chain_reuses_partial_areas(M):
    """Nine dependent ops (nine segments) at M = 1 / 8 / 16: at 8 and 16 tokens
    the partial-sum areas are fewer than the segments and are reused after a
    completion wait.  Checked against the same sequence of separate calls."""
    H = 2560
    g = torch.Generator().manual_seed(50 + M)
    fmts = ["spfp2", "fp3", "nvfp4"]
    layers = []
    for i in range(9):
        W = (torch.randn(H, H, generator=g) * 0.02).cuda()
        fmt = fmts[i % 3]
        if fmt == "spfp2":
            wq, s = ops().spfp2_pack(W)[0], None
        elif fmt == "fp3":
            wq, s = ops().fp3_pack(W)
        else:
            wq, s = ops().nvfp4_pack(W)
        layers.append((fmt, ops().tile_weights(fmt, wq, s, H, H)))
    x = torch.randn(M, H, generator=g).bfloat16().cuda()
    bufs = [x] + [torch.empty(M, H, dtype=torch.bfloat16, device="cuda") for _ in layers]
    batch = [ops().BatchOp(fmt, wt, bufs[i], bufs[i + 1], deps=[i - 1] if i else ())
             for i, (fmt, wt) in enumerate(layers)]
    for _ in range(2):
        ops().linear_batch(batch)
    torch.cuda.synchronize()
    y = x
    for i, (fmt, wt) in enumerate(layers):
        y = ops().linear(fmt, wt, None, y, H, H, out_dtype=torch.bfloat16, tiled=True)
        assert torch.equal(bufs[i + 1], y), (M, i)
    ops().check_device_errors()


def test_batch_mixed_paths():
    """One batch where one op's activations hold an inf (that op runs the bf16
    path) and the others are finite (f16 path): the same inf / NaN pattern as
    the op's own call, finite values within TOL of fp64."""
    specs = [("spfp2", 1024, 2560), ("fp3", 512, 2560), ("nvfp4", 768, 4096)]
    g = torch.Generator().manual_seed(61)
    batch, singles, refs = [], [], []
    for i, (fmt, oc, ic) in enumerate(specs):
        wq, s, wt, dec = make(fmt, oc, ic, seed=200 + i)
        x = torch.randn(2, ic, generator=g).bfloat16().cuda()
        if i == 1:
            x[0, 11] = float("inf")
        y = torch.empty(2, oc, dtype=torch.float32, device="cuda")
        batch.append(ops().BatchOp(fmt, wt, x, y))
        singles.append(ops().linear(fmt, wt, None, x, oc, ic, out_dtype=torch.float32, tiled=True))
        refs.append(ref(x, dec))
    ops().linear_batch(batch)
    torch.cuda.synchronize()
    for op, one, y64 in zip(batch, singles, refs):
        assert torch.equal(torch.isnan(op.y), torch.isnan(one)) and torch.equal(torch.isinf(op.y), torch.isinf(one))
        fin = torch.isfinite(one).cpu().numpy()
        assert np.abs(op.y.cpu().numpy()[fin] - y64[fin]).max() <= TOL
    ops().check_device_errors()


def test_weights_rewritten_in_place_before_the_call():
    """Tile new weights into the SAME buffer and call the linear right after,
    with nothing in between on the stream: the call must see the new weights
    (its weight prefetch runs before it waits for the previous kernel)."""
    from spark_b200 import ops as O2, _lib
    oc, ic = 1024, 2560
    wq_a, _, wt, dec_a = make("spfp2", oc, ic, seed=71)
    wq_b, _, _, dec_b = make("spfp2", oc, ic, seed=72)
    x = torch.randn(1, ic).bfloat16().cuda()
    y = torch.empty(1, oc, dtype=torch.float32, device="cuda")
    f = O2.FORMATS["spfp2"]
    for wq, dec in ((wq_b, dec_b), (wq_a, dec_a), (wq_b, dec_b)):
        _lib.call("spark_tile_weights", f, O2._p(O2._bytes(wq)), None, oc, ic, O2._p(wt), O2._stream(wt))
        O2.linear("spfp2", wt, None, x, oc, ic, out=y, tiled=True)
        torch.cuda.synchronize()
        assert np.abs(y.cpu().numpy() - ref(x, dec)).max() <= TOL
