"""The tcgen05 linear (A = decoded weights in tensor memory, B = x in
shared memory, fp32 accumulation in tensor memory) against an fp64
accumulation of the oracle-decoded weights: max |y - y_ref| <= 5e-4 for fp32
output (bf16 output within its own rounding).  Covers the decode shape
(M <= 16, stream-K split with partial sums), every token tile (16, 64, 128,
256), ragged row blocks and several token tiles."""
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


def pack(fmt, W):
    if fmt == "spfp2":
        return ops().spfp2_pack(W)[0], None
    if fmt == "twofour":
        return ops().twofour_pack(W), None
    if fmt == "fp3":
        return ops().fp3_pack(W)
    return ops().nvfp4_pack(W)


def oracle_decode(fmt, wq, s, oc, ic):
    if fmt == "spfp2":
        return O.unpack_blockwise_paired(wq.cpu().numpy(), oc * ic).reshape(oc, ic)
    if fmt == "twofour":
        return O.two_four_unpack(wq.cpu().numpy(), oc * ic).reshape(oc, ic)
    sb = s.cpu().view(torch.uint8).numpy()
    if fmt == "fp3":
        return O.fp3_unpack_3bit(wq.cpu().numpy(), sb, oc, ic)
    return O.nvfp4_unpack(wq.cpu().numpy(), sb, oc, ic)


def run(oc, ic, M, seed=0, bias=False, out_dtype=torch.float32, fmt="spfp2"):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(oc, ic, generator=g) * 0.02
    wq, s = pack(fmt, W.cuda())
    x = torch.randn(M, ic, generator=g).bfloat16()
    b = (torch.randn(oc, generator=g) * 0.1) if bias else None
    y = ops().linear(fmt, wq, s, x.cuda(), oc, ic, bias=b.cuda() if b is not None else None,
                     out_dtype=out_dtype, tcgen05=True)
    torch.cuda.synchronize()
    ops().check_device_errors()
    return wq, s, x, b, y


def check_oracle(oc, ic, M, fmt="spfp2", **kw):
    wq, s, x, b, y = run(oc, ic, M, fmt=fmt, **kw)
    dec = oracle_decode(fmt, wq, s, oc, ic)
    y64 = O.linear_f64(x.float().numpy(), dec, b.numpy() if b is not None else None)
    err = np.abs(y.float().cpu().numpy().astype(np.float64) - y64)
    if y.dtype == torch.float32:
        assert err.max() <= TOL, (oc, ic, M, err.max())
    else:
        assert np.all(err <= TOL + 2.0 ** -8 * np.abs(y64)), (oc, ic, M, err.max())


@pytest.mark.parametrize("oc,ic", [(9728, 2560), (2560, 9728), (256, 256), (1000, 512), (130, 768)])
@pytest.mark.parametrize("M", [1, 4, 16])
def test_tc_decode_shapes(oc, ic, M):
    check_oracle(oc, ic, M)


@pytest.mark.parametrize("M", [17, 64, 100, 128, 200, 256, 300, 520])
def test_tc_token_tiles(M):
    check_oracle(1000, 1024, M, seed=M)


@pytest.mark.parametrize("fmt", ["fp3", "nvfp4"])
@pytest.mark.parametrize("oc,ic,M", [(4096, 2560, 1), (2560, 4096, 16), (1000, 512, 3), (640, 768, 64),
                                     (1000, 1024, 300), (130, 256, 200)])
def test_tc_scaled_formats(fmt, oc, ic, M):
    check_oracle(oc, ic, M, fmt=fmt, seed=oc + M)


@pytest.mark.parametrize("oc,ic,M", [(2560, 9728, 1), (2560, 9728, 16), (1000, 1024, 3), (640, 1536, 64),
                                     (1000, 512, 300), (130, 512, 200)])
def test_tc_twofour(oc, ic, M):
    check_oracle(oc, ic, M, fmt="twofour", seed=oc + M)


@pytest.mark.parametrize("fmt", ["fp3", "nvfp4"])
def test_tc_scaled_formats_bias_bf16(fmt):
    check_oracle(512, 512, 40, fmt=fmt, bias=True, out_dtype=torch.bfloat16)


def test_tc_bias_bf16_out():
    check_oracle(2560, 2560, 3, bias=True, out_dtype=torch.bfloat16)
    check_oracle(2560, 2560, 3, bias=True)
    check_oracle(640, 512, 300, bias=True, out_dtype=torch.bfloat16)


def test_tc_repeat_calls_bit_identical():
    """Stream-K partial sums are added in CTA order: repeated calls agree bit for bit."""
    g = torch.Generator().manual_seed(5)
    W = (torch.randn(9728, 2560, generator=g) * 0.02).cuda()
    wq, _ = ops().spfp2_pack(W)
    x = torch.randn(4, 2560, generator=g).bfloat16().cuda()
    ys = [ops().linear("spfp2", wq, None, x, 9728, 2560, out_dtype=torch.float32, tcgen05=True) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(ys[0], t) for t in ys[1:])


@pytest.mark.parametrize("fmt,oc,ic", [("spfp2", 9728, 2560), ("spfp2", 2560, 9728), ("fp3", 4096, 2560),
                                       ("nvfp4", 2560, 4096), ("twofour", 2560, 9728)])
def test_tc_prefill_full_size(fmt, oc, ic):
    """Config-3 shapes (M = 2048) against an fp64 GEMM of the GPU-decoded weights
    (decode is bit-exact against the oracle, tests/test_gpu_formats.py)."""
    M = 2048
    g = torch.Generator(device="cuda").manual_seed(11)
    W = torch.randn(oc, ic, device="cuda", generator=g) * 0.02
    wq, s = pack(fmt, W)
    x = torch.randn(M, ic, device="cuda", generator=g).bfloat16()
    y = ops().linear(fmt, wq, s, x, oc, ic, out_dtype=torch.float32, tcgen05=True)
    if fmt == "spfp2":
        Wd = ops().spfp2_unpack(wq, oc * ic).view(oc, ic).double()
    elif fmt == "twofour":
        Wd = ops().twofour_unpack(wq, oc * ic).view(oc, ic).double()
    elif fmt == "fp3":
        Wd = ops().fp3_unpack(wq, s, oc, ic).view(oc, ic).double()
    else:
        Wd = ops().nvfp4_unpack(wq, s, oc, ic).view(oc, ic).double()
    y64 = x.double() @ Wd.T
    err = (y.double() - y64).abs().max().item()
    assert err <= TOL, err
    ops().check_device_errors()


def test_tc_rejects_unsupported():
    from spark_b200 import _lib
    wq, _ = ops().spfp2_pack(torch.randn(256, 200, device="cuda"))   # ic % 256 != 0
    with pytest.raises(_lib.SparkError) as e:
        ops().linear("spfp2", wq, None, torch.randn(1, 200, device="cuda").bfloat16(), 256, 200, tcgen05=True)
    assert e.value.code == _lib.ERR_UNSUPPORTED


@pytest.mark.parametrize("fmt", ["spfp2", "fp3", "nvfp4", "twofour"])
def test_tc_activation_range(fmt):
    """bf16 x enters the tensor core unscaled: products are exact at any magnitude."""
    oc, ic, M = 256, 1024, 40
    g = torch.Generator().manual_seed(21)
    if fmt == "twofour":
        ic = 1024
    wq, s = pack(fmt, (torch.randn(oc, ic, generator=g) * 0.02).cuda())
    dec = oracle_decode(fmt, wq, s, oc, ic)
    for scale in (1e-6, 1.0, 3e4, 1e8):
        x = (torch.randn(M, ic, generator=g) * scale).bfloat16()
        y = ops().linear(fmt, wq, s, x.cuda(), oc, ic, out_dtype=torch.float32).cpu().numpy()
        y64 = O.linear_f64(x.float().numpy(), dec)
        rel = np.abs(y - y64).max() / max(np.abs(y64).max(), 1e-30)
        assert rel < 1e-5, (fmt, scale, rel)


@pytest.mark.parametrize("oc,ic", [(1536, 4096), (4096, 1536), (12288, 4096)])
def test_tc_config4_shapes_m64(oc, ic):
    """Config-4 shards at M = 64: 64-token stream-K with partial sums."""
    check_oracle(oc, ic, 64, seed=oc)
