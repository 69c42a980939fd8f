"""spark_linear (decode GEMV / GEMM) against an fp64 accumulation of the
oracle-decoded weights.  Tolerance: max |y - y_ref| <= 5e-4 for fp32 output
bf16 output within its own rounding (2^-8 relative)."""
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
    """Pack a seeded weight on the GPU; return (wq, scales, W_decoded_by_oracle)."""
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(oc, ic, generator=g) * std
    Wc = W.cuda()
    if fmt == "spfp2":
        wq, _ = ops().spfp2_pack(Wc)
        dec = O.unpack_blockwise_paired(wq.cpu().numpy(), oc * ic).reshape(oc, ic)
        return wq, None, dec
    if fmt == "spfp2_v1":
        wq, _ = ops().spfp2_pack_v1(Wc)
        dec = O.unpack_blockwise(wq.cpu().numpy()).reshape(oc, ic)
        return wq, None, dec
    if fmt == "fp3":
        wq, s = ops().fp3_pack(Wc)
        dec = O.fp3_unpack_3bit(wq.cpu().numpy(), s.cpu().view(torch.uint8).numpy(), oc, ic)
        return wq, s, dec
    if fmt == "nvfp4":
        wq, s = ops().nvfp4_pack(Wc)
        dec = O.nvfp4_unpack(wq.cpu().numpy(), s.cpu().view(torch.uint8).numpy(), oc, ic)
        return wq, s, dec
    if fmt == "twofour":
        wq = ops().twofour_pack(Wc)
        n = oc * ((ic + 15) // 16) * 16
        dec = O.two_four_unpack(wq.cpu().numpy(), n).reshape(oc, -1)[:, :ic]
        return wq, None, np.ascontiguousarray(dec)
    raise ValueError(fmt)


def check(fmt, oc, ic, M, seed=0, bias=False, out_dtype=torch.float32, x_dtype=torch.bfloat16, tiled=False):
    wq, s, dec = make(fmt, oc, ic, seed)
    if tiled:
        wq, s = ops().tile_weights(fmt, wq, s, oc, ic), None
        assert wq is not None
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(M, ic, generator=g).to(x_dtype)
    b = (torch.randn(oc, generator=g) * 0.1) if bias else None
    y = ops().linear(fmt, wq, s, x.cuda(), oc, ic, bias=b.cuda() if b is not None else None, out_dtype=out_dtype,
                     tiled=tiled)
    torch.cuda.synchronize()
    y64 = O.linear_f64(x.float().numpy(), dec, b.numpy() if b is not None else None)
    err = np.abs(y.float().cpu().numpy().astype(np.float64) - y64)
    if out_dtype == torch.float32:
        assert err.max() <= TOL, (fmt, oc, ic, M, err.max())
    else:
        assert np.all(err <= TOL + 2.0 ** -8 * np.abs(y64)), (fmt, oc, ic, M, err.max())
    ops().check_device_errors()


FAST = [("spfp2", 9728, 2560), ("spfp2", 2560, 9728), ("fp3", 4096, 2560), ("nvfp4", 2560, 4096),
        ("twofour", 2560, 9728), ("spfp2", 12288, 4096), ("fp3", 512, 1024), ("nvfp4", 1000, 768)]


@pytest.mark.parametrize("fmt,oc,ic", FAST)
@pytest.mark.parametrize("M", [1, 4, 16])
def test_linear_fast_path(fmt, oc, ic, M):
    check(fmt, oc, ic, M)


@pytest.mark.parametrize("fmt,oc,ic", FAST)
@pytest.mark.parametrize("M", [1, 4, 16])
def test_linear_tiled(fmt, oc, ic, M):
    check(fmt, oc, ic, M, tiled=True)


@pytest.mark.parametrize("fmt", ["spfp2", "fp3", "nvfp4", "twofour"])
def test_linear_tiled_chunks_bias_dtypes(fmt):
    check(fmt, 1024, 1024, 17, bias=True, tiled=True)
    if fmt == "spfp2":
        # the tiled SPFP2 layout takes bf16 activations only
        from spark_b200._lib import SparkError
        for xd in (torch.float32, torch.float16):
            with pytest.raises(SparkError, match="bf16"):
                check(fmt, 1024, 1024, 3, seed=4, x_dtype=xd, tiled=True)
        return
    check(fmt, 1024, 1024, 3, seed=4, x_dtype=torch.float32, bias=True, tiled=True)
    check(fmt, 1000, 1024, 5, seed=6, x_dtype=torch.float16, out_dtype=torch.float16, tiled=True)


@pytest.mark.parametrize("fmt", ["spfp2", "fp3", "nvfp4", "twofour"])
def test_linear_token_chunks_bias_dtypes(fmt):
    oc, ic = (1024, 1024)
    check(fmt, oc, ic, 17, bias=True)
    check(fmt, oc, ic, 40, seed=3, out_dtype=torch.bfloat16)
    check(fmt, oc, ic, 3, seed=4, x_dtype=torch.float32, bias=True)
    check(fmt, oc, ic, 5, seed=6, x_dtype=torch.float16, out_dtype=torch.float16)


@pytest.mark.parametrize("fmt,oc,ic", [("spfp2", 5, 24), ("spfp2", 12, 48), ("spfp2", 7, 40), ("spfp2_v1", 16, 256),
                                       ("fp3", 7, 40), ("nvfp4", 7, 40), ("twofour", 5, 40), ("fp3", 33, 100)])
def test_linear_generic_path(fmt, oc, ic):
    check(fmt, oc, ic, 1)
    check(fmt, oc, ic, 9, seed=2, bias=True)


def test_linear_activation_range():
    """Large and tiny activations: the per-token power-of-two scaling keeps fp16 exact."""
    wq, s, dec = make("spfp2", 256, 1024, 9)
    g = torch.Generator().manual_seed(10)
    for scale in (1e-6, 1.0, 3e4, 1e8):
        x = (torch.randn(3, 1024, generator=g) * scale).bfloat16()
        y = ops().linear("spfp2", wq, None, x.cuda(), 256, 1024, out_dtype=torch.float32).cpu().numpy()
        y64 = O.linear_f64(x.float().numpy(), dec)
        rel = np.abs(y - y64).max() / max(np.abs(y64).max(), 1e-30)
        assert rel < 1e-5, (scale, rel)
