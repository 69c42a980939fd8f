"""Native NVFP4 x NVFP4 linear (spark_nvfp4_native_linear, tcgen05.mma
kind::mxf4nvf4): a reported mode beside the parity path.

1. Against the exact product of the two dequantised operands (both packs
   decoded by spark_nvfp4_unpack, fp64 matmul): every product of two e2m1
   codes and two e4m3 scales is exact in fp32, so the only difference is the
   fp32 accumulation; the bound is K * 2^-23 of sum |x_k w_k| (plus 1e-6
   relative), far below any layout or scale mistake.
2. Against the parity path (bf16 x times the decoded weights): the measured
   relative Frobenius error is the activations' FP4 rounding, about 0.094 for
   N(0, 1) activations (the oracle's quantiser on the CPU gives 0.094 too);
   pinned below 0.12.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def ops():
    from spark_b200 import ops as o
    return o


@pytest.mark.parametrize("M,oc,ic", [(1, 128, 256), (37, 256, 512), (300, 384, 1024), (128, 128, 4096)])
def test_native_matches_dequantised_product(M, oc, ic):
    g = torch.Generator().manual_seed(M * 7 + oc)
    w = (torch.randn(oc, ic, generator=g) * 0.02).cuda()
    x = torch.randn(M, ic, generator=g).bfloat16().cuda()
    wc, wsc = ops().nvfp4_pack(w)
    xc, xsc = ops().nvfp4_pack(x)
    y = ops().nvfp4_native_linear(wc, wsc, x, oc, ic, out_dtype=torch.float32, xq=(xc, xsc))
    torch.cuda.synchronize()
    ops().check_device_errors()
    wd = ops().nvfp4_unpack(wc, wsc, oc, ic).double()
    xd = ops().nvfp4_unpack(xc, xsc, M, ic).double()
    ref = xd @ wd.T
    mag = xd.abs() @ wd.abs().T
    bound = mag * (ic * 2.0 ** -23 + 1e-6) + 1e-30
    err = (y.double() - ref).abs()
    assert bool((err <= bound).all()), float((err / (mag + 1e-30)).max())


def test_native_error_against_parity_path():
    M, oc, ic = 256, 512, 2048
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(oc, ic, generator=g) * 0.02).cuda()
    x = torch.randn(M, ic, generator=g).bfloat16().cuda()
    wc, wsc = ops().nvfp4_pack(w)
    y_nat = ops().nvfp4_native_linear(wc, wsc, x, oc, ic, out_dtype=torch.float32).double()
    wd = ops().nvfp4_unpack(wc, wsc, oc, ic).double()
    y_par = x.double() @ wd.T
    rel = float((y_nat - y_par).norm() / y_par.norm())
    assert 0.05 < rel < 0.12, rel
    ops().check_device_errors()


def test_native_rejects_bad_shapes():
    from spark_b200._lib import SparkError
    w = torch.randn(100, 256).cuda()
    wc, wsc = ops().nvfp4_pack(w)
    with pytest.raises(SparkError, match="multiple of 128"):
        ops().nvfp4_native_linear(wc, wsc, torch.randn(4, 256).bfloat16().cuda(), 100, 256)
