"""2:4 linear on the sparse tensor cores (spark_twofour_sparse_linear,
tcgen05.mma.sp kind::f16): the kept values of every group of four and their
positions as the MMA's metadata.

Every kept weight is +-2^(e - 10) (exact in bf16) and x is bf16, so every
product is exact in fp32; against the fp64 product of x and the weights the
reference unpacker decodes (spark_twofour_unpack, bit-exact against the
golden vectors) the only difference is the fp32 accumulation, bounded by
K * 2^-23 of sum |x_k w_k| (plus 1e-6 relative).  A wrong metadata bit, a
swapped kept pair or a misplaced row breaks that bound by orders of
magnitude.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def ops():
    from spark_b200 import ops as o
    return o


def _case(M, oc, ic, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(oc, ic, generator=g) * 0.02).cuda()
    x = torch.randn(M, ic, generator=g).bfloat16().cuda()
    packed = ops().twofour_pack(w)
    wd = ops().twofour_unpack(packed, oc * ic).view(oc, ic).double()
    return x, packed, wd


def _check(y, x, wd, bias=None):
    ref = x.double() @ wd.T
    if bias is not None:
        ref = ref + bias.double()
    mag = x.double().abs() @ wd.abs().T
    bound = mag * (x.shape[1] * 2.0 ** -23 + 1e-6) + 1e-30
    err = (y.double() - ref).abs()
    assert bool((err <= bound).all()), float((err / (mag + 1e-30)).max())


@pytest.mark.parametrize("M,oc,ic", [(1, 128, 128), (77, 256, 512), (300, 384, 1024), (128, 2560, 9728)])
def test_sparse_matches_decoded_product(M, oc, ic):
    x, packed, wd = _case(M, oc, ic, seed=M + oc)
    y = ops().twofour_sparse_linear(packed, x, oc, ic, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops().check_device_errors()
    _check(y, x, wd)
    # and against the dense decode path on the same bytes (one accumulation order apart)
    yd = ops().linear("twofour", packed, None, x, oc, ic, out_dtype=torch.float32)
    _check(yd, x, wd)


def test_sparse_bias_and_bf16_output():
    M, oc, ic = 64, 256, 768
    x, packed, wd = _case(M, oc, ic, seed=9)
    bias = torch.randn(oc).cuda()
    y = ops().twofour_sparse_linear(packed, x, oc, ic, bias=bias, out_dtype=torch.float32)
    _check(y, x, wd, bias)
    yb = ops().twofour_sparse_linear(packed, x, oc, ic, bias=bias)
    assert yb.dtype == torch.bfloat16
    assert torch.equal(yb, y.bfloat16())
    ops().check_device_errors()


def test_sparse_rejects_bad_shapes():
    from spark_b200._lib import SparkError
    x, packed, _ = _case(4, 128, 128, seed=3)
    with pytest.raises(SparkError, match="multiple of 128"):
        ops().twofour_sparse_linear(packed, x[:, :96].contiguous(), 128, 96)
