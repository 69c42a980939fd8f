"""spark_linear_noalloc (static scratch, no workspace argument) against
spark_linear with a caller-provided workspace, through the C ABI.

Tolerance: max |y_noalloc - y_linear| <= 5e-4 (the linear's own bound; both
run the same kernels, so in practice they agree bit for bit).  Each case makes
two calls in a row with different activations, so stale scratch contents from
the first call would show in the second.  This file is collected last so it
also runs after every other GPU test has used the library in the process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from spark_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 5e-4
DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def ops():
    from spark_b200 import ops as _ops
    return _ops


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _args(fmt, wq, s, x, b, y, oc, ic):
    return (fmt, _ptr(wq), _ptr(s), _ptr(x), DT[x.dtype], x.shape[0], oc, ic, x.stride(0), _ptr(b),
            DT[b.dtype] if b is not None else 0, _ptr(y), DT[y.dtype], y.stride(0))


def run_linear(fmt, wq, s, x, b, y, oc, ic):
    n = ops().workspace_size(fmt, x.shape[0], oc, ic)
    ws = ops().workspace(x.device, n)
    _lib.call("spark_linear", *_args(fmt, wq, s, x, b, y, oc, ic), _ptr(ws), n, _stream())


def run_noalloc(fmt, wq, s, x, b, y, oc, ic):
    _lib.call("spark_linear_noalloc", *_args(fmt, wq, s, x, b, y, oc, ic), _stream())


def weights(name, oc, ic, tiled, seed):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(oc, ic, generator=g) * 0.02).cuda()
    if name == "spfp2":
        wq, s = ops().spfp2_pack(W)[0], None
    elif name == "fp3":
        wq, s = ops().fp3_pack(W)
    elif name == "twofour":
        wq, s = ops().twofour_pack(W), None
    else:
        wq, s = ops().nvfp4_pack(W)
    fmt = ops().FORMATS[name]
    if tiled:
        wq, s = ops().tile_weights(name, wq, s, oc, ic), None
        fmt |= _lib.LAYOUT_TILED
    return fmt, wq, s


CASES = [
    # name, oc, ic, M, tiled, x dtype, y dtype, bias
    ("spfp2", 9728, 2560, 1, True, torch.bfloat16, torch.float32, False),   # bf16 MMA, no prepared x
    ("fp3", 4096, 2560, 20, False, torch.float32, torch.float32, False),    # prepared hi/lo x, two token chunks
    ("nvfp4", 2560, 4096, 4, True, torch.bfloat16, torch.bfloat16, True),   # prepared x, bias, bf16 out
    # the tcgen05 GEMM route: bf16 x on the reference layout above 16 tokens,
    # and 2:4 at every token count (its stream-K partials live in the scratch)
    ("spfp2", 4096, 2560, 64, False, torch.bfloat16, torch.float32, False),
    ("fp3", 2560, 4096, 300, False, torch.bfloat16, torch.bfloat16, True),
    ("twofour", 2560, 9728, 4, False, torch.bfloat16, torch.float32, False),
]


@pytest.mark.parametrize("name,oc,ic,M,tiled,xd,yd,bias", CASES)
def test_noalloc_matches_linear(name, oc, ic, M, tiled, xd, yd, bias):
    fmt, wq, s = weights(name, oc, ic, tiled, seed=oc + ic)
    g = torch.Generator().manual_seed(M)
    b = (torch.randn(oc, generator=g) * 0.1).cuda() if bias else None
    for call in range(2):
        x = torch.randn(M, ic, generator=g).to(xd).cuda()
        y_ref = torch.empty(M, oc, dtype=yd, device="cuda")
        y = torch.full((M, oc), float("nan"), dtype=yd, device="cuda")
        run_linear(fmt, wq, s, x, b, y_ref, oc, ic)
        run_noalloc(fmt, wq, s, x, b, y, oc, ic)
        torch.cuda.synchronize()
        err = (y.float() - y_ref.float()).abs().max().item()
        assert err <= TOL, (name, call, err)
    ops().check_device_errors()


def test_noalloc_allocates_nothing():
    fmt, wq, s = weights("spfp2", 2560, 2560, True, seed=7)
    x = torch.randn(1, 2560, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(1, 2560, dtype=torch.float32, device="cuda")
    run_noalloc(fmt, wq, s, x, None, y, 2560, 2560)     # first call on the device: set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        run_noalloc(fmt, wq, s, x, None, y, 2560, 2560)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_oversized_ic():
    p = ctypes.c_void_p(256)
    rc = _lib.lib().spark_linear_noalloc(0, p, None, p, _lib.DTYPE_BF16, 1, 16, 1 << 20, 1 << 20, None, 0, p,
                                         _lib.DTYPE_F32, 16, None)
    assert rc == _lib.ERR_WORKSPACE
    msg = _lib.last_error()
    assert "spark_linear_noalloc" in msg and "static" in msg, msg
