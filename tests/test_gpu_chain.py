"""spark_linear_chain: one persistent launch running a config-2 layer as the
model does it -- q/k/v (FP3) on x, out_proj (NVFP4) on q's output, gate/up
(SPFP2) on out's output, SiLU(gate) * up, down (SPFP2) -- and a second layer
on the first one's output.  Every linear is checked against an fp64
accumulation of the oracle-decoded weights applied to the input that op
actually read (tolerance 5e-4 + bf16 output rounding); SiLU within bf16
rounding of a float64 evaluation."""
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


def packed(fmt, oc, ic, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.randn(oc, ic, device="cuda", generator=g) * 0.02
    if fmt == "spfp2":
        wq, s = ops().spfp2_pack(W)[0], None
        dec = O.unpack_blockwise_paired(wq.cpu().numpy(), oc * ic).reshape(oc, ic)
    elif fmt == "fp3":
        wq, s = ops().fp3_pack(W)
        dec = O.fp3_unpack_3bit(wq.cpu().numpy(), s.cpu().view(torch.uint8).numpy(), oc, ic)
    else:
        wq, s = ops().nvfp4_pack(W)
        dec = O.nvfp4_unpack(wq.cpu().numpy(), s.cpu().view(torch.uint8).numpy(), oc, ic)
    return wq, s, dec


def layer_ops(x, seed, M, layers_base):
    """ops for one layer reading x; returns (ops, outputs dict, weights dict)."""
    C = ops().ChainOp
    dev = x.device
    H, I, A = 2560, 9728, 4096
    W = {n: packed(f, oc, ic, seed + i) for i, (n, f, oc, ic) in enumerate(
        [("q", "fp3", A, H), ("k", "fp3", A, H), ("v", "fp3", A, H), ("o", "nvfp4", H, A),
         ("gate", "spfp2", I, H), ("up", "spfp2", I, H), ("down", "spfp2", H, I)])}
    Y = {n: torch.full((M, W[n][2].shape[0]), float("nan"), device=dev, dtype=torch.bfloat16) for n in W}
    Y["h"] = torch.full((M, I), float("nan"), device=dev, dtype=torch.bfloat16)
    b = layers_base
    L = [C("linear", x, Y["q"], "fp3", W["q"][0], W["q"][1], deps=[b - 1] if b else []),
         C("linear", x, Y["k"], "fp3", W["k"][0], W["k"][1], deps=[b - 1] if b else []),
         C("linear", x, Y["v"], "fp3", W["v"][0], W["v"][1], deps=[b - 1] if b else []),
         C("linear", Y["q"], Y["o"], "nvfp4", W["o"][0], W["o"][1], deps=[b]),
         C("linear", Y["o"], Y["gate"], "spfp2", W["gate"][0], deps=[b + 3]),
         C("linear", Y["o"], Y["up"], "spfp2", W["up"][0], deps=[b + 3]),
         C("silu_mul", Y["gate"], Y["h"], x2=Y["up"], deps=[b + 4, b + 5]),
         C("linear", Y["h"], Y["down"], "spfp2", W["down"][0], deps=[b + 6])]
    return L, Y, W


def check_linear(xin, y, dec):
    y64 = O.linear_f64(xin.float().cpu().numpy(), dec)
    err = np.abs(y.float().cpu().numpy() - y64)
    assert np.all(err <= TOL + 2.0 ** -8 * np.abs(y64)), err.max()


@pytest.mark.parametrize("M", [1, 4, 16])
def test_chain_two_layers(M):
    g = torch.Generator(device="cuda").manual_seed(M)
    x = torch.randn(M, 2560, device="cuda", generator=g).bfloat16()
    L1, Y1, W1 = layer_ops(x, 100, M, 0)
    L2, Y2, W2 = layer_ops(Y1["down"], 200, M, 8)
    for _ in range(2):                      # twice: counters and done flags reset between launches
        ops().linear_chain(L1 + L2)
        torch.cuda.synchronize()
    ops().check_device_errors()
    for (Y, W, xin) in ((Y1, W1, x), (Y2, W2, Y1["down"])):
        check_linear(xin, Y["q"], W["q"][2])
        check_linear(xin, Y["k"], W["k"][2])
        check_linear(xin, Y["v"], W["v"][2])
        check_linear(Y["q"], Y["o"], W["o"][2])
        check_linear(Y["o"], Y["gate"], W["gate"][2])
        check_linear(Y["o"], Y["up"], W["up"][2])
        gg, uu = Y["gate"].double().cpu().numpy(), Y["up"].double().cpu().numpy()
        h64 = gg / (1.0 + np.exp(-gg)) * uu
        assert np.all(np.abs(Y["h"].double().cpu().numpy() - h64) <= 1e-6 + 2.0 ** -7 * np.abs(h64))
        check_linear(Y["h"], Y["down"], W["down"][2])
