"""Generate the golden vectors that pin the oracle to the reference emulators.

Run where a checkout of the DJAzzs/SPARK tree is readable, naming its root
in ``SPARK_REFERENCE`` or as the first argument::

    python tests/golden/make_golden.py <path to the SPARK checkout>

It imports the reference's own emulators (``01_core/block_fp2_emu.py``,
``fp3_emu.py``, ``nvfp4_emu.py``, ``two_four.py``) read-only, runs them on
seeded inputs and writes ``tests/golden/*.npz``.  Full-size outputs that are
too large to commit are stored as SHA-256 digests of their bytes; the tests
regenerate the same inputs with torch's seeded CPU generator and compare the
oracle's output digests.  Nothing at test time imports the reference.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPARK_REFERENCE", "")
if not os.path.isdir(os.path.join(REF, "01_core")):
    sys.exit("make_golden.py: pass the SPARK checkout's root (it holds 01_core/) as the first argument "
             "or in SPARK_REFERENCE")
sys.path.insert(0, os.path.join(REF, "01_core"))

import block_fp2_emu as fp2  # noqa: E402
import fp3_emu  # noqa: E402
import nvfp4_emu  # noqa: E402
import two_four  # noqa: E402
import int8_emu  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
META = dict(torch_version=torch.__version__,
            cpu_capability=torch.backends.cpu.get_cpu_capability())

# exact centre thresholds measured against torch.log2 (see test_oracle_golden)
CENTER_T = [0x3b1837f4, 0x3b9837ef, 0x3c1837f2, 0x3c9837ef, 0x3d1837f2, 0x3d9837ee,
            0x3e1837f3, 0x3e9837ed, 0x3f1837f4, 0x3f9837ed, 0x401837f5, 0x409837ed,
            0x411837f5, 0x419837ec, 0x421837f6]


def sha(t) -> str:
    a = t.detach().cpu().contiguous().numpy() if isinstance(t, torch.Tensor) else np.ascontiguousarray(t)
    return hashlib.sha256(a.tobytes()).hexdigest()


def f32(bits: int) -> float:
    return float(np.array([bits], np.uint32).view(np.float32)[0])


def npy(t):
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.detach().cpu().contiguous().numpy().copy()


def save(name, **arrs):
    path = os.path.join(OUT, name)
    np.savez_compressed(path, **arrs, **{f"meta_{k}": np.array(v) for k, v in META.items()})
    print(f"wrote {path} ({os.path.getsize(path)} B)")


# --------------------------------------------------------------------------
def spfp2_adversarial(gen) -> torch.Tensor:
    """8-blocks aimed at every decision boundary of the window search."""
    blocks = []
    # centre thresholds +-2 ulp, with random smaller companions
    for t in CENTER_T:
        for d in (-2, -1, 0, 1, 2):
            m = f32(t + d)
            b = (torch.rand(8, generator=gen) * 2 - 1) * m
            b[int(torch.randint(0, 8, (1,), generator=gen))] = m * (1 if d % 2 else -1)
            blocks.append(b)
    # candidate ties: |w| exactly s/2 for several exponents
    for e in range(16):
        s = 2.0 ** (e - 10)
        blocks.append(torch.tensor([s / 2, -s / 2, s, -s, 0.75 * s, -0.25 * s, s / 2, 1.5 * s]))
    # the reference's initialisation quirk (strict minimum at c-2 keeps c)
    q = torch.tensor([0.002886, 0.0011, -0.0009, 0.0004, 0.0, -0.0012, 0.0006, 0.0013])
    blocks.append(q)
    for k in range(64):
        mag = 10 ** (-4 + 6 * float(torch.rand(1, generator=gen)))
        blocks.append(torch.randn(8, generator=gen) * mag)
    # zeros, signed zeros, denormals, huge values
    blocks.append(torch.zeros(8))
    blocks.append(torch.tensor([-0.0, 0.0, -0.0, 0.0, 0.0, -0.0, 0.0, 0.0]))
    blocks.append(torch.tensor([1e-40, -1e-41, 3e-39, 0.0, -2e-39, 1e-45, 0.0, 5e-40]))
    blocks.append(torch.tensor([1e5, -3e4, 2.0, -7.0, 40.0, 0.1, -1e3, 12.0]))
    blocks.append(torch.tensor([64.0, -33.0, 31.0, 0.5, -0.5, 16.0, 48.0, -64.0]))
    # 1e-38 clamp boundary and tiny maxima
    blocks.append(torch.tensor([1e-38, -1e-38, 0.0, 0.0, 0.0, 0.0, 0.0, 1e-39]))
    blocks.append(torch.tensor([9.765625e-4, -4.8828125e-4, 4.8828125e-4, 0.0, 2e-4, -9e-4, 1e-3, 0.0]))
    return torch.stack(blocks).float().reshape(-1)


def gen_spfp2():
    torch.manual_seed(0)
    W = torch.randn(9728, 2560) * 0.02
    x = torch.randn(1, 2560).bfloat16()
    packed5, expv = fp2.pack_blockwise_paired(W)
    dec = fp2.unpack_blockwise_paired(packed5, W.numel(), dtype=torch.float32)
    y = x.float() @ dec.view(9728, 2560).T
    p3, e3 = fp2.pack_blockwise_search(W)
    fq = fp2.channel_fake_quantize(W)
    rows = 16
    nb_rows = rows * 2560 // 8
    gen = torch.Generator().manual_seed(1234)
    adv = spfp2_adversarial(gen)
    adv_p5, adv_e = fp2.pack_blockwise_paired(adv)
    adv_p3, _ = fp2.pack_blockwise_search(adv)
    adv_dec = fp2.unpack_blockwise_paired(adv_p5, adv.numel())
    adv_fq = fp2.channel_fake_quantize(adv.view(-1, 8))
    # odd block count, and a ragged (oc=5, ic=20 -> padded to 24) layer as the layer classes do it
    odd = torch.randn(7 * 8, generator=gen) * 0.05
    odd_p5, odd_e = fp2.pack_blockwise_paired(odd)
    odd_dec = fp2.unpack_blockwise_paired(odd_p5, odd.numel())
    # unpack of random bytes (every code, including the unused code 3)
    rnd5 = torch.randint(0, 256, (5 * 97,), generator=gen, dtype=torch.uint8)
    rnd5_dec = fp2.unpack_blockwise_paired(rnd5, 97 * 16)
    rnd3 = torch.randint(0, 256, (3 * 61,), generator=gen, dtype=torch.uint8)
    rnd3_dec = fp2.unpack_blockwise(rnd3, 61 * 8)
    # bf16 weights through the QAT fake-quant (x.float() first)
    wb = (torch.randn(64, 128, generator=gen) * 0.03).bfloat16()
    wb_fq = fp2.channel_fake_quantize(wb)
    save("spfp2.npz",
         cfg1_packed5_sha=sha(packed5), cfg1_expv_sha=sha(expv), cfg1_dec_sha=sha(dec),
         cfg1_packed3_sha=sha(p3), cfg1_fq_sha=sha(fq),
         cfg1_rows_w=npy(W[:rows]), cfg1_rows_packed5=npy(packed5[: nb_rows // 2 * 5]),
         cfg1_rows_dec=npy(dec[: rows * 2560]), cfg1_x=npy(x.float()), cfg1_y=npy(y),
         adv_w=npy(adv), adv_packed5=npy(adv_p5), adv_expv=npy(adv_e), adv_packed3=npy(adv_p3),
         adv_dec=npy(adv_dec), adv_fq=npy(adv_fq.reshape(-1)),
         odd_w=npy(odd), odd_packed5=npy(odd_p5), odd_expv=npy(odd_e), odd_dec=npy(odd_dec),
         rnd5=npy(rnd5), rnd5_dec=npy(rnd5_dec), rnd3=npy(rnd3), rnd3_dec=npy(rnd3_dec),
         bf16_w=npy(wb.float()), bf16_fq=npy(wb_fq.float()))


# --------------------------------------------------------------------------
def scaled_edge_blocks(gen, top: float) -> torch.Tensor:
    """16-blocks for FP3 (top=1.5) / NVFP4 (top=6): zero, tiny, subnormal
    scale, exact bucket ties, huge (fp8 overflow -> NaN scale), signed zeros."""
    rows = []
    rows.append(torch.zeros(16))
    rows.append(torch.tensor([-0.0, 0.0] * 8))
    rows.append(torch.randn(16, generator=gen) * 1e-12)                 # scale underflows to 0
    rows.append(torch.randn(16, generator=gen) * 2e-3 * top)            # subnormal scales
    rows.append(torch.randn(16, generator=gen) * 5e-3 * top)
    for amax in (448.0 * top, 460.0 * top, 464.0 * top, 470.0 * top, 1e4):   # fp8 top end
        r = torch.rand(16, generator=gen) * amax
        r[3] = amax
        rows.append(r)
    # exact ties: choose a block whose scale is exact, put values on bucket edges
    s = 0.25  # amax/top rounds to exactly 0.25 in e4m3 when amax = 0.25*top
    edges = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    vals = [v * s for v in edges if v <= top] + [top * s]
    r = torch.tensor((vals + [-v for v in vals]) * 4)[:16]
    r[0] = top * s
    rows.append(r)
    rows.append(torch.tensor([float('inf')] + [0.1] * 15))
    rows.append(torch.tensor([float('nan')] + [0.1] * 15))
    return torch.stack(rows).float()


def gen_fp3_nvfp4():
    gen = torch.Generator().manual_seed(77)
    torch.manual_seed(1)
    Wq = torch.randn(4096, 2560) * 0.02                                   # config-2 q_proj
    Wo = torch.randn(2560, 4096) * 0.02                                   # config-2 out_proj
    c3, s3 = fp3_emu.fp3_pack_3bit(Wq)
    d3 = fp3_emu.fp3_unpack_3bit(c3, s3, 4096, 2560)
    c4, s4 = nvfp4_emu.nvfp4_pack(Wo)
    d4 = nvfp4_emu.nvfp4_unpack(c4, s4, 2560, 4096)
    out = dict(q_c3_sha=sha(c3), q_s3_sha=sha(s3.view(torch.uint8)), q_d3_sha=sha(d3),
               o_c4_sha=sha(c4), o_s4_sha=sha(s4.view(torch.uint8)), o_d4_sha=sha(d4))
    for tag, top in (("fp3", 1.5), ("nvfp4", 6.0)):
        edge = scaled_edge_blocks(gen, top)
        rnd = torch.randn(24, 256, generator=gen) * 0.02
        rag = torch.randn(7, 40, generator=gen) * 0.05                    # ic % 16 != 0, odd group count
        for name, w in (("edge", edge), ("rnd", rnd), ("rag", rag)):
            oc, ic = w.shape
            out[f"{tag}_{name}_w"] = npy(w)
            if tag == "fp3":
                c, s = fp3_emu.fp3_pack_3bit(w)
                cn, sn = fp3_emu.fp3_pack(w)
                out[f"{tag}_{name}_c3"] = npy(c)
                out[f"{tag}_{name}_cn"] = npy(cn)
                out[f"{tag}_{name}_s"] = npy(s)
                out[f"{tag}_{name}_dec3"] = npy(fp3_emu.fp3_unpack_3bit(c, s, oc, ic))
                out[f"{tag}_{name}_decn"] = npy(fp3_emu.fp3_unpack(cn, sn, oc, ic))
                out[f"{tag}_{name}_fq"] = npy(fp3_emu.fp3_fake_quant(w))
            else:
                c, s = nvfp4_emu.nvfp4_pack(w)
                out[f"{tag}_{name}_c"] = npy(c)
                out[f"{tag}_{name}_s"] = npy(s)
                out[f"{tag}_{name}_dec"] = npy(nvfp4_emu.nvfp4_unpack(c, s, oc, ic))
                out[f"{tag}_{name}_fq"] = npy(nvfp4_emu.nvfp4_fake_quant(w))
    # every float8 byte -> float, and a sweep of float -> float8 around every code
    allb = torch.arange(256, dtype=torch.uint8)
    out["e4m3_all_f32"] = npy(allb.view(torch.float8_e4m3fn).float())
    xs = torch.cat([torch.logspace(-12, 3.2, 20000, base=10.0), torch.tensor([464.0, 463.99997, 464.00003, 480.0,
                    448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, 2.0 ** -6, 1e-30, 0.0])]).float()
    xs = torch.cat([xs, -xs])
    out["e4m3_sweep_x"] = npy(xs)
    out["e4m3_sweep_b"] = npy(xs.to(torch.float8_e4m3fn))
    # random bytes through both unpackers
    rb = torch.randint(0, 256, (3 * 20 * 2,), generator=gen, dtype=torch.uint8)
    rs = torch.randint(0, 256, (10,), generator=gen, dtype=torch.uint8)
    rs[rs == 0x7f] = 0x11
    rs[rs == 0xff] = 0x91
    out["rnd_fp3_c3"] = npy(rb)
    out["rnd_fp3_s"] = npy(rs)
    out["rnd_fp3_dec3"] = npy(fp3_emu.fp3_unpack_3bit(rb, rs.view(torch.float8_e4m3fn), 5, 32))
    rb4 = torch.randint(0, 256, (80,), generator=gen, dtype=torch.uint8)
    out["rnd_nvfp4_c"] = npy(rb4)
    out["rnd_nvfp4_s"] = npy(rs)
    out["rnd_nvfp4_dec"] = npy(nvfp4_emu.nvfp4_unpack(rb4, rs.view(torch.float8_e4m3fn), 5, 32))
    save("fp3_nvfp4.npz", **out)


# --------------------------------------------------------------------------
def gen_two_four():
    gen = torch.Generator().manual_seed(99)
    rnd = torch.randn(32, 256, generator=gen) * 0.02
    rag = torch.randn(5, 40, generator=gen) * 0.05                       # pads ic, odd block count
    edge_rows = []
    for pattern in ([1, 1, 1, 1], [1, -1, 1, 0], [0, 1, 1, 1], [-1, -1, -1, -1], [0, 0, 0, 0], [0, 0, 0, -1]):
        edge_rows.append(torch.tensor(pattern * 4, dtype=torch.float32) * 0.03)
    edge_rows.append(torch.zeros(16))
    edge_rows.append(torch.randn(16, generator=gen) * 10.0)
    edge_rows.append(torch.tensor([f32(t) for t in CENTER_T[:15]] + [0.0]))
    edge = torch.stack(edge_rows)
    out = {}
    for name, w in (("rnd", rnd), ("rag", rag), ("edge", edge)):
        oc, ic = w.shape
        p = two_four.two_four_pack(w)
        nbp = oc * ((ic + 15) // 16) * 16
        out[f"{name}_w"] = npy(w)
        out[f"{name}_packed"] = npy(p)
        out[f"{name}_dec"] = npy(two_four.two_four_unpack(p, nbp))
        if w.numel() % 8 == 0:
            out[f"{name}_fq"] = npy(two_four.two_four_fake_quant(w))
    rb = torch.randint(0, 256, (7 * 33,), generator=gen, dtype=torch.uint8)
    out["rnd_bytes"] = npy(rb)
    out["rnd_bytes_dec"] = npy(two_four.two_four_unpack(rb, 33 * 32))
    save("two_four.npz", **out)


def gen_int8():
    """int8_emu: per-row symmetric INT8 (lm_head tier).  Rows: Gaussian, huge,
    tiny (scale clamps at 1e-12), all-zero, exact .5 ties of w/scale, a NaN row."""
    gen = torch.Generator().manual_seed(8)
    w = torch.randn(24, 200, generator=gen) * 0.02
    w[1] *= 1e4
    w[2] *= 1e-12
    w[3] = 0.0
    w[4] = torch.arange(200, dtype=torch.float32) * 0.5 - 50.0       # scale 0.3937..: many near-ties
    w[5, :] = torch.tensor([(k + 0.5) for k in range(-100, 100)], dtype=torch.float32) * (1.0 / 127.0) * 99.5 / 99.5
    w[6, 7] = float("nan")
    out = {"w": npy(w), "fq": npy(int8_emu.int8_fake_quant(w))}
    wp = w[torch.arange(24) != 6]
    q, scale = int8_emu.ptq_int8_pack(wp)
    out.update(w_pack=npy(wp), q=npy(q), scale=npy(scale), unpack=npy(int8_emu.ptq_int8_unpack(q, scale)))
    g2 = torch.Generator().manual_seed(9)
    wb = (torch.randn(16, 96, generator=g2) * 0.05).bfloat16()
    out.update(w_bf16_bits=npy(wb.view(torch.int16)), fq_bf16_in=npy(int8_emu.int8_fake_quant(wb)))
    save("int8.npz", **out)


def gen_thresholds():
    save("thresholds.npz", center_t=np.array(CENTER_T, np.uint32))


if __name__ == "__main__":
    gen_thresholds()
    gen_spfp2()
    gen_fp3_nvfp4()
    gen_two_four()
    gen_int8()
