"""Benchmark of SPARK's online-dequant linear path on B200.

Metric: dequant-GEMV HBM GB/s at M=1 (and prefill TFLOP/s).

Workload: the tiered decode linears of one hybrid-attention
layer at 4B-like shapes -- gate/up [9728,2560] and down [2560,9728] in SPFP2,
q/k/v [4096,2560] in FP3 E1M1, out_proj [2560,4096] in NVFP4 -- random
N(0, 0.02) weights packed on the GPU, bf16 N(0,1) activations, M = 1.
One step runs one token through L = 8 distinct copies of that layer
(56 linears, 344 MB of packed weights: more than the 126 MB L2, so every
step streams its weights from HBM).  `value` is algorithmic bytes (packed
weights + scales + x + y) per second with everything resident in HBM, the
step replayed as a CUDA graph.  `e2e` is the same metric through the public
layer API (spark_b200.inference_v3.V3PackedLinear) with the token read from
pinned host memory and every output copied back to the host inside the
timed region.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With torchrun (N > 1) every rank runs its own replica (weak scaling); the
step time is the max over ranks.  The same line carries `tp_mlp`: BASELINE
config 4 (a 32-layer SPFP2 MLP stack at 64 tokens) tensor-parallel over the N
ranks (gate/up column-split, down row-split, one NCCL all-reduce of fp32
partials per layer), with a parity check of a 2-layer slice against an fp64
evaluation of the unsharded weights, and `tp_decode`: the same stack at 8
decode tokens, NCCL form against one launch per layer with the all-reduce
inside the kernel (spark_linear_batch_ar).  `--impl reference` times the
reference's CPU path (decode + fp32 matmul per call, ported to C in oracle/)
on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS = 8                     # distinct layer copies per step
SHAPES = [                     # (name, fmt, oc, ic)
    ("gate_proj", "spfp2", 9728, 2560),
    ("up_proj", "spfp2", 9728, 2560),
    ("down_proj", "spfp2", 2560, 9728),
    ("q_proj", "fp3", 4096, 2560),
    ("k_proj", "fp3", 4096, 2560),
    ("v_proj", "fp3", 4096, 2560),
    ("out_proj", "nvfp4", 2560, 4096),
]
# Projections that read the same activations run as one row-merged launch
# (spark_b200.inference_v3.V3MergedLinear), as inference engines fuse q/k/v
# and gate/up: the same weights, bytes and outputs in 4 launches per layer.
GROUPS = [                     # (launch name, fmt, projections in row order)
    ("qkv_proj", "fp3", ("q_proj", "k_proj", "v_proj")),
    ("out_proj", "nvfp4", ("out_proj",)),
    ("gate_up_proj", "spfp2", ("gate_proj", "up_proj")),
    ("down_proj", "spfp2", ("down_proj",)),
]
CONFIG = {
    "workload": "BASELINE config 2: tiered decode linears of one 4B-like hybrid-attention layer "
                "(SPFP2 gate/up/down, FP3 q/k/v, NVFP4 out_proj), M=1, one token through 8 layer copies per step",
    "M": 1,
    "layers_per_step": LAYERS,
    "l2": "weights rotate over 8 distinct layer copies (344 MB) > 126 MB L2",
    "graph": "each step replayed as one CUDA graph",
    "projections": "q|k|v and gate|up row-merged into one packed weight each (V3MergedLinear): 32 linears per "
                   "step, all in ONE spark_linear_batch launch; per_launch repeats the step with one launch per "
                   "linear, per_projection with one launch per unmerged projection (56)",
    "dependencies": "none: each linear reads its layer-copy's fixed activation, as the metric's GEMVs are "
                    "independent; spark_linear_batch also takes ops that read earlier ops' outputs",
}
METRIC = "dequant-GEMV HBM GB/s (% of 8 TB/s) at M=1; prefill dequant-GEMM TFLOP/s"
PREFILL_M = 2048               # prefill tokens through one layer's 7 linears


def weight_bytes(fmt, oc, ic):
    if fmt == "spfp2":
        return oc * ic // 16 * 5
    if fmt == "fp3":
        return oc * ic // 8 * 3 + oc * ic // 16
    if fmt == "nvfp4":
        return oc * ic // 2 + oc * ic // 16
    raise ValueError(fmt)


def linear_bytes(fmt, oc, ic, M=1, act_bytes=2):
    return weight_bytes(fmt, oc, ic) + M * ic * act_bytes + M * oc * act_bytes


STEP_BYTES = LAYERS * sum(linear_bytes(f, oc, ic) for _, f, oc, ic in SHAPES)
SPFP2_BYTES = LAYERS * sum(linear_bytes(f, oc, ic) for _, f, oc, ic in SHAPES if f == "spfp2")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the measured cuBLAS burst figure (the prefill loop is
    timed for a few ms), else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured MEASURED_PEAKS.json bf16_tflops (burst)"
    except Exception:
        return 1590.0, "fallback 1590 TFLOP/s"


def host_threads() -> int:
    """Host threads this process may run on (torchrun sets OMP_NUM_THREADS=1 per
    rank; the CPU legs set their thread counts from this instead)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def host_info() -> dict:
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except Exception:
        pass
    return {"cpu_model": model, "cpu_count": os.cpu_count(), "threads": host_threads(), "torch": torch.__version__}


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ distributed
def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ GPU arm
def build_layers(device):
    from spark_b200 import ops
    layers = []
    g = torch.Generator(device=device)
    for li in range(LAYERS):
        g.manual_seed(1000 + li)
        L = {}
        for name, fmt, oc, ic in SHAPES:
            W = torch.randn(oc, ic, device=device, generator=g) * 0.02
            if fmt == "spfp2":
                wq, s = ops.spfp2_pack(W)[0], None
            elif fmt == "fp3":
                wq, s = ops.fp3_pack(W)
            else:
                wq, s = ops.nvfp4_pack(W)
            # the layer API keeps the fragment-major copy for the GEMV
            L[name] = (fmt, wq, s, oc, ic, ops.tile_weights(fmt, wq, s, oc, ic))
            del W
        layers.append(L)
    torch.cuda.synchronize()
    return layers


def merge_layer(L):
    """Row-merged launches of one layer: packed bytes (and scales) concatenated."""
    from spark_b200 import ops
    out = {}
    for gname, fmt, parts in GROUPS:
        wq = torch.cat([L[p][1] for p in parts])
        s = torch.cat([L[p][2] for p in parts]) if L[parts[0]][2] is not None else None
        oc, ic = sum(L[p][3] for p in parts), L[parts[0]][4]
        out[gname] = (fmt, wq, s, oc, ic, ops.tile_weights(fmt, wq, s, oc, ic))
    return out


def run_gpu(args, rank, world, local):
    from spark_b200 import ops
    device = torch.device("cuda", local)
    layers = build_layers(device)
    merged = [merge_layer(L) for L in layers]
    g = torch.Generator(device=device).manual_seed(7)
    x = {ic: torch.randn(1, ic, device=device, generator=g).bfloat16() for ic in (2560, 4096, 9728)}
    outs = {}
    stream = torch.cuda.Stream(device)
    max_ws = max(ops.workspace_size(ops.FORMATS[f], 1, oc, ic) for _, f, oc, ic in SHAPES)
    ops.workspace(device, max_ws, stream=stream)

    def step(only=None, which=None):
        # one spark_linear launch per linear; every decode GEMV pulls the next
        # launch's weight into L2 (the last one the first's: the next token
        # starts over)
        seq = [((name, id(L)), fmt, oc, ic, wt) for L in (which or merged) for name, (fmt, _, _, oc, ic, wt)
               in L.items() if not only or fmt == only]
        for k, (key, fmt, oc, ic, wt) in enumerate(seq):
            nxt = seq[(k + 1) % len(seq)][4]
            outs[key] = ops.linear(fmt, wt, None, x[ic], oc, ic, out=outs.get(key), tiled=True, prefetch=nxt)

    def make_batch(xs, only=None):
        """The step's row-merged linears as ONE spark_linear_batch launch."""
        ys = {}
        batch = []
        for L in merged:
            for name, (fmt, _, _, oc, ic, wt) in L.items():
                if only and fmt != only:
                    continue
                y = torch.empty(xs[ic].shape[0], oc, dtype=torch.bfloat16, device=device)
                ys[(name, id(L))] = y
                batch.append(ops.BatchOp(fmt, wt, xs[ic], y))
        return batch, ys

    batch_all, _ = make_batch(x)
    batch_spfp2, _ = make_batch(x, "spfp2")

    # warm every path once eagerly (allocates outputs), then capture
    with torch.cuda.stream(stream):
        for _ in range(2):
            ops.linear_batch(batch_all)
            ops.linear_batch(batch_spfp2)
            step()
            step(which=layers)
    torch.cuda.synchronize()
    graph, graph_spfp2, graph_pl, graph_pp = (torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph(),
                                              torch.cuda.CUDAGraph())
    with torch.cuda.graph(graph, stream=stream):
        ops.linear_batch(batch_all)
    with torch.cuda.graph(graph_spfp2, stream=stream):
        ops.linear_batch(batch_spfp2)
    with torch.cuda.graph(graph_pl, stream=stream):
        step()
    with torch.cuda.graph(graph_pp, stream=stream):
        step(which=layers)
    torch.cuda.synchronize()

    def timed(gr, k):
        for _ in range(args.warmup):
            gr.replay()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(k):
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        barrier(world)
        torch.cuda.synchronize()
        return max_over_ranks(ms, world)

    # clocks are sampled from the first timed replay through the prefill and
    # the tensor-parallel stack (the decode step alone lasts milliseconds,
    # shorter than one nvidia-smi sample)
    clk = Clocks(local)
    clk.__enter__()
    ms_total = timed(graph, args.steps)
    ms_spfp2 = timed(graph_spfp2, args.steps)
    ms_pl = timed(graph_pl, args.steps)
    ms_pp = timed(graph_pp, args.steps)
    ops.check_device_errors()

    # config 2 also names 4 and 16 tokens: the batched step at those M (the
    # decode kernel serves up to 16 tokens per launch), bytes counted as above
    decode_tokens = {}
    for m_tok in (4, 16):
        xm = {ic: torch.randn(m_tok, ic, device=device, generator=g).bfloat16() for ic in x}
        batch_m, _ = make_batch(xm)

        with torch.cuda.stream(stream):
            ops.linear_batch(batch_m)
            ops.linear_batch(batch_m)
        torch.cuda.synchronize()
        gm = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gm, stream=stream):
            ops.linear_batch(batch_m)
        k_m = max(5, args.steps // 5)
        ms_m = timed(gm, k_m)
        bytes_m = LAYERS * sum(linear_bytes(f, oc, ic, M=m_tok) for _, f, oc, ic in SHAPES)
        decode_tokens[str(m_tok)] = {"value": round(world * bytes_m * k_m / (ms_m * 1e-3) / 1e9, 1), "unit": "GB/s",
                                     "ms_per_step": round(ms_m / k_m, 4),
                                     "tokens_per_s": round(world * m_tok * k_m / (ms_m * 1e-3), 1)}
        del gm
    ops.check_device_errors()

    # ---------------- e2e through the public layer API with host buffers
    from spark_b200.inference_v3 import V3LinearBatch, V3MergedLinear, V3PackedLinear, chain_prefetch
    mods = []
    for L in layers:
        lin = {name: V3PackedLinear.from_packed(fmt, wq, s, oc, ic) for name, (fmt, wq, s, oc, ic, _) in L.items()}
        mods.append({gname: V3MergedLinear([lin[p] for p in parts]) if len(parts) > 1 else lin[parts[0]]
                     for gname, _, parts in GROUPS})
    chain_prefetch([L[gname] for L in mods for gname, _, _ in GROUPS])
    xh = {ic: x[ic].cpu().pin_memory() for ic in x}
    # every projection's output lands in one device buffer (the layers' out=
    # argument), copied to pinned host memory once per step
    width = {gname: sum(next(o for n, _, o, _ in SHAPES if n == p) for p in parts) for gname, _, parts in GROUPS}
    total = LAYERS * sum(width.values())
    ydev = torch.empty(1, total, dtype=torch.bfloat16, device=device)
    yhost = torch.empty(1, total, dtype=torch.bfloat16).pin_memory()
    yslot, off = {}, 0
    for L in mods:
        for gname, _, _ in GROUPS:
            yslot[(gname, id(L))] = ydev[:, off:off + width[gname]]
            off += width[gname]
    h2d = sum(t.numel() * 2 for t in xh.values())
    d2h = yhost.numel() * 2

    # the step's layers as one V3LinearBatch call (one launch)
    order = [(L, gname) for L in mods for gname, _, _ in GROUPS]
    step_layers = V3LinearBatch([L[gname] for L, gname in order])
    step_outs = [yslot[(gname, id(L))] for L, gname in order]

    def e2e_step():
        xd = {ic: xh[ic].to(device, non_blocking=True) for ic in xh}
        step_layers([xd[L[gname].in_features] for L, gname in order], step_outs)
        yhost.copy_(ydev, non_blocking=True)

    def time_e2e(run, k):
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 1)):
                run()
            torch.cuda.synchronize()
            barrier(world)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(k):
                run()
            e1.record(stream)
            torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1), world)
        barrier(world)
        return ms

    # eager: every module call dispatched from Python
    ms_e2e_eager = time_e2e(e2e_step, args.steps)
    # the same public-API step captured as a CUDA graph, as a decode loop runs it:
    # the pinned host->device copy of the token and every device->host copy of
    # the projections' outputs stay inside each replayed step
    e2e_mode = "cuda_graph"
    try:
        graph_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            e2e_step()
            torch.cuda.synchronize()
            with torch.cuda.graph(graph_e2e, stream=stream):
                e2e_step()
        torch.cuda.synchronize()
        ms_e2e = time_e2e(graph_e2e.replay, args.steps)
    except RuntimeError as exc:          # capture refused: report the eager number, say why
        e2e_mode = f"eager (graph capture failed: {str(exc).splitlines()[0][:120]})"
        torch.cuda.synchronize()
        ms_e2e = ms_e2e_eager

    # ---------------- prefill: PREFILL_M bf16 tokens through the
    # 7 linears of one layer, reference-layout weights -> the tcgen05 GEMM
    xs = {ic: torch.randn(PREFILL_M, ic, device=device, generator=g).bfloat16() for ic in (2560, 4096, 9728)}

    yg = {name: torch.empty(PREFILL_M, oc, device=device, dtype=torch.bfloat16)
          for name, (_, _, _, oc, _, _) in merged[0].items()}

    def prefill_step():
        # the row-merged launches of the decode step, on the reference-layout bytes
        for name, (fmt, wq, s, oc, ic, _) in merged[0].items():
            ops.linear(fmt, wq, s, xs[ic], oc, ic, out=yg[name])

    with torch.cuda.stream(stream):
        prefill_step()
        prefill_step()
    torch.cuda.synchronize()
    graph_pre = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_pre, stream=stream):
        prefill_step()
    pre_steps = max(50, args.steps // 10)
    ms_pre = timed(graph_pre, pre_steps)
    ops.check_device_errors()
    del graph_pre, graph, graph_spfp2, graph_pl, graph_pp

    # ---------------- native NVFP4 x NVFP4 (a reported mode): the out_proj weight
    # [2560, 4096] at PREFILL_M tokens on tcgen05.mma kind::mxf4nvf4, activations
    # quantised to NVFP4 by the weights' quantiser; error against the parity path
    _, wq_o, s_o, oc_o, ic_o, _ = merged[0]["out_proj"]
    x_o = xs[ic_o]
    xq_o = ops.nvfp4_pack(x_o)
    y_nat = ops.nvfp4_native_linear(wq_o, s_o, x_o, oc_o, ic_o, out_dtype=torch.float32, xq=xq_o)
    y_par = ops.linear("nvfp4", wq_o, s_o, x_o, oc_o, ic_o, out_dtype=torch.float32)
    nat_rel = float((y_nat.double() - y_par.double()).norm() / y_par.double().norm())
    del y_nat, y_par
    y_n = torch.empty(PREFILL_M, oc_o, device=device, dtype=torch.bfloat16)
    x_c, x_s = xq_o

    def native_gemm():
        ops.nvfp4_native_linear(wq_o, s_o, x_o, oc_o, ic_o, xq=(x_c, x_s))

    def native_full():
        ops.nvfp4_native_linear(wq_o, s_o, x_o, oc_o, ic_o)

    nat = {}
    for name, fn in (("gemm", native_gemm), ("with_x_quantisation", native_full)):
        with torch.cuda.stream(stream):
            fn()
            fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for _ in range(4):
                fn()
        nat[name] = timed(gr, pre_steps) / (4 * pre_steps)
        del gr
    ops.check_device_errors()
    del y_n

    # ---------------- 2:4 down_proj [2560, 9728] (seeded N(0, 0.02) weights) on the
    # sparse tensor cores (spark_linear's route at 128-1024 tokens, and the kernel
    # called directly at PREFILL_M) against the dense decode (tcgen05 kind::f16)
    g24 = torch.Generator(device=device).manual_seed(24)
    oc24, ic24 = 2560, 9728
    w24 = ops.twofour_pack(torch.randn(oc24, ic24, device=device, generator=g24) * 0.02)
    tf24 = {}
    for name, m24, fn in (
            ("sparse_m1", 1, lambda x: ops.linear("twofour", w24, None, x, oc24, ic24)),
            ("dense_m1", 1, lambda x: ops.linear("twofour", w24, None, x, oc24, ic24, tcgen05=True)),
            ("sparse_m512", 512, lambda x: ops.linear("twofour", w24, None, x, oc24, ic24)),
            ("dense_m512", 512, lambda x: ops.linear("twofour", w24, None, x, oc24, ic24, tcgen05=True)),
            ("sparse_m2048", PREFILL_M, lambda x: ops.twofour_sparse_linear(w24, x, oc24, ic24)),
            ("dense_m2048", PREFILL_M, lambda x: ops.linear("twofour", w24, None, x, oc24, ic24))):
        x24 = torch.randn(m24, ic24, device=device, generator=g24).bfloat16()
        with torch.cuda.stream(stream):
            fn(x24)
            fn(x24)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for _ in range(4):
                fn(x24)
        ms24 = timed(gr, pre_steps) / (4 * pre_steps)
        tf24[name] = {"ms": round(ms24, 4), "TFLOP/s dense-equivalent": round(2.0 * m24 * oc24 * ic24 / (ms24 * 1e-3) / 1e12, 1)}
        del gr, x24
    ops.check_device_errors()
    del w24

    # ---------------- BASELINE config 4, tensor-parallel over the ranks of this run
    tp = tp_mlp_measure(args, rank, world, local)
    try:
        tp_dec = tp_decode_measure(args, rank, world, local)
    except Exception as e:        # a device-side error reaches every rank alike; keep the line
        tp_dec = {"error": f"{type(e).__name__}: {e}"[:300]}
    clk.__exit__(None, None, None)
    pre_flops = sum(2.0 * PREFILL_M * oc * ic for _, _, oc, ic in SHAPES)
    pre_tflops = world * pre_flops * pre_steps / (ms_pre * 1e-3) / 1e12
    nat_flops = 2.0 * PREFILL_M * oc_o * ic_o
    nat_tf = {k: round(nat_flops / (v * 1e-3) / 1e12, 1) for k, v in nat.items()}
    tpeak, tpeak_kind = tensor_peak()

    peak, peak_kind = peaks()
    value = world * STEP_BYTES * args.steps / (ms_total * 1e-3) / 1e9
    spfp2_gbs = SPFP2_BYTES * args.steps / (ms_spfp2 * 1e-3) / 1e9
    e2e_gbs = world * STEP_BYTES * args.steps / (ms_e2e * 1e-3) / 1e9
    e2e_eager_gbs = world * STEP_BYTES * args.steps / (ms_e2e_eager * 1e-3) / 1e9
    # one batched launch per step; per_launch: one launch per row-merged linear
    launches = args.steps
    launches_pl = args.steps * LAYERS * len(GROUPS)
    launches_pp = args.steps * LAYERS * len(SHAPES)
    value_pl = world * STEP_BYTES * args.steps / (ms_pl * 1e-3) / 1e9
    value_pp = world * STEP_BYTES * args.steps / (ms_pp * 1e-3) / 1e9
    traffic = load_traffic()
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_total / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 activations, packed 2.5/3.5/4.5-bit weights, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) bf16 activations)",
        "config": {**CONFIG, "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "hbm_frac": round(value / world / peak, 4),
        "roofline": {"bound": "hbm", "kernel": "k_stream (spark_linear_batch): the step's 32 row-merged linears "
                                               "(FP3 q|k|v, NVFP4 out, SPFP2 gate|up and down x 8 layers) in one launch",
                     "achieved": round(value / world, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(value / world / peak, 4), "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs"
                     if peak_kind == "measured" else "fallback 6650 GB/s",
                     "traffic": traffic, "bytes_per_launch": STEP_BYTES},
        "gpu_launches": launches,
        "spfp2_only": {"value": round(spfp2_gbs, 1), "unit": "GB/s", "frac": round(spfp2_gbs / peak, 4),
                       "ms_per_step": round(ms_spfp2 / args.steps, 4),
                       "note": "the 16 SPFP2 linears (gate|up, down) of the step in one launch"},
        "per_launch": {"value": round(value_pl, 1), "unit": "GB/s", "ms_per_step": round(ms_pl / args.steps, 4),
                       "gpu_launches": launches_pl,
                       "note": "the same 32 linears as separate spark_linear launches (graph-replayed)"},
        "per_projection": {"value": round(value_pp, 1), "unit": "GB/s", "ms_per_step": round(ms_pp / args.steps, 4),
                           "gpu_launches": launches_pp},
        "decode_tokens": decode_tokens,
        "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "spark_b200.inference_v3.V3LinearBatch over the step's V3MergedLinear / V3PackedLinear layers, "
                       "called per step with its pinned host<->device copies", "mode": e2e_mode,
                "eager": {"value": round(e2e_eager_gbs, 1), "unit": "GB/s",
                          "note": "the same calls dispatched from Python every step"}},
        "clocks": clk.summary(),
        "tp_mlp": tp,
        "tp_decode": tp_dec,
        "prefill": {
            "workload": f"BASELINE config 3: M={PREFILL_M} bf16 tokens through the 7 linears of one layer "
                        "(SPFP2 gate/up/down, FP3 q/k/v, NVFP4 out_proj) as 4 row-merged launches (q|k|v, "
                        "out, gate|up, down), reference-layout weights, one CUDA graph per step",
            "value": round(pre_tflops, 1), "unit": "TFLOP/s", "steps": pre_steps,
            "ms_per_step": round(ms_pre / pre_steps, 4), "flops_per_step": pre_flops,
            "kernel": "k_tc_linear<FMT, 128 or 256 tokens> (tcgen05.mma kind::f16, A = decoded weights in TMEM)",
            "roofline": {"bound": "tensor", "achieved": round(pre_tflops / world, 1), "peak": tpeak,
                         "unit": "TFLOP/s", "frac": round(pre_tflops / world / tpeak, 4), "peak_source": tpeak_kind},
            "nvfp4_native": {
                "workload": f"out_proj [{oc_o}, {ic_o}] NVFP4 at M={PREFILL_M}, activations quantised to NVFP4 "
                            "(spark_nvfp4_native_linear: tcgen05.mma kind::mxf4nvf4 block16, fp32 accumulate)",
                "value": nat_tf["gemm"], "unit": "TFLOP/s", "ms": round(nat["gemm"], 4),
                "with_x_quantisation": {"value": nat_tf["with_x_quantisation"], "unit": "TFLOP/s",
                                        "ms": round(nat["with_x_quantisation"], 4)},
                "roofline": {"bound": "tensor", "achieved": nat_tf["gemm"], "peak": 9000.0, "unit": "TFLOP/s",
                             "frac": round(nat_tf["gemm"] / 9000.0, 4),
                             "peak_source": "nominal dense FP4 (no measured FP4 peak on this pool)"},
                "rel_frobenius_vs_parity_path": round(nat_rel, 5),
                "note": "a reported mode, not the parity path: the error is the activations' FP4 rounding",
            },
            "twofour": {
                "workload": "2:4 down_proj [2560, 9728], bf16 x: tcgen05.mma.sp kind::f16 on the kept values "
                            "(spark_twofour_sparse_linear; spark_linear's route at up to 16 tokens, K split, and at "
                            "128-1024 tokens) vs the dense decode on tcgen05.mma kind::f16",
                **tf24,
            },
        },
    }
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args, budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)


def load_traffic():
    """Per-launch DRAM bytes (read + write) of the dominant kernel, k_stream over the headline
    step, from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "stream_step_m1.json")
    try:
        with open(p) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except Exception:
        return None


# ------------------------------------------------------------------ CPU (reference) arm
def cpu_layer(seed):
    """One layer's packed weights for the CPU path (packed by the oracle)."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    out = {}
    for name, fmt, oc, ic in SHAPES:
        W = (rng.standard_normal((oc, ic), dtype=np.float32) * 0.02).astype(np.float32)
        if fmt == "spfp2":
            out[name] = (fmt, O.pack_blockwise_paired(W)[0], None, oc, ic)
        elif fmt == "fp3":
            c, s = O.fp3_pack_3bit(W)
            out[name] = (fmt, c, s, oc, ic)
        else:
            c, s = O.nvfp4_pack(W)
            out[name] = (fmt, c, s, oc, ic)
    return out


def cpu_step(layer, xs):
    from oracle import oracle as O
    for name, (fmt, wq, s, oc, ic) in layer.items():
        x = xs[ic]
        if fmt == "spfp2":
            O.cpu_spfp2_linear(wq, x, oc, ic)
        elif fmt == "fp3":
            O.cpu_fp3_linear(wq, s, x, oc, ic)
        else:
            O.cpu_nvfp4_linear(wq, s, x, oc, ic)


def _cpu_decode_layer(layer):
    """Decode-at-load form of a CPU layer: fp32 weights as torch tensors (what
    the reference's apply_spark_state leaves in the model, 02_model/spark_loader.py:102-163)."""
    from oracle import oracle as O
    out = {}
    for name, (fmt, wq, s, oc, ic) in layer.items():
        if fmt == "spfp2":
            W = O.unpack_blockwise_paired(wq, oc * ic)
        elif fmt == "fp3":
            W = O.fp3_unpack_3bit(wq, s, oc, ic)
        else:
            W = O.nvfp4_unpack(wq, s, oc, ic)
        out[name] = (ic, torch.from_numpy(np.ascontiguousarray(W, dtype=np.float32).reshape(oc, ic)))
    return out


def cpu_baseline(args, budget_s=15.0):
    """Time the reference's CPU path on a bounded sample, on all host threads:
    (b) decode + fp32 matmul per call (the online path the GPU kernels run) as
    the value, and (a) decode once at load + torch fp32 matmul per call (what
    the reference ships) beside it."""
    from oracle import oracle as O
    threads = host_threads()
    O.set_num_threads(threads)
    torch.set_num_threads(threads)
    layer = cpu_layer(1)
    rng = np.random.default_rng(2)
    xs = {ic: rng.standard_normal((1, ic)).astype(np.float32) for ic in (2560, 4096, 9728)}
    cpu_step(layer, xs)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s and n < 200:
        cpu_step(layer, xs)
        n += 1
    dt = time.perf_counter() - t0
    per_layer = STEP_BYTES / LAYERS
    dec = _cpu_decode_layer(layer)
    xt = {ic: torch.from_numpy(v) for ic, v in xs.items()}

    def load_step():
        for ic, W in dec.values():
            torch.matmul(xt[ic], W.T)

    load_step()
    na, t1 = 0, time.perf_counter()
    while time.perf_counter() - t1 < budget_s / 2 and na < 2000:
        load_step()
        na += 1
    da = time.perf_counter() - t1
    return {"value": round(per_layer * n / dt / 1e9, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} passes over one config-2 layer (7 linears) at M=1 in {dt:.1f} s: "
                      "decode + fp32 matmul per call, rows split over OpenMP threads",
            "decode_at_load": {"value": round(per_layer * na / da / 1e9, 3), "unit": "GB/s",
                               "ms_per_layer": round(da * 1e3 / na, 3), "threads": torch.get_num_threads(),
                               "sample": f"{na} passes: weights decoded to fp32 once, torch CPU matmul per call "
                                         "(bytes counted as the packed layer, as for the value)"},
            "host": host_info()}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as O
    # every host thread, whatever OMP_NUM_THREADS the launcher set
    O.set_num_threads(host_threads())
    layer = cpu_layer(1)
    rng = np.random.default_rng(2)
    xs = {ic: rng.standard_normal((1, ic)).astype(np.float32) for ic in (2560, 4096, 9728)}
    for _ in range(args.warmup):
        cpu_step(layer, xs)
    # a CPU step is a bounded sample of the GPU step: one token through ONE layer
    # copy (7 linears, 43 MB of packed weights) instead of eight
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(layer, xs)
    dt = time.perf_counter() - t0
    value = STEP_BYTES / LAYERS * args.steps / dt / 1e9
    # beside it: decode once at load + torch fp32 matmul per call (the form the
    # reference ships), same steps
    torch.set_num_threads(host_threads())
    dec = _cpu_decode_layer(layer)
    xt = {ic: torch.from_numpy(v) for ic, v in xs.items()}
    for ic, W in dec.values():
        torch.matmul(xt[ic], W.T)
    t1 = time.perf_counter()
    for _ in range(args.steps):
        for ic, W in dec.values():
            torch.matmul(xt[ic], W.T)
    da = time.perf_counter() - t1
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (reference CPU emulator path)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {**CONFIG, "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}, "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
                         "sample": f"{args.steps} steps, each one token through one config-2 layer (7 linears), "
                                   "decode + fp32 matmul per call (oracle/spark_oracle.c port of the reference's "
                                   "CPU path)", "host": host_info(),
                         "decode_at_load": {"value": round(STEP_BYTES / LAYERS * args.steps / da / 1e9, 3),
                                            "unit": "GB/s", "ms_per_step": round(da * 1e3 / args.steps, 3),
                                            "threads": torch.get_num_threads()}},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


TP_LAYERS, TP_H, TP_I, TP_M = 32, 4096, 12288, 64


def _tp_stack(rank, world, device, peer=None, keep_full=0, fused=None):
    """The config-4 stack as TPMLP layers of this rank (TPMLPFused layers sharing
    the BatchAllReduce `fused`, when given), and (keep_full > 0) the first
    keep_full layers' unsharded weights decoded from their SPFP2 packing (the
    GPU unpack, bit-exact against the reference emulator) in fp64."""
    from spark_b200 import ops
    from spark_b200.tp import TPMLP, TPMLPFused
    g = torch.Generator(device=device)
    layers, full = [], []
    for li in range(TP_LAYERS):
        g.manual_seed(4000 + li)
        gate = torch.randn(TP_I, TP_H, device=device, generator=g) * 0.015
        up = torch.randn(TP_I, TP_H, device=device, generator=g) * 0.015
        down = torch.randn(TP_H, TP_I, device=device, generator=g) * 0.015
        layers.append(TPMLPFused(gate, up, down, rank, world, ar=fused) if fused is not None else
                      TPMLP(gate, up, down, rank, world, peer=peer))
        if li < keep_full:
            full.append(tuple(ops.spfp2_unpack(ops.spfp2_pack(w)[0], w.numel()).view(w.shape).double()
                              for w in (gate, up, down)))
        del gate, up, down
    return layers, full


def _tp_reference(x, full):
    """fp64 evaluation of the unsharded layers with the stack's rounding points:
    gate / up outputs, SiLU(gate) * up and each layer's output are bf16."""
    def bf(t):
        return t.to(torch.bfloat16).double()
    y = x.double()
    for wg, wu, wd in full:
        gv, uv = bf(y @ wg.T), bf(y @ wu.T)
        h = bf(gv * torch.sigmoid(gv) * uv)
        y = bf(h @ wd.T)
    return y


def _time_stack(layers, x0, stream, warmup, k, world, graph_it=True):
    out = {}

    def step():
        x = x0
        for layer in layers:
            x = layer(x)
        out["y"] = x

    with torch.cuda.stream(stream):
        step()
        step()
    torch.cuda.synchronize()
    graph = None
    if graph_it:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step
    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            run()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(k):
            run()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    finite = bool(torch.isfinite(out["y"].float()).all().item())
    del graph
    return ms / k, finite


def tp_mlp_measure(args, rank, world, local):
    """a 32-layer SPFP2 MLP stack (hidden 4096, intermediate
    12288, N(0, 0.015) weights, SiLU(gate) * up), 64 bf16 tokens, tensor-
    parallel over the `world` ranks (gate/up column-parallel, down row-parallel
    + one all-reduce of fp32 partials per layer: NCCL, or this library's peer
    all-reduce with --tp-allreduce peer).  Every rank returns the same dict.

    Parity: rank 0's output of layers 0-1 (all ranks run them, the all-reduces
    included) against _tp_reference of the unsharded weights; the bound is two
    bf16 units in the last place at the output's largest magnitude (fp32 vs
    fp64 accumulation may flip a bf16 rounding at any of the rounding points).
    At world > 1 rank 0 also times the unsharded stack on its own GPU (TP1) for
    the strong-scaling efficiency tp1_ms / (world * ms)."""
    import math
    from spark_b200 import ops
    from spark_b200.tp import PeerAllReduce
    device = torch.device("cuda", local)
    peer = PeerAllReduce(TP_M * TP_H, dtype=torch.float32) if args.tp_allreduce == "peer" else None
    layers, full = _tp_stack(rank, world, device, peer=peer, keep_full=2 if rank == 0 else 0)
    g = torch.Generator(device=device).manual_seed(4)
    x0 = torch.randn(TP_M, TP_H, device=device, generator=g).bfloat16()
    stream = torch.cuda.Stream(device)

    # parity of a 2-layer slice (every rank takes part in its all-reduces)
    with torch.cuda.stream(stream):
        y2 = layers[1](layers[0](x0))
    torch.cuda.synchronize()
    parity = None
    if rank == 0:
        ref = _tp_reference(x0, full)
        err = float((y2.double() - ref).abs().max().item())
        ymax = float(ref.abs().max().item())
        tol = 2.0 ** (math.floor(math.log2(max(ymax, 2.0 ** -20))) - 6)
        parity = {"layers": 2, "max_abs": err, "bound": tol, "ok": bool(err <= tol), "max_abs_ref": ymax,
                  "reference": "fp64 of the unsharded SPFP2-decoded weights, bf16 at the stack's rounding points"}
        del ref
    del full, y2

    k = max(20, args.steps // 10)
    sec, finite = _time_stack(layers, x0, stream, args.warmup, k, world, graph_it=bool(args.tp_graph))
    sec *= 1e-3
    ops.check_device_errors()
    if peer is not None:
        peer.check()
    barrier(world)
    if peer is not None:
        peer.close()
    del layers
    torch.cuda.empty_cache()

    tp1 = None
    if world > 1:
        if rank == 0:
            solo, _ = _tp_stack(0, 1, device)
            tp1, _ = _time_stack(solo, x0, stream, args.warmup, k, 1)
            tp1 *= 1e-3
            del solo
            torch.cuda.empty_cache()
        t = torch.tensor([tp1 or 0.0], dtype=torch.float64, device=device)
        if world > 1:
            import torch.distributed as dist
            dist.broadcast(t, 0)
        tp1 = float(t.item())
        barrier(world)
    else:
        tp1 = sec

    packed_total = TP_LAYERS * 3 * (TP_I * TP_H // 16 * 5)
    peak, peak_kind = peaks()
    per_gpu = packed_total / world / sec / 1e9
    return {
        "metric": "config-4 tensor-parallel SPFP2 MLP stack", "n_gpus": world, "steps": k,
        "ms_per_step": round(sec * 1e3, 4), "tokens_per_s": round(TP_M / sec, 1),
        "weight_GBps_total": round(packed_total / sec / 1e9, 1),
        "tp1_ms_per_step": round(tp1 * 1e3, 4),
        "strong_scaling_eff": round(tp1 / (world * sec), 4),
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s per GPU",
                     "frac": round(per_gpu / peak, 4), "peak_source": peak_kind},
        "parity": parity, "finite": finite,
        "config": {"workload": "BASELINE config 4: 32 x (gate/up [12288,4096], down [4096,12288]) SPFP2, "
                               "N(0,0.015), M=64 bf16, SiLU(gate)*up", "tp": world,
                   "parallelism": f"tp{world}: gate/up column-parallel (one row-merged launch), down "
                                  "row-parallel + " + ("one-shot peer all-reduce (spark_peer_allreduce)"
                                                       if peer is not None else "NCCL all-reduce")
                                  + " of fp32 partials", "graph": bool(args.tp_graph)},
    }


TP_DEC_M = 8      # decode tokens of the in-kernel all-reduce comparison


def tp_decode_measure(args, rank, world, local):
    """The config-4 stack's layers at decode size (TP_DEC_M bf16 tokens),
    tensor-parallel over the ranks two ways: TPMLP (per layer a gate|up
    launch, a SiLU launch, a down launch and an NCCL all-reduce of the fp32
    partials) and TPMLPFused (ONE launch per layer: gate|up with the SiLU
    epilogue, then the down projection, whose partials are summed over the
    ranks inside the same kernel over peer memory).  Both replay as CUDA
    graphs.  Parity: rank 0's output of the fused layers 0-1 against
    _tp_reference of the unsharded weights, with tp_mlp's bound."""
    import math
    from spark_b200 import ops
    from spark_b200.tp import BatchAllReduce
    device = torch.device("cuda", local)
    g = torch.Generator(device=device).manual_seed(5)
    x0 = torch.randn(TP_DEC_M, TP_H, device=device, generator=g).bfloat16()
    stream = torch.cuda.Stream(device)
    k = max(50, args.steps // 5)
    ar = BatchAllReduce(TP_H, TP_DEC_M)
    out, parity = {}, None
    for kind in ("fused", "nccl"):
        layers, full = _tp_stack(rank, world, device, keep_full=2 if rank == 0 and kind == "fused" else 0,
                                 fused=ar if kind == "fused" else None)
        if kind == "fused":
            with torch.cuda.stream(stream):
                y2 = layers[1](layers[0](x0))
            torch.cuda.synchronize()
            if rank == 0:
                ref = _tp_reference(x0, full)
                err = float((y2.double() - ref).abs().max().item())
                ymax = float(ref.abs().max().item())
                tol = 2.0 ** (math.floor(math.log2(max(ymax, 2.0 ** -20))) - 6)
                parity = {"layers": 2, "max_abs": err, "bound": tol, "ok": bool(err <= tol), "max_abs_ref": ymax}
            del full, y2
        ms, finite = _time_stack(layers, x0, stream, args.warmup, k, world)
        out[kind] = {"ms_per_step": round(ms, 4), "finite": finite,
                     "gpu_launches_per_step": TP_LAYERS * (1 if kind == "fused" else 3)}
        ops.check_device_errors()
        barrier(world)
        del layers
        torch.cuda.empty_cache()
    ar.check()
    ar.close()
    packed_total = TP_LAYERS * 3 * (TP_I * TP_H // 16 * 5)
    peak, peak_kind = peaks()
    for kind, d in out.items():
        per_gpu = packed_total / world / (d["ms_per_step"] * 1e-3) / 1e9
        d["tokens_per_s"] = round(TP_DEC_M / (d["ms_per_step"] * 1e-3), 1)
        d["roofline"] = {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s per GPU",
                         "frac": round(per_gpu / peak, 4), "peak_source": peak_kind}
    return {
        "workload": f"the config-4 stack (32 x SPFP2 gate/up [12288,4096], down [4096,12288]) at {TP_DEC_M} "
                    f"decode tokens, tp{world}", "tp": world, "steps": k,
        "fused": {**out["fused"], "path": "TPMLPFused: one spark_linear_batch_ar launch per layer, the down "
                                          "projection's all-reduce inside the kernel (peer stores + flags)"},
        "nccl": {**out["nccl"], "path": "TPMLP: row-merged gate|up, SiLU, down launches + NCCL all-reduce"},
        "speedup_fused_vs_nccl": round(out["nccl"]["ms_per_step"] / out["fused"]["ms_per_step"], 3),
        "parity": parity,
    }


def run_tp_mlp(args, rank, world, local):
    """--tp-mlp: config 4 alone, its own JSON line."""
    clk = Clocks(local)
    clk.__enter__()
    line = tp_mlp_measure(args, rank, world, local)
    clk.__exit__(None, None, None)
    line["clocks"] = clk.summary()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_tp_decode(args, rank, world, local):
    """--tp-decode: the decode-size tensor-parallel comparison alone, its own JSON line."""
    clk = Clocks(local)
    clk.__enter__()
    line = tp_decode_measure(args, rank, world, local)
    clk.__exit__(None, None, None)
    line["clocks"] = clk.summary()
    if rank == 0:
        print(json.dumps(line), flush=True)


QAT_TOKENS, QAT_H, QAT_I = 8 * 4096, 2560, 9728     # BASELINE config 5 (QAT variant)


def run_qat(args):
    """BASELINE config 5, QAT variant: STE fake-quant forward + backward on the
    gate/up/down projections (ChannelFP2QATLinear, bf16 weights) for a training
    micro-batch of 8 x 4096 tokens, hidden 2560.  Each step bumps the weight
    version (as an optimizer step does), so every step re-runs the SPFP2 window
    search + fake quant of all three weights on the GPU; the linears and their
    backward are torch GEMMs.  Reports the fake-quant kernels alone against the
    HBM roofline (bf16 in + bf16 out per weight) and the whole step."""
    from spark_b200 import ops
    from spark_b200 import quant_linear as ql
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device).manual_seed(11)
    layers = []
    for name, oc, ic in (("gate", QAT_I, QAT_H), ("up", QAT_I, QAT_H), ("down", QAT_H, QAT_I)):
        m = ql.ChannelFP2QATLinear(ic, oc, bias=False, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            m.weight.copy_(torch.randn(oc, ic, device=device, generator=g) * 0.02)
        layers.append(m.train())
    gate, up, down = layers
    x = torch.randn(QAT_TOKENS, QAT_H, device=device, generator=g).bfloat16().requires_grad_(True)

    def step():
        ql.bump_wq_version()
        y = down(torch.nn.functional.silu(gate(x)) * up(x))
        y.float().square().mean().backward()

    def fq():
        for m in layers:
            ops.spfp2_fake_quant(m.weight.detach())

    def timed(fn, k):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(k):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / k

    ms_fq = timed(fq, max(20, args.steps))
    ms_step = timed(step, max(5, args.steps // 20))
    w_down = down.weight.detach()
    ms_24 = timed(lambda: ops.twofour_fake_quant(w_down), max(20, args.steps))
    ops.check_device_errors()
    n_w = sum(m.weight.numel() for m in layers)
    fq_bytes = n_w * 4                                  # bf16 weight in, bf16 fake-quant out
    peak, peak_kind = peaks()
    gbs = fq_bytes / (ms_fq * 1e-3) / 1e9
    gbs24 = w_down.numel() * 4 / (ms_24 * 1e-3) / 1e9
    flops = 3 * 2.0 * QAT_TOKENS * (2 * QAT_I * QAT_H + QAT_H * QAT_I)
    print(json.dumps({
        "metric": "config-5 QAT: SPFP2 STE fake-quant of gate/up/down + micro-batch step", "n_gpus": 1,
        "fake_quant": {"ms": round(ms_fq, 4), "GBps": round(gbs, 1), "weights": n_w,
                       "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                    "frac": round(gbs / peak, 4), "peak_source": peak_kind}},
        "twofour_fake_quant_down": {"ms": round(ms_24, 4), "GBps": round(gbs24, 1)},
        "step": {"ms": round(ms_step, 3), "tokens_per_s": round(QAT_TOKENS / (ms_step * 1e-3), 1),
                 "fake_quant_share": round(ms_fq / ms_step, 4),
                 "gemm_TFLOPs": round(flops / (ms_step * 1e-3) / 1e12, 1),
                 "note": "forward + backward of the three linears are torch (cuBLAS) GEMMs; the STE backward "
                         "is the identity"},
        "config": {"workload": "BASELINE config 5 QAT variant: ChannelFP2QATLinear gate/up [9728,2560], down "
                               "[2560,9728], bf16, micro-batch 8x4096 tokens, hidden 2560, SiLU(gate)*up",
                   "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)"}}), flush=True)


def run_profile_step(args):
    """The config-2 decode step (8 layer copies, 32 row-merged linears) as one
    spark_linear_batch launch, replayed --steps times after 3 warm-up launches;
    prints the step time and GB/s (the bench's headline step without the rest
    of the bench around it, for ncu)."""
    from spark_b200 import ops
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    merged = [merge_layer(L) for L in build_layers(device)]
    g = torch.Generator(device=device).manual_seed(7)
    x = {ic: torch.randn(args.M, ic, device=device, generator=g).bfloat16() for ic in (2560, 4096, 9728)}
    batch = [ops.BatchOp(fmt, wt, x[ic], torch.empty(args.M, oc, dtype=torch.bfloat16, device=device))
             for L in merged for (fmt, _, _, oc, ic, wt) in L.values()]
    for _ in range(3):
        ops.linear_batch(batch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ops.linear_batch(batch)
    e1.record()
    torch.cuda.synchronize()
    ops.check_device_errors()
    ms = e0.elapsed_time(e1) / args.steps
    step_bytes = LAYERS * sum(linear_bytes(f, oc, ic, M=args.M) for _, f, oc, ic in SHAPES)
    print(json.dumps({"profile": "step", "M": args.M, "ms_per_step": round(ms, 4),
                      "GBps": round(step_bytes / (ms * 1e-3) / 1e9, 1)}))


def run_profile(args):
    """Timing of one linear shape on its own (also the target of ncu captures).

    Weight copies rotate so their total exceeds L2 (126 MB) unless --copies is
    given; one pass over the copies is captured as a CUDA graph and replayed
    --steps times.  Prints per-call time, weight GB/s and, for M >= 64,
    TFLOP/s (2*M*oc*ic per call)."""
    from spark_b200 import ops
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    shapes = {"spfp2": (9728, 2560), "fp3": (4096, 2560), "nvfp4": (2560, 4096), "twofour": (2560, 9728)}
    oc, ic = shapes[args.profile]
    oc = args.oc or oc
    ic = args.ic or ic
    nbytes = weight_bytes(args.profile, oc, ic) if args.profile != "twofour" else oc * ic // 32 * 7
    copies = args.copies or max(1, min(64, -(-300_000_000 // nbytes)))
    g = torch.Generator(device=device).manual_seed(3)
    ws = []
    for _ in range(copies):
        W = torch.randn(oc, ic, device=device, generator=g) * 0.02
        s = None
        if args.profile == "spfp2":
            wq, _ = ops.spfp2_pack(W)
        elif args.profile == "fp3":
            wq, s = ops.fp3_pack(W)
        elif args.profile == "nvfp4":
            wq, s = ops.nvfp4_pack(W)
        else:
            wq = ops.twofour_pack(W)
        if args.path == "tiled":
            wq, s = ops.tile_weights(args.profile, wq, s, oc, ic), None
        ws.append((wq, s))
        del W
    x = torch.randn(args.M, ic, device=device, generator=g).bfloat16()
    ys = [torch.empty(args.M, oc, device=device, dtype=torch.bfloat16) for _ in range(copies)]
    stream = torch.cuda.Stream(device)

    def one_pass():
        for k, ((wq, s), y) in enumerate(zip(ws, ys)):
            nxt = ws[(k + 1) % len(ws)][0] if args.prefetch else None
            ops.linear(args.profile, wq, s, x, oc, ic, out=y, tiled=args.path == "tiled", tcgen05=args.path == "tc",
                       prefetch=nxt)

    with torch.cuda.stream(stream):
        one_pass()
        one_pass()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        one_pass()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ops.check_device_errors()
    calls = args.steps * copies
    us = e0.elapsed_time(e1) * 1e3 / calls
    out = {"profile": args.profile, "path": args.path, "M": args.M, "oc": oc, "ic": ic, "copies": copies,
           "calls": calls, "us_per_call": round(us, 3), "weight_GBps": round(nbytes / us / 1e3, 1)}
    if args.M >= 64:
        out["TFLOPs"] = round(2.0 * args.M * oc * ic / us / 1e6, 1)
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="spark_b200", choices=["spark_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--profile", choices=["spfp2", "fp3", "nvfp4", "twofour", "step"],
                    help="run a few plain launches of one linear, or 'step': the batched decode step alone "
                         "(ncu captures)")
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--path", default="tiled", choices=["tiled", "tc", "plain"],
                    help="profile mode: tiled-layout GEMV, tcgen05 kernel, or reference-layout GEMV")
    ap.add_argument("--copies", type=int, default=0, help="profile mode: weight copies to rotate over")
    ap.add_argument("--tp-mlp", action="store_true", help="run the config-4 tensor-parallel MLP stack instead")
    ap.add_argument("--tp-decode", action="store_true",
                    help="run the decode-size tensor-parallel stack (fused vs NCCL all-reduce) instead")
    ap.add_argument("--qat", action="store_true", help="run the config-5 QAT fake-quant measurement instead")
    ap.add_argument("--prefetch", action="store_true", help="profile: each launch prefetches the next copy into L2")
    ap.add_argument("--tp-graph", type=int, default=1, help="tp-mlp: replay each step as a CUDA graph")
    ap.add_argument("--tp-allreduce", default="nccl", choices=["nccl", "peer"],
                    help="tp-mlp: all-reduce of the down projection's partial sums")
    ap.add_argument("--oc", type=int, default=0, help="profile mode: output features")
    ap.add_argument("--ic", type=int, default=0, help="profile mode: input features")
    args = ap.parse_args()
    if args.profile == "step":
        run_profile_step(args)
        return
    if args.profile:
        run_profile(args)
        return
    if args.qat:
        run_qat(args)
        return
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, rank, world)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.tp_mlp:
            run_tp_mlp(args, rank, world, local)
        elif args.tp_decode:
            run_tp_decode(args, rank, world, local)
        else:
            run_gpu(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
