"""One-shot peer all-reduce (spark_peer_allreduce / tp.PeerAllReduce) and the
tensor-parallel MLP on it.  One rank on one GPU checks the buffer alternation
and the copy path; with two or more GPUs, two ranks (one process per GPU,
NCCL process group with a short timeout) check exact fp32 sums against the
expected values and the TP MLP against its NCCL all-reduce form."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_allreduce_single_rank_alternates_buffers():
    from spark_b200.tp import PeerAllReduce
    torch.cuda.set_device(0)
    ar = PeerAllReduce(1003, dtype=torch.float32)
    for it in range(5):
        buf = ar.buffer()
        assert buf.numel() == 1003
        src = torch.arange(1003, device="cuda", dtype=torch.float32) * (it + 1) / 7.0
        buf.copy_(src)
        out = ar(torch.empty(1003, device="cuda", dtype=torch.bfloat16))
        assert torch.equal(out, src.bfloat16())
    assert ar.calls == 5 and ar.buffer().data_ptr() != ar.local[0].data_ptr()
    ar.check()
    ar.close()


def _fused_reference(mlp, x):
    """This rank's partial of the fused MLP: the same two-op batch through
    spark_linear_batch with the down projection's output kept in fp32 (the
    same plan, so the same bits as the partial the fused launch exchanges)."""
    from spark_b200 import ops
    gu, dn = mlp.gate_up.merged, mlp.down
    M = x.shape[0]
    h = torch.empty(M, mlp.inter, dtype=torch.bfloat16, device=x.device)
    part = torch.empty(M, mlp.hidden, dtype=torch.float32, device=x.device)
    ops.linear_batch([ops.BatchOp(gu.fmt, gu.w_tiled, x, h, silu=True),
                      ops.BatchOp(dn.fmt, dn.w_tiled, h, part, deps=[0])])
    return part


def _graph_of(fn):
    """Capture fn() (after a warm-up call on the capture stream); returns the
    graph and fn's output tensor inside it."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = fn()
    return g, out


@pytest.mark.parametrize("M", [1, 6, 16])
def test_batch_allreduce_single_rank(M):
    """One rank: the fused all-reduce is the identity on the fp32 partial, so
    the one-launch MLP equals the batch with an fp32 down output rounded
    once; repeated calls and graph replays keep it (the launch counter
    alternates the receive slots)."""
    from spark_b200 import ops
    from spark_b200.tp import TPMLPFused
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda").manual_seed(11 + M)
    H, I = 1024, 2048
    gate = torch.randn(I, H, device="cuda", generator=gen) * 0.03
    up = torch.randn(I, H, device="cuda", generator=gen) * 0.03
    down = torch.randn(H, I, device="cuda", generator=gen) * 0.03
    mlp = TPMLPFused(gate, up, down)
    for it in range(3):
        x = torch.randn(M, H, device="cuda", generator=gen).bfloat16()
        y = mlp(x)
        assert torch.equal(y, _fused_reference(mlp, x).bfloat16()), it
    x = torch.randn(M, H, device="cuda", generator=gen).bfloat16()
    want = _fused_reference(mlp, x).bfloat16()
    g, out = _graph_of(lambda: mlp(x))
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    mlp.ar.check()
    ops.check_device_errors()
    del g
    mlp.ar.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from spark_b200 import ops
        from spark_b200.tp import TPMLP, PeerAllReduce
        n = 64 * 512
        ar = PeerAllReduce(n, dtype=torch.float32)
        ok = True
        for it in range(4):
            base = torch.arange(n, device="cuda", dtype=torch.float32) % 97
            ar.buffer().copy_(base * (rank + 1) + it)
            out = ar(torch.empty(n, device="cuda", dtype=torch.float32))
            want = base * sum(r + 1 for r in range(world)) + it * world
            ok &= bool(torch.equal(out, want))
        ar.check()
        # TP MLP: peer all-reduce vs NCCL all-reduce on the same shards
        gen = torch.Generator(device="cuda").manual_seed(5)
        H, I = 512, 1024
        gate = torch.randn(I, H, device="cuda", generator=gen) * 0.05
        up = torch.randn(I, H, device="cuda", generator=gen) * 0.05
        down = torch.randn(H, I, device="cuda", generator=gen) * 0.05
        x = torch.randn(64, H, device="cuda", generator=gen).bfloat16()
        ar2 = PeerAllReduce(64 * H, dtype=torch.float32)
        a = TPMLP(gate, up, down, rank, world, peer=ar2)(x)
        b = TPMLP(gate, up, down, rank, world)(x)
        diff = (a.float() - b.float()).abs().max().item()
        scale = b.float().abs().max().item()
        ar2.check()
        torch.cuda.synchronize()
        ar.close()
        ar2.close()
        dist.barrier()
        q.put((rank, ok, diff, scale))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_allreduce_two_ranks_and_tp_mlp():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, diff, scale in res:
        assert ok, rank
        # bf16 outputs of two reduction orders: within a few bf16 ulps of the magnitude
        assert diff <= 2e-2 * max(scale, 1.0), (rank, diff, scale)


def _rank_fused(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from spark_b200 import ops
        from spark_b200.tp import TPMLP, TPMLPFused
        gen = torch.Generator(device="cuda").manual_seed(9)
        H, I = 1024, 4096
        gate = torch.randn(I, H, device="cuda", generator=gen) * 0.03
        up = torch.randn(I, H, device="cuda", generator=gen) * 0.03
        down = torch.randn(H, I, device="cuda", generator=gen) * 0.03
        mlp = TPMLPFused(gate, up, down, rank, world)
        res = []
        for M in (1, 6, 16):
            for it in range(3):
                x = torch.randn(M, H, device="cuda", generator=gen).bfloat16()
                y = mlp(x)
                # the exact expectation: the ranks' fp32 partials summed in rank order
                part = _fused_reference(mlp, x)
                parts = [torch.empty_like(part) for _ in range(world)]
                dist.all_gather(parts, part)
                acc = torch.zeros_like(part)
                for p in parts:
                    acc = acc + p
                exact = torch.equal(y, acc.bfloat16())
                ys = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(ys, y)
                same = all(torch.equal(ys[0], t) for t in ys)
                nccl = TPMLP(gate, up, down, rank, world)(x) if it == 0 else y
                diff = (y.float() - nccl.float()).abs().max().item()
                res.append((M, it, exact, same, diff, nccl.float().abs().max().item()))
        # graph replay: two fused launches per replay, each replay checked
        x1 = torch.randn(8, H, device="cuda", generator=gen).bfloat16()
        x2 = torch.randn(8, H, device="cuda", generator=gen).bfloat16()
        w1, w2 = mlp(x1).clone(), mlp(x2).clone()
        g, (o1, o2) = _graph_of(lambda: (mlp(x1), mlp(x2)))
        replay_ok = True
        for _ in range(3):
            g.replay()
            torch.cuda.synchronize()
            replay_ok &= bool(torch.equal(o1, w1) and torch.equal(o2, w2))
        mlp.ar.check()
        ops.check_device_errors()
        del g
        mlp.ar.close()
        dist.barrier()
        q.put((rank, res, replay_ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_batch_allreduce_two_ranks():
    """The tensor-parallel MLP in one launch per rank (gate|up + SiLU, then the
    K-sharded down projection all-reduced inside the kernel over peer memory):
    bit-exact against the rank-order sum of the ranks' fp32 partials, the same
    bits on both ranks, close to the NCCL-all-reduce TPMLP, and stable under
    repeated calls, changing token counts and CUDA graph replay."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fused, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, res, replay_ok in out:
        assert replay_ok, rank
        for M, it, exact, same, diff, scale in res:
            assert exact and same, (rank, M, it, exact, same)
            # two kernels' decode orders and bf16 roundings: a few bf16 ulps of the magnitude
            assert diff <= 2e-2 * max(scale, 1.0), (rank, M, it, diff, scale)
