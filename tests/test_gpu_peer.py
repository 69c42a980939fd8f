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
