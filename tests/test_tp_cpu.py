"""Tensor-parallel sharding and the layer-split pack with world_size-2 gloo
ranks on the CPU.  The per-rank math runs on the oracle (decode in C, fp64
matmul), so the test checks the partition itself: column-parallel gate/up,
row-parallel down cut on whole 16-blocks, one all-reduce of the partial sums,
and per-layer packing gathered from both ranks."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from spark_b200.tp import pack_layers_split, shard_bounds, shard_cols, shard_rows


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dec(w: np.ndarray) -> np.ndarray:
    oc, ic = w.shape
    return O.unpack_blockwise_paired(O.pack_blockwise_paired(w)[0], oc * ic).reshape(oc, ic).astype(np.float64)


def _silu(v):
    return v / (1.0 + np.exp(-v))


def _weights():
    g = np.random.RandomState(4)
    H, I = 64, 256
    return (g.randn(I, H).astype(np.float32) * 0.05, g.randn(I, H).astype(np.float32) * 0.05,
            g.randn(H, I).astype(np.float32) * 0.05, g.randn(3, H).astype(np.float32))


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        gate, up, down, x = _weights()
        gr = shard_rows(torch.from_numpy(gate), rank, world).numpy()
        ur = shard_rows(torch.from_numpy(up), rank, world).numpy()
        dr = shard_cols(torch.from_numpy(down), rank, world).numpy()
        h = _silu(x @ _dec(gr).T) * (x @ _dec(ur).T)
        part = torch.from_numpy(h @ _dec(dr).T)
        dist.all_reduce(part)
        layers = [torch.from_numpy(np.random.RandomState(10 + l).randn(16, 64).astype(np.float32)) for l in range(5)]
        packed = pack_layers_split(layers, lambda w: torch.from_numpy(O.pack_blockwise_paired(w.numpy())[0]),
                                   rank, world)
        q.put((rank, part.numpy(), [p.numpy() for p in packed]))
    finally:
        dist.destroy_process_group()


def test_tp_mlp_and_layer_split_pack_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gate, up, down, x = _weights()
    # unsharded reference: the column / row cuts are on 16-block boundaries, so
    # every rank's blocks are the full weight's blocks
    want = (_silu(x @ _dec(gate).T) * (x @ _dec(up).T)) @ _dec(down).T
    for rank, y, packed in res:
        assert np.allclose(y, want, rtol=1e-12, atol=1e-12), rank
        for l, p in enumerate(packed):
            w = np.random.RandomState(10 + l).randn(16, 64).astype(np.float32)
            assert np.array_equal(p, O.pack_blockwise_paired(w)[0]), (rank, l)


def test_shard_bounds_alignment():
    assert shard_bounds(12288, 7, 8) == (10752, 12288)
    assert shard_bounds(9728, 1, 8) == (1216, 2432)
    try:
        shard_bounds(100, 0, 2)
    except ValueError:
        pass
    else:
        raise AssertionError("unaligned split accepted")
