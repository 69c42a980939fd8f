"""Tensor-parallel MLP and layer-split packing over one node.

The path shards the way the model does (no collective is invented):
* gate_proj / up_proj are column-parallel: rank r keeps output rows
  [r*I/W, (r+1)*I/W) -- a contiguous byte range of the packed weight;
* down_proj is row-parallel: rank r keeps input columns [r*I/W, (r+1)*I/W),
  cut on 16-weight boundaries so SPFP2 block pairs never straddle it; each
  rank's partial [M, H] sums meet in one all-reduce (NCCL over NVLink on the
  GPUs, gloo in the CPU tests);
* whole-model pack / quantize is independent per layer: layers go to ranks
  round-robin and the packed bytes are gathered on the host.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

ALIGN = 16      # SPFP2 pairs, FP3 groups and 2:4 pairs of 16-blocks stay whole


def shard_bounds(n: int, rank: int, world: int, align: int = ALIGN) -> tuple[int, int]:
    """[lo, hi) of rank's share of n rows or columns, cut on `align` boundaries."""
    if n % (world * align):
        raise ValueError(f"{n} does not split into {world} shards of whole {align}-blocks")
    step = n // world
    return rank * step, (rank + 1) * step


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Column-parallel share (gate / up): output rows of rank."""
    lo, hi = shard_bounds(w.shape[0], rank, world)
    return w[lo:hi]


def shard_cols(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Row-parallel share (down): input columns of rank."""
    lo, hi = shard_bounds(w.shape[1], rank, world)
    return w[:, lo:hi]


# Peer allocations mapped into this process: IPC handle -> [base pointer,
# users].  A handle names a whole allocation, and one allocation can hold
# several shared buffers; CUDA maps it once per process.
_IPC_MAPS: dict[bytes, list] = {}


def _ipc_map(handle: bytes) -> int:
    import ctypes
    from . import _lib
    m = _IPC_MAPS.get(handle)
    if m is None:
        p = ctypes.c_void_p()
        _lib.call("spark_ipc_open", (ctypes.c_uint8 * 64).from_buffer_copy(handle), 0, ctypes.byref(p))
        m = _IPC_MAPS[handle] = [p.value, 0]
    m[1] += 1
    return m[0]


def _ipc_unmap(handle: bytes) -> None:
    import ctypes
    from . import _lib
    m = _IPC_MAPS[handle]
    m[1] -= 1
    if m[1] == 0:
        _lib.call("spark_ipc_close", ctypes.c_void_p(m[0]), 0)
        del _IPC_MAPS[handle]


def _share(tensors: list[torch.Tensor], rank: int, world: int, group=None) -> tuple[list[list[int]], list[bytes]]:
    """Exchange the CUDA IPC handles of this rank's `tensors` over the group and
    map every other rank's: returns, per tensor, the device address of every
    rank's copy (this rank's own pointer at index `rank`) and the handles
    opened (to _ipc_unmap on close)."""
    import ctypes
    from . import _lib

    def handle(t):
        h = (ctypes.c_uint8 * 64)()
        off = ctypes.c_int64(0)
        _lib.call("spark_ipc_handle", ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off))
        return bytes(h), off.value

    mine = [handle(t) for t in tensors]
    every = [mine]
    if world > 1:
        every = [None] * world
        dist.all_gather_object(every, mine, group=group)
    ptrs: list[list[int]] = [[] for _ in tensors]
    opened: list[bytes] = []
    for r, theirs in enumerate(every):
        for i, (h, off) in enumerate(theirs):
            if r == rank:
                ptrs[i].append(tensors[i].data_ptr())
                continue
            ptrs[i].append(_ipc_map(h) + off)
            opened.append(h)
    return ptrs, opened


class PeerAllReduce:
    """One-shot all-reduce of per-rank partial sums over peer memory
    (spark_peer_allreduce): the NCCL all-reduce after the row-parallel down
    projection, done by this library's kernel on NVLink peer loads.

    Each rank owns two alternating partial buffers of `numel` elements and a
    flag array; their CUDA IPC handles are exchanged once through the process
    group, so every rank maps every other rank's buffers.  Use:
    ``buf = ar.buffer()``, write this rank's partial into it (e.g. as the
    down projection's output), then ``ar(out)``.  Every rank must make the same
    sequence of calls; a captured CUDA graph must hold an even number of them
    (the buffers alternate by call)."""

    def __init__(self, numel: int, dtype=torch.float32, group=None):
        import ctypes
        from . import _lib
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("PeerAllReduce: at most 8 ranks")
        self.numel = numel
        self.dtype = dtype
        self._group = group
        dev = torch.device("cuda", torch.cuda.current_device())
        L = _lib.lib()
        self._lib, self._ct = L, ctypes
        n_pad = (numel + 7) // 8 * 8
        self.local = torch.zeros(2, n_pad, dtype=dtype, device=dev)
        self.flags = torch.zeros(L.spark_peer_flags_count(self.world), dtype=torch.int32, device=dev)
        self.epochs = torch.zeros(L.spark_peer_flags_count(1), dtype=torch.int32, device=dev)
        self.err = torch.zeros(64, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        (bufs, flags), self._opened = _share([self.local, self.flags], self.rank, self.world, group)
        half = n_pad * self.local.element_size()
        P = ctypes.c_void_p * self.world
        self._bufs = [P(*[b + k * half for b in bufs]) for k in (0, 1)]
        self._flags = P(*flags)
        self.calls = 0
        if self.world > 1:
            dist.barrier(group=group)

    def buffer(self) -> torch.Tensor:
        """This rank's partial buffer for the next call."""
        return self.local[self.calls % 2][: self.numel]

    def __call__(self, out: torch.Tensor) -> torch.Tensor:
        from . import _lib, ops
        if out.numel() != self.numel or not out.is_contiguous():
            raise ValueError("PeerAllReduce: out must be a contiguous tensor of numel elements")
        ct = self._ct
        _lib.call("spark_peer_allreduce", ct.cast(self._bufs[self.calls % 2], ct.c_void_p),
                  ct.cast(self._flags, ct.c_void_p), self.world, self.rank, self.numel, ops._dt(self.local),
                  ct.c_void_p(out.data_ptr()), ops._dt(out), ct.c_void_p(self.epochs.data_ptr()),
                  ct.c_void_p(self.err.data_ptr()), ops._stream(out))
        self.calls += 1
        return out

    def check(self) -> None:
        """Raise if a call's barrier gave up waiting for a peer (synchronises)."""
        from . import _lib
        _lib.call("spark_workspace_check", self._ct.c_void_p(self.err.data_ptr()),
                  self._ct.c_void_p(torch.cuda.current_stream().cuda_stream))

    def close(self) -> None:
        """Unmap the other ranks' buffers.  Every rank calls it: after the local
        synchronize, a barrier over the group makes sure no peer's last call still
        reads this rank's buffers before any rank unmaps or frees them."""
        torch.cuda.synchronize()
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=self._group)
        for h in self._opened:
            _ipc_unmap(h)
        self._opened = []


class TPMLP(torch.nn.Module):
    """One SPFP2 MLP layer, tensor-parallel over the default process group:
    y = all_reduce( down_r( silu(gate_r x) * up_r x ) ).

    The shares are packed on this rank's GPU from the full fp32 weights (or
    given already packed via from_packed)."""

    def __init__(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, rank: int = 0, world: int = 1,
                 group=None, peer: PeerAllReduce | None = None):
        """peer: a PeerAllReduce sized M x hidden replaces the NCCL all-reduce
        (the down projection then writes its fp32 partial straight into the
        peer buffer)."""
        super().__init__()
        self.peer = peer
        from .inference_v3 import V3MergedLinear, V3PackedLinear
        from . import ops
        self.world, self.group = world, group
        g, u, d = shard_rows(gate, rank, world), shard_rows(up, rank, world), shard_cols(down, rank, world)
        gate_l = V3PackedLinear("spfp2", ops.spfp2_pack(g.contiguous())[0], g.shape[0], g.shape[1])
        up_l = V3PackedLinear("spfp2", ops.spfp2_pack(u.contiguous())[0], u.shape[0], u.shape[1])
        # gate and up read the same x: one row-merged weight, one launch
        self.gate_up = V3MergedLinear([gate_l, up_l])
        self.down = V3PackedLinear("spfp2", ops.spfp2_pack(d.contiguous())[0], d.shape[0], d.shape[1])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from . import ops
        g, u = self.gate_up(x)
        h = ops.silu_mul(g, u)
        if self.peer is not None:
            d = self.down
            d(h, out=self.peer.buffer().view(h.shape[0], d.out_features))
            return self.peer(torch.empty(h.shape[0], d.out_features, dtype=x.dtype, device=x.device))
        if self.world == 1:
            return self.down(h)
        # the ranks' partial sums meet in fp32 (as in the peer path), rounded
        # to the activation dtype once, after the sum
        d = self.down
        y = d(h, out=torch.empty(h.shape[0], d.out_features, dtype=torch.float32, device=x.device))
        dist.all_reduce(y, group=self.group)
        return y.to(x.dtype)


class BatchAllReduce:
    """The shared buffers of spark_linear_batch_ar: the all-reduce of one op of
    a batched decode launch (width `oc`, up to `max_tokens` tokens) done
    inside that launch over peer memory.

    Every rank owns a receive buffer (2 call parities x ranks x row groups x
    tokens x 16 words of 8 bytes: an fp32 value tagged with the call number)
    and a call counter; the buffers' CUDA IPC handles are exchanged once
    through the process group.  The counter lives on the device, so calls can
    be captured in a CUDA graph and replayed any number of times.  Every rank
    must make the same sequence of calls, each with the same batch shapes."""

    def __init__(self, oc: int, max_tokens: int = 16, group=None):
        from . import _lib
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("BatchAllReduce: at most 8 ranks")
        if not 1 <= max_tokens <= 16:
            raise ValueError("BatchAllReduce: 1 to 16 tokens")
        self.oc, self.max_tokens, self._group = oc, max_tokens, group
        dev = torch.device("cuda", torch.cuda.current_device())
        n = _lib.lib().spark_batch_ar_recv_bytes(self.world, max_tokens, oc)
        self.recv = torch.zeros(n // 8, dtype=torch.int64, device=dev)
        self.counter = torch.zeros(4, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        (self._recv,), self._opened = _share([self.recv], self.rank, self.world, group)
        if self.world > 1:
            dist.barrier(group=group)

    def __call__(self, batch: list, op: int, stream=None) -> None:
        """Run `batch` (ops.BatchOp list) in one launch; op `op`'s y receives the
        sum over the ranks (fp32, rank order 0..W-1) plus its bias."""
        from . import ops
        y, M = batch[op].y, batch[op].x.shape[0]
        if batch[op].silu or y.shape[1] != self.oc or M > self.max_tokens:
            raise ValueError(f"BatchAllReduce: op {op} must be a plain linear of width {self.oc} "
                             f"on at most {self.max_tokens} tokens")
        ops.linear_batch_allreduce(batch, op, self.world, self.rank, self._recv, self.counter, stream=stream)

    def check(self) -> None:
        """Raise if a launch gave up waiting for a peer (synchronises)."""
        from . import ops
        ops.check_device_errors()

    def close(self) -> None:
        """Unmap the other ranks' buffers (every rank calls it; see PeerAllReduce.close)."""
        torch.cuda.synchronize()
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=self._group)
        for h in self._opened:
            _ipc_unmap(h)
        self._opened = []


class TPMLPFused(torch.nn.Module):
    """TPMLP in ONE kernel launch: gate|up with the SiLU epilogue, then the
    row-parallel down projection, whose ranks' fp32 partials are summed inside
    the same launch over peer memory (BatchAllReduce): no NCCL call and no
    separate all-reduce kernel.  Decode sizes: bf16 x [M, H], M <= max_tokens."""

    def __init__(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, rank: int = 0, world: int = 1,
                 group=None, max_tokens: int = 16, fmt: str = "spfp2", ar: BatchAllReduce | None = None):
        """ar: a BatchAllReduce of width hidden shared with other layers (the
        calls run one after another on a stream); by default the layer owns one."""
        super().__init__()
        from . import ops
        from .inference_v3 import V3GateUpSiLU, V3PackedLinear

        def packed(w):
            w = w.contiguous()
            if fmt == "spfp2":
                return V3PackedLinear(fmt, ops.spfp2_pack(w)[0], w.shape[0], w.shape[1])
            c, sc = ops.nvfp4_pack(w) if fmt == "nvfp4" else ops.fp3_pack(w)
            return V3PackedLinear(fmt, c, w.shape[0], w.shape[1], scales=sc)

        g, u, d = shard_rows(gate, rank, world), shard_rows(up, rank, world), shard_cols(down, rank, world)
        self.gate_up = V3GateUpSiLU(packed(g), packed(u))
        self.down = packed(d)
        self.hidden, self.inter = down.shape[0], g.shape[0]
        if ar is not None and (ar.oc != self.hidden or ar.world != world):
            raise ValueError("TPMLPFused: the shared BatchAllReduce has another width or rank count")
        self.ar = ar if ar is not None else BatchAllReduce(self.hidden, max_tokens, group)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        from . import ops
        M = x.shape[0]
        h = torch.empty(M, self.inter, dtype=torch.bfloat16, device=x.device)
        y = out if out is not None else torch.empty(M, self.hidden, dtype=x.dtype, device=x.device)
        gu, dn = self.gate_up.merged, self.down
        self.ar([ops.BatchOp(gu.fmt, gu.w_tiled, x, h, bias=gu.bias, silu=True),
                 ops.BatchOp(dn.fmt, dn.w_tiled, h, y, bias=dn.bias, deps=[0])], 1)
        return y


def pack_layers_split(weights: list[torch.Tensor], pack: Callable[[torch.Tensor], torch.Tensor], rank: int,
                      world: int, group=None) -> list[torch.Tensor]:
    """Pack layer l on rank l % world, then gather every layer's bytes to every
    rank (host memory).  `pack` maps a weight to its packed uint8 tensor."""
    mine = {l: pack(w).detach().cpu() for l, w in enumerate(weights) if l % world == rank}
    if world == 1:
        return [mine[l] for l in range(len(weights))]
    gathered: list = [None] * world
    dist.all_gather_object(gathered, mine, group=group)
    out = {}
    for part in gathered:
        out.update(part)
    return [out[l] for l in range(len(weights))]
