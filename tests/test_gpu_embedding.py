"""NVFP4 embedding lookup on the packed table (V3NVFP4Embedding /
spark_nvfp4_embedding): rows bit-exact against the oracle's nvfp4_unpack of
the same codes, ragged dims, repeated and multi-dimensional ids, empty ids, and
out-of-range ids reported through the workspace error word (no fault)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _table(rows, dim, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, dim)) * 0.05).astype(np.float32)
    codes, scales = O.nvfp4_pack(w)
    return codes, scales, O.nvfp4_unpack(codes, scales, rows, dim).reshape(rows, dim)


@pytest.mark.parametrize("rows,dim", [(1000, 256), (317, 100), (64, 2560)])
def test_embedding_rows_match_oracle(rows, dim):
    from spark_b200 import ops
    codes, scales, deq = _table(rows, dim, seed=rows + dim)
    c, s = torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda()
    ids = torch.tensor([[0, rows - 1, 5, 5], [3, 2, 1, rows // 2]], device="cuda")
    out = ops.nvfp4_embedding(c, s, rows, dim, ids)
    assert out.shape == (2, 4, dim) and out.dtype == torch.float32
    want = deq[ids.cpu().numpy()]
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    bf = ops.nvfp4_embedding(c, s, rows, dim, ids, dtype=torch.bfloat16)
    assert torch.equal(bf, torch.from_numpy(want).cuda().bfloat16())
    empty = ops.nvfp4_embedding(c, s, rows, dim, torch.empty(0, dtype=torch.int64, device="cuda"))
    assert empty.shape == (0, dim)


def test_embedding_module_and_loader():
    from torch import nn
    from spark_b200.inference_v3 import V3NVFP4Embedding, build_v3_layers
    rows, dim = 500, 512
    codes, scales, deq = _table(rows, dim, seed=9)

    class Net(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(rows, dim, padding_idx=0)

    net = Net()
    st = {"embed_nvfp4_codes": torch.from_numpy(codes), "embed_nvfp4_scales": torch.from_numpy(scales),
          "embed_meta": torch.tensor([rows, dim])}
    assert build_v3_layers(net, st) == 1
    assert isinstance(net.embed, V3NVFP4Embedding) and net.embed.padding_idx == 0
    ids = torch.randint(0, rows, (3, 7), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    out = net.embed(ids)
    assert out.dtype == torch.float32
    assert np.array_equal(out.cpu().numpy(), deq[ids.cpu().numpy()])


def test_embedding_out_of_range_is_reported_not_faulted():
    from spark_b200 import ops
    rows, dim = 100, 64
    codes, scales, deq = _table(rows, dim, seed=3)
    c, s = torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda()
    ops.check_device_errors()
    out = ops.nvfp4_embedding(c, s, rows, dim, torch.tensor([1, rows, -1, 2], device="cuda"))
    with pytest.raises(RuntimeError, match="out of range"):
        ops.check_device_errors()
    o = out.cpu().numpy()
    assert np.array_equal(o[0], deq[1]) and np.array_equal(o[3], deq[2])
    assert not o[1].any() and not o[2].any()
    ops.check_device_errors()       # the error word was cleared
