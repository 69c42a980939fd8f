"""Drop-in for 02_model/fp3_linear.py: the FP3 E1M1 QAT layer, with its
fake-quant on the sm_100a kernels.

The fake-quant cache version is the single counter that
spark_b200.quant_linear.bump_wq_version() advances (the reference keeps a
separate, never-bumped copy here, fp3_linear.py:23, so its FP3 cache went stale
across optimizer steps).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from .fp3 import fp3_fake_quant, fp3_pack

_WQ_VERSION = [0]            # shared with quant_linear.bump_wq_version


class FP3QATLinear(nn.Module):
    """fp3_linear.py:25-62: STE fake-quant forward with a per-version cache;
    quantize() writes the nibble codes and e4m3 scales."""

    force_fake_quant: bool = False

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=dtype))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, device=device, dtype=dtype))
        else:
            self.register_parameter("bias", None)
        self._wq_cache: Optional[torch.Tensor] = None
        self._wq_ver: int = -1

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.training or self.force_fake_quant:
            if self._wq_cache is None or self._wq_ver != _WQ_VERSION[0]:
                with torch.no_grad():
                    self._wq_cache = fp3_fake_quant(self.weight.detach()).to(self.weight.dtype)
                self._wq_ver = _WQ_VERSION[0]
            w_eff = self.weight + (self._wq_cache - self.weight).detach()
            return nn.functional.linear(x, w_eff, self.bias)
        return nn.functional.linear(x, self.weight, self.bias)

    def quantize(self):
        codes, scales = fp3_pack(self.weight.data.detach().float())
        self._fp3_codes = codes
        self._fp3_scales = scales
