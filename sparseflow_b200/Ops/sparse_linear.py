"""SparseLinear: drop-in for nn.Linear fed by spikes (reference: Ops/sparse_linear.py:68-200, 426+).

Same constructor, ``from_dense`` and parameter keys as nn.Linear; forward takes
[..., in_features] (leading dimensions, e.g. T and N, are folded into rows) and
returns [..., out_features] in x's dtype. On CUDA it runs
``Kernels.linear.sparse_linear_forward``; there is no CPU path.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..Kernels.linear import pack_linear_weight, sparse_linear_forward
from ..Utils.config import PRESCAN_ACTIVITY_EPS


class SparseLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 threshold: float = PRESCAN_ACTIVITY_EPS, return_ms: bool = False, **_ignored):
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.threshold = float(threshold)
        self.return_ms = bool(return_ms)
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.empty(out_features)) if bias else None
        if not bias:
            self.register_parameter("bias", None)
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            bound = 1.0 / math.sqrt(max(in_features, 1))
            nn.init.uniform_(self.bias, -bound, bound)
        self._last_sparse_ms = 0.0
        self._last_dense_ms = 0.0
        self._w_t = None
        self._w_key = None
        self._inference_mode = False
        self.collect_diag = False
        self._last_diag = {}

    @classmethod
    def from_dense(cls, linear: nn.Linear, threshold: float = PRESCAN_ACTIVITY_EPS, return_ms: bool = False,
                   **kwargs) -> "SparseLinear":
        m = cls(linear.in_features, linear.out_features, bias=linear.bias is not None, threshold=threshold,
                return_ms=return_ms, **kwargs).to(linear.weight.device, linear.weight.dtype)
        with torch.no_grad():
            m.weight.copy_(linear.weight)
            if linear.bias is not None:
                m.bias.copy_(linear.bias)
        return m

    def set_inference_mode(self, enabled: bool):
        self._inference_mode = bool(enabled)

    def _packed(self):
        key = (self.weight._version, self.weight.data_ptr(), self.weight.dtype, self.weight.device)
        if self._w_key != key:
            self._w_t = pack_linear_weight(self.weight.detach())
            self._w_key = key
        return self._w_t

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"SparseLinear expects [..., {self.in_features}], got {tuple(x.shape)}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        out = sparse_linear_forward(x2, self.weight.detach(), None if self.bias is None else self.bias.detach(),
                                    threshold=self.threshold, w_t=self._packed(), return_ms=self.return_ms)
        y, ms = out[0], out[1]
        if self.return_ms:
            self._last_sparse_ms = float(ms)
        return y.reshape(*lead, self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"
