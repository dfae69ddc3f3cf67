"""FusedSparseConvLIF: stateful conv + (folded BN) + LIF module.

Reference: Ops/sparse_fused_conv_lif.py:24-302. Kept: constructor arguments,
``from_conv_and_lif`` (:110-135), ``v`` as the membrane state allocated as
zeros on a shape change (:202-203), 5-D multi-step and 4-D single-step
inputs (:184-197), spikes in the input dtype, ValueError for other ranks
(:189), ``_last_sparse_ms``. Added: ``from_conv_bn_lif`` folds an eval-mode
BatchNorm2d into the weights, which is the conv -> BN -> LIF block of
spiking ResNets. The whole T loop runs in one native launch.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from ..Kernels.fused_conv_lif import SUPPORTED_LIF_PATTERNS, fold_bn, sparse_fused_conv_lif_forward
from ..Kernels.conv2d import output_hw, pack_weight


class FusedSparseConvLIF(nn.Module):
    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias=True, tau: float = 2.0, v_threshold: float = 1.0, v_reset: Optional[float] = 0.0,
                 detach_reset: bool = False, decay_input: bool = True, backend: str = "torch",
                 threshold: float = 1e-6, block_size=None, return_ms: bool = False):
        super().__init__()
        pair = lambda v: v if isinstance(v, tuple) else (v, v)  # noqa: E731
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = pair(kernel_size)
        self.stride = pair(stride)
        self.padding = pair(padding)
        self.dilation = pair(dilation)
        self.groups = groups
        self.tau = float(tau)
        self.v_threshold = float(v_threshold)
        self.v_reset = v_reset
        self.detach_reset = detach_reset
        self.decay_input = bool(decay_input)
        self.backend = backend
        self.threshold = float(threshold)
        self.block_size = block_size
        self.return_ms = bool(return_ms)
        # Opt-in: the same kernel also writes the output spikes' event masks and
        # attaches them to the spikes, so a following SparseConv2d skips its mask
        # pass. Measured on the C3 layer: +0.126 ms to emit vs 0.063 ms saved
        # downstream, hence off by default.
        self.emit_event_masks = False
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels // groups, *self.kernel_size))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_channels))
        else:
            self.register_parameter("bias", None)
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)
        self.v = None
        self._last_sparse_ms = 0.0
        self._w_packed = None
        self._w_key = None
        self.collect_diag = False
        self.profile_runtime = False
        self._inference_mode = False
        if (self.kernel_size[0], self.stride[0], self.padding[0]) not in SUPPORTED_LIF_PATTERNS or groups != 1 \
                or self.dilation != (1, 1):
            raise ValueError("FusedSparseConvLIF supports 3x3/s1/p1 and 1x1/s1/p0 convolutions with groups=1")

    def reset(self):
        self.v = None

    def set_inference_mode(self, enabled: bool):
        self._inference_mode = bool(enabled)

    @classmethod
    def from_conv_and_lif(cls, conv: nn.Conv2d, lif_node, block_size=None, threshold: float = 1e-6,
                          return_ms: bool = False):
        mod = cls(conv.in_channels, conv.out_channels, conv.kernel_size, conv.stride, conv.padding,
                  conv.dilation, conv.groups, bias=conv.bias is not None,
                  tau=float(getattr(lif_node, "tau", 2.0)),
                  v_threshold=float(getattr(lif_node, "v_threshold", 1.0)),
                  v_reset=getattr(lif_node, "v_reset", 0.0),
                  detach_reset=bool(getattr(lif_node, "detach_reset", False)),
                  decay_input=bool(getattr(lif_node, "decay_input", True)),
                  threshold=threshold, block_size=block_size, return_ms=return_ms)
        mod = mod.to(conv.weight.device)
        mod.weight.data.copy_(conv.weight.data)
        if conv.bias is not None:
            mod.bias.data.copy_(conv.bias.data)
        return mod

    @classmethod
    def from_conv_bn_lif(cls, conv: nn.Conv2d, bn: nn.BatchNorm2d, lif_node, **kw):
        """conv -> eval-mode BN -> LIF as one module (BN folded into weight and bias)."""
        mod = cls.from_conv_and_lif(conv, lif_node, **kw)
        w, b = fold_bn(conv.weight, conv.bias, bn)
        mod.weight = nn.Parameter(w.to(conv.weight.device))
        mod.bias = nn.Parameter(b.to(conv.weight.device))
        return mod

    def _packed(self):
        key = (self.weight._version, self.weight.data_ptr(), self.weight.dtype)
        if self._w_packed is None or self._w_key != key:
            self._w_packed = pack_weight(self.weight.data)
            self._w_key = key
        return self._w_packed

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() not in (4, 5):
            raise ValueError(f"Expected 4D or 5D input, got {x.dim()}D")
        n, h, w = (x.shape[1], x.shape[3], x.shape[4]) if x.dim() == 5 else (x.shape[0], x.shape[2], x.shape[3])
        ho, wo = output_hw(h, w, self.kernel_size[0], self.stride[0], self.padding[0])
        shape = (n, self.out_channels, ho, wo)
        if self.v is None or tuple(self.v.shape) != shape or self.v.device != x.device:
            self.v = torch.zeros(shape, dtype=torch.float32, device=x.device)
        spikes, v_next, ms = sparse_fused_conv_lif_forward(
            x, self.v, self.weight, self.bias, self.tau, self.v_threshold, self.v_reset, self.decay_input,
            kernel_size=self.kernel_size[0], stride=self.stride[0], padding=self.padding[0],
            w_packed=self._packed(), return_ms=self.return_ms, emit_event_masks=self.emit_event_masks)
        self.v = v_next
        self._last_sparse_ms = ms
        return spikes

    def extra_repr(self):
        bs = self.block_size if self.block_size is not None else "auto"
        return (f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, stride={self.stride}, "
                f"padding={self.padding}, tau={self.tau}, v_threshold={self.v_threshold}, "
                f"v_reset={self.v_reset}, block_size={bs}, fused=True")
