"""Multi-step LIF neuron used by the synthetic spiking models.

spikingjelly (the reference's neuron library, pinned 0.0.0.0.14) is not
installed here, so models built for benchmarks and tests use this module: the
same charge / fire / reset rule as spikingjelly's ``LIFNode`` with
``decay_input=True`` and the rule restated in Ops/sparse_fused_conv_lif.py:283-292
of the reference, applied over the leading time axis of a [T, N, ...] input
(``step_mode='m'``). On CUDA a multi-step call is one ``sf_lif_multistep``
launch (v kept in registers across the steps); on CPU the same formula runs
as tensor code.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn


class LIFNode(nn.Module):
    def __init__(self, tau: float = 2.0, v_threshold: float = 1.0, v_reset: Optional[float] = 0.0,
                 decay_input: bool = True, detach_reset: bool = False, step_mode: str = "m"):
        super().__init__()
        self.tau = float(tau)
        self.v_threshold = float(v_threshold)
        self.v_reset = v_reset
        self.decay_input = bool(decay_input)
        self.detach_reset = detach_reset
        self.step_mode = step_mode
        self.v = None
        # Opt-in: a 5-D multi-step call on CUDA also writes the spikes' event masks
        # (sf_lif_multistep_events) and attaches them to the output, so a following
        # SparseConv2d given that very tensor skips its mask pass over the spikes.
        self.emit_event_masks = False

    def reset(self):
        self.v = None

    def _step(self, x: torch.Tensor) -> torch.Tensor:
        vr = 0.0 if self.v_reset is None else float(self.v_reset)
        if self.v is None or self.v.shape != x.shape:
            self.v = torch.full_like(x, vr, dtype=torch.float32)
        v = self.v
        xf = x.float()
        if self.decay_input:
            v_tmp = v + (xf - (v - vr)) / self.tau
        else:
            v_tmp = v - (v - vr) / self.tau + xf
        spike = (v_tmp >= self.v_threshold).to(torch.float32)
        if self.v_reset is None:
            self.v = v_tmp - spike * self.v_threshold
        else:
            self.v = torch.where(spike.bool(), torch.full_like(v_tmp, vr), v_tmp)
        return spike.to(x.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.step_mode == "s":
            return self._step(x)
        if x.is_cuda:
            return self._multistep_cuda(x)
        return torch.stack([self._step(x[t]) for t in range(x.shape[0])], 0)

    def _multistep_cuda(self, x: torch.Tensor) -> torch.Tensor:
        """All T steps in one sf_lif_multistep launch (v kept in registers across steps)."""
        from .. import _lib
        vr = 0.0 if self.v_reset is None else float(self.v_reset)
        x = x.contiguous()
        if self.v is None or self.v.shape != x.shape[1:] or self.v.device != x.device:
            self.v = torch.full(x.shape[1:], vr, dtype=torch.float32, device=x.device)
        else:
            self.v = self.v.float().contiguous()
        spikes = torch.empty_like(x)
        if self.emit_event_masks and x.dim() == 5:
            from ..Kernels.fused_conv_lif import attach_event_masks
            t, n, c, h, w = x.shape
            masks = torch.empty(_lib.event_masks_bytes(t * n, c, h, w) // 8, dtype=torch.int64, device=x.device)
            _lib.lif_multistep_events(x, self.v, spikes, masks, self.tau, self.v_threshold, self.v_reset,
                                      self.decay_input)
            attach_event_masks(spikes, masks)
            return spikes
        _lib.lif_multistep(x, self.v, spikes, self.tau, self.v_threshold, self.v_reset, self.decay_input)
        return spikes

    def extra_repr(self):
        return f"tau={self.tau}, v_threshold={self.v_threshold}, v_reset={self.v_reset}, step_mode={self.step_mode}"


def reset_net(model: nn.Module) -> None:
    """Clear the membrane state of every stateful module (spikingjelly's functional.reset_net)."""
    for m in model.modules():
        if hasattr(m, "reset") and callable(m.reset) and m is not model:
            m.reset()
