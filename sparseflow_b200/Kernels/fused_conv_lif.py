"""Fused sparse conv + bias + LIF over all time steps (one native launch).

Reference: Kernels/fused_conv_lif.py:310-484 (``sparse_fused_conv_lif_forward``,
one Triton launch per step, currently unimportable) and the LIF semantics of
Ops/sparse_fused_conv_lif.py:271-293:
    decay_input: v_tmp = v + (I - (v - v_reset)) / tau
    otherwise:   v_tmp = v - (v - v_reset) / tau + I
    spike = v_tmp >= v_threshold
    hard reset (v_reset given): v = v_reset where spike, else v_tmp
    soft reset (v_reset None):  v = v_tmp - spike * v_threshold  (v_reset taken as 0 above)
The native kernel keeps v in registers across the T steps, so the membrane
state crosses HBM once per sequence instead of twice per step.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _lib
from .conv2d import output_hw, pack_weight, prepare_input

SUPPORTED_LIF_PATTERNS = ((1, 1, 0), (3, 1, 1))


def fold_bn(weight: torch.Tensor, bias: Optional[torch.Tensor], bn) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fold an eval-mode BatchNorm2d into conv weight and bias (fp32)."""
    w = weight.detach().to(torch.float32)
    mean = bn.running_mean.detach().to(torch.float32)
    var = bn.running_var.detach().to(torch.float32)
    gamma = bn.weight.detach().to(torch.float32) if bn.weight is not None else torch.ones_like(mean)
    beta = bn.bias.detach().to(torch.float32) if bn.bias is not None else torch.zeros_like(mean)
    scale = gamma / torch.sqrt(var + bn.eps)
    b = bias.detach().to(torch.float32) if bias is not None else torch.zeros_like(mean)
    return w * scale.view(-1, 1, 1, 1), (b - mean) * scale + beta


def sparse_fused_conv_lif_forward(
    x: torch.Tensor,
    v_prev: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    tau: float = 2.0,
    v_threshold: float = 1.0,
    v_reset: Optional[float] = 0.0,
    decay_input: bool = True,
    kernel_size: int = 3,
    stride: int = 1,
    padding: Optional[int] = None,
    w_packed: Optional[torch.Tensor] = None,
    return_ms: bool = False,
    emit_event_masks: bool = False,
):
    """x: [T, N, C, H, W] (or [N, C, H, W] for one step); v_prev: [N, C_out, H_out, W_out].

    Returns (spikes with x's shape convention and dtype, v_next fp32, ms).
    """
    if not x.is_cuda:
        raise RuntimeError("sparse_fused_conv_lif_forward needs CUDA tensors (no CPU fallback)")
    single = x.dim() == 4
    x5 = x.unsqueeze(0) if single else x
    if x5.dim() != 5:
        raise ValueError(f"Expected 4D or 5D input, got {x.dim()}D")
    if padding is None:
        padding = 1 if kernel_size == 3 else 0
    if (kernel_size, stride, padding) not in SUPPORTED_LIF_PATTERNS:
        raise ValueError(f"fused conv+LIF supports 3x3/s1/p1 and 1x1/s1/p0, got k={kernel_size} s={stride} p={padding}")
    t, n, c, h, w = x5.shape
    co = weight.shape[0]
    ho, wo = output_hw(h, w, kernel_size, stride, padding)
    x5 = prepare_input(x5)
    wp = w_packed if w_packed is not None else pack_weight(weight)
    b = None if bias is None else bias.detach().to(torch.float32).contiguous()
    v = v_prev.detach().to(torch.float32).contiguous().clone()
    if tuple(v.shape) != (n, co, ho, wo):
        raise ValueError(f"v_prev shape {tuple(v.shape)} != {(n, co, ho, wo)}")
    spikes = torch.empty(t, n, co, ho, wo, dtype=x5.dtype, device=x5.device)
    masks = None
    if emit_event_masks:
        nbytes = _lib.event_masks_bytes(t * n, co, ho, wo)
        masks = torch.empty(nbytes // 8, dtype=torch.int64, device=x5.device)
    ms = 0.0
    if return_ms:
        se, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        se.record()
    _lib.fused_conv_lif(x5, wp, b, v, spikes, kernel_size, stride, padding, tau, v_threshold, v_reset, decay_input,
                        masks_out=masks)
    if return_ms:
        ee.record()
        torch.cuda.synchronize(x5.device)
        ms = se.elapsed_time(ee)
    out = spikes[0] if single else spikes
    if masks is not None:
        attach_event_masks(out, masks)
    return out, v, ms


def attach_event_masks(spikes: torch.Tensor, masks: torch.Tensor) -> None:
    """Record on the spikes tensor its event masks ([T*N][H][W][ceil(C/64)] 64-bit words), so that a
    following SparseConv2d that receives this very tensor runs from them instead of re-reading it."""
    spikes._sf_event_masks = (masks, spikes.data_ptr(), tuple(spikes.shape), spikes.dtype)


def event_masks_of(x: torch.Tensor):
    """The masks attached by attach_event_masks if x is still the tensor they describe, else None."""
    rec = getattr(x, "_sf_event_masks", None)
    if rec is None:
        return None
    masks, ptr, shape, dtype = rec
    if ptr != x.data_ptr() or shape != tuple(x.shape) or dtype != x.dtype or x._version != 0:
        return None
    return masks
