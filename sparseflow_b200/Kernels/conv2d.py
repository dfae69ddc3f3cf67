"""Sparse conv2d entry point on the native sm_100a kernels.

Reference: Kernels/conv2d.py:893-1178 (``sparse_conv2d_forward``), with the
same argument list and the same variable-arity return
``(y, ms[, avg_active_ratio][, tile_stats][, backend_meta])``.

What differs is the machinery behind it. The reference casts x to fp16,
repacks it NHWC, runs a torch-op prescan, syncs on ``torch.nonzero`` and
launches a Triton kernel over active (tile, group) blocks in fp16. Here one
native launch reads x in its own NCHW layout and dtype, skips every exact
zero element (element-level sparsity), accumulates in fp32 against fp32 (or
bf16) weights and writes y; no host sync happens unless timing or
statistics are requested. The stage-1 prescan runs only when its metadata is
asked for (statistics, or caller-provided metadata buffers).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from .. import _lib
from ..Utils.config import PRESCAN_ACTIVITY_EPS, SPARSE_DENSE_RATIO_THRESHOLD, TC3X3_MAX_CIN
from ..Utils.sparse_helpers import (TILE_DENSEISH, TILE_SPARSE, TILE_ZERO, choose_group_size, popcount_buf,
                                    select_tile_sizes)
from ._prescan_common import prescan2d

FALLBACK_RATIO = SPARSE_DENSE_RATIO_THRESHOLD

SUPPORTED_PATTERNS = ((1, 1, 0), (1, 2, 0), (3, 1, 1), (3, 2, 1))


def _select_tile_sizes(h: int, w: int):
    return select_tile_sizes(h, w)


def _select_block_sizes(h, w, c_in, c_out, kernel_size, n):
    bh, bw = select_tile_sizes(h, w)
    return bh, bw, bh * bw, 64, choose_group_size(c_in)


def _popcount_buf(ag_mask_buf, n_tiles):
    return popcount_buf(ag_mask_buf, n_tiles)


def output_hw(h: int, w: int, k: int, s: int, p: int, d: int = 1):
    return (h + 2 * p - d * (k - 1) - 1) // s + 1, (w + 2 * p - d * (k - 1) - 1) // s + 1


def prepare_input(x: torch.Tensor) -> torch.Tensor:
    """The kernels read x in its own NCHW layout; only contiguity is required."""
    return x.contiguous()


def pack_weight(weight: torch.Tensor) -> torch.Tensor:
    """Pack [C_out, C_in, k, k] for the kernel: fp32 stays fp32 (fp16 widens
    exactly to fp32), bf16 stays bf16."""
    out_dtype = torch.bfloat16 if weight.dtype == torch.bfloat16 else torch.float32
    return _lib.pack_weights(weight, out_dtype)


def uses_event_masks(c_in: int, h_in: int, w_in: int, kernel_size: int, stride: int, padding: int) -> bool:
    """Whether a convolution handed its input's event masks runs from them.

    1x1/s2 has no mask-driven kernel. 1x1/s1 always does: on images of at
    least one 128-pixel MMA tile the tcgen05 kernel builds its A operand from
    the masks (32 bytes per pixel for 256 channels instead of 1 KB of fp32
    spikes; C2 cell 0.34 ms from the spikes), on smaller images the gather
    kernel reads them. The 3x3/s1 tensor-core kernel with C_in <= 64 reads the
    spikes faster than the gather kernel reads masks (C64 56x56: 0.37 ms
    against 0.46 ms; 8x8 maps: 0.027 against 0.06 ms), so those layers ignore
    them. Wider 3x3/s1 layers run from the masks when the spikes are sparse and
    from x on the tensor cores otherwise, chosen on the device."""
    if (kernel_size, stride) == (1, 2):
        return False
    lib = _lib.load()
    if (kernel_size, stride, padding) == (3, 1, 1) and c_in <= TC3X3_MAX_CIN and \
            lib.sf_get_path_policy(_lib.SF_POLICY_CONV3X3_PATH) != 1:
        return False
    return True


def sparse_conv2d_forward(
    x, weight, bias,
    kernel_size=3, stride=1, padding=0, dilation=1, groups=1,
    threshold=PRESCAN_ACTIVITY_EPS, w_cl=None,
    ag_mask_buf=None, tile_class_buf=None,
    return_ms=False, fallback_ratio=FALLBACK_RATIO,
    return_avg_active_ratio=False, return_tile_stats=False,
    return_backend_meta=False,
    x_nhwc=None, active_tile_ids_buf=None,
    launch_all_tiles=False,
    output_dtype=None,
    event_masks=None,
):
    """Sparse conv2d of an NCHW CUDA tensor. See the module docstring.

    ``w_cl`` is an optional pre-packed weight buffer (from ``pack_weight``);
    ``x_nhwc`` and ``fallback_ratio`` are accepted for signature compatibility
    and unused (the kernel reads NCHW; the runtime dense policy is off).
    ``event_masks``: x's per-pixel nonzero-channel masks as written by a fused
    conv + LIF (x then holds binary spikes); the mask pass over x is skipped.
    """
    if not x.is_cuda:
        raise RuntimeError("sparse_conv2d_forward needs a CUDA tensor (the B200 path has no CPU fallback)")
    if isinstance(stride, (tuple, list)):
        stride = stride[0]
    if isinstance(padding, (tuple, list)):
        padding = padding[0]
    if isinstance(dilation, (tuple, list)):
        dilation = dilation[0]
    n, c_in, h_in, w_in = x.shape
    c_out = weight.shape[0]
    out_dtype = x.dtype if output_dtype is None else output_dtype
    need_stats = bool(return_tile_stats or return_avg_active_ratio)

    def _finalize(y, ms, ratio=None, tile_stats=None, meta=None):
        ret = (y, ms)
        if return_avg_active_ratio:
            ret = ret + (ratio,)
        if return_tile_stats:
            ret = ret + (tile_stats,)
        if return_backend_meta:
            ret = ret + (meta,)
        return ret

    def _dense(reason):
        # Patterns outside the sparse kernels (never produced by the analyzer)
        # keep the reference's behaviour: the dense GPU convolution.
        ms = 0.0
        if return_ms:
            se, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            se.record()
        y = F.conv2d(x, weight, bias, stride=stride, padding=padding, dilation=dilation, groups=groups)
        if y.dtype != out_dtype:
            y = y.to(out_dtype)
        if return_ms:
            ee.record()
            torch.cuda.synchronize(x.device)
            ms = se.elapsed_time(ee)
        return _finalize(y, ms, 1.0, None, {"backend": "dense_fallback", "reason": reason})

    if groups != 1 or dilation != 1:
        return _dense("unsupported_groups_or_dilation")
    h_out, w_out = output_hw(h_in, w_in, kernel_size, stride, padding, dilation)
    if h_out <= 0 or w_out <= 0:
        return _dense("invalid_output_shape")
    if (kernel_size, stride, padding) not in SUPPORTED_PATTERNS:
        return _dense("split_1x1s2_downsample" if (kernel_size, stride) == (1, 2) else "unsupported_pattern")

    gs = choose_group_size(c_in)
    n_groups = -(-c_in // gs)
    bh, bw = select_tile_sizes(h_out, w_out)
    gh, gw = -(-h_out // bh), -(-w_out // bw)
    n_tiles = n * gh * gw

    x = prepare_input(x)
    w_packed = w_cl if w_cl is not None else pack_weight(weight)
    b = None if bias is None else bias.detach().to(torch.float32).contiguous()

    avg_ratio = None
    tile_stats = None
    active_tiles = None
    want_meta = need_stats or ag_mask_buf is not None or tile_class_buf is not None or active_tile_ids_buf is not None
    if want_meta:
        count = torch.zeros(1, dtype=torch.int32, device=x.device) if active_tile_ids_buf is not None else None
        tc, agm, _, _ = prescan2d(x, _lib.SF_LAYOUT_NCHW, (h_out, w_out), (kernel_size, kernel_size), stride,
                                  padding, (bh, bw), gs, threshold, ag_mask_out=ag_mask_buf,
                                  tile_class_out=tile_class_buf, active_ids_out=active_tile_ids_buf,
                                  active_count_out=count)
        if need_stats:
            zc = int((tc == TILE_ZERO).sum().item())
            sc = int((tc == TILE_SPARSE).sum().item())
            dc = int((tc == TILE_DENSEISH).sum().item())
            active_tiles = sc + dc
            pc = popcount_buf(agm, n_tiles)
            avg_ratio = float(pc.sum().item()) / max(float(n_tiles * n_groups), 1.0)
            if return_tile_stats:
                tile_stats = {
                    "zero_tiles": zc, "sparse_tiles": sc, "denseish_tiles": dc, "total_tiles": n_tiles,
                    "prescan_mode": "b200_single_pass", "active_tiles": active_tiles,
                    "active_tile_ratio": active_tiles / max(n_tiles, 1),
                    "denseish_ratio_nonzero": dc / max(active_tiles, 1),
                }

    y = torch.empty(n, c_out, h_out, w_out, dtype=x.dtype, device=x.device)
    ms = 0.0
    if return_ms:
        se, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        se.record()
    used_masks = event_masks is not None and uses_event_masks(c_in, h_in, w_in, kernel_size, stride, padding)
    if used_masks and (kernel_size, stride, padding) == (3, 1, 1):
        # Dense enough spikes run on the tensor cores from x; the choice is made on the device.
        _lib.sparse_conv2d_masks_or_x(x, event_masks, w_packed, b, y, kernel_size, stride, padding)
    elif used_masks:
        _lib.sparse_conv2d_from_masks(event_masks, tuple(x.shape), x.dtype, w_packed, b, y, kernel_size, stride,
                                      padding)
    else:
        _lib.sparse_conv2d(x, w_packed, b, y, c_out, kernel_size, stride, padding)
    if return_ms:
        ee.record()
        torch.cuda.synchronize(x.device)
        ms = se.elapsed_time(ee)
    if y.dtype != out_dtype:
        y = y.to(out_dtype)
    meta = {
        "backend": "sparse_b200", "reason": "element_gather_sm100a",
        "total_tiles": n_tiles, "launch_count": n_tiles,
        "launch_mode": "persistent", "launch_mode_reason": "persistent_gather",
        "event_masks": used_masks,
    }
    if active_tiles is not None:
        meta["active_tiles"] = active_tiles
    return _finalize(y, ms, avg_ratio, tile_stats, meta)

