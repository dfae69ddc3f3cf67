"""Stage-1 receptive-field prescan, on the native sm_100a kernel.

Reference: Kernels/_prescan_common.py:231-306. The metadata is bit-identical:
for each output tile (row-major over n, gh, gw) bit g of ``ag_mask`` is set
iff channel group g has |half(x)| > half(threshold) somewhere in the tile's
receptive field, and ``tile_class`` is ZERO / SPARSE / DENSEISH. The native
kernel additionally compacts the ids of non-ZERO tiles (the reference's
``torch.nonzero`` step, Kernels/conv2d.py:113-123) without a host sync.

Only the 2-D case is on the B200 path; 1-D and 3-D prescans belong to the
conv1d/conv3d operators, which are outside it.
"""
from __future__ import annotations

import threading
from typing import Dict, Optional, Tuple

import torch

from .. import _lib
from ..Utils.sparse_helpers import TILE_DENSEISH, TILE_SPARSE, TILE_ZERO

_ws_lock = threading.Lock()
_workspaces: Dict[Tuple[int, int], torch.Tensor] = {}


def _tuple(value, ndim: int) -> Tuple[int, ...]:
    if isinstance(value, int):
        return (int(value),) * ndim
    if len(value) != ndim:
        raise ValueError(f"Expected {ndim} values, got {value}")
    return tuple(int(v) for v in value)


def prescan_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised prescan workspace for (device, current stream).

    The kernel keeps the workspace consistent across launches by itself, so
    it is zeroed only when (re)allocated. Launches on different streams get
    different workspaces.
    """
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
    return ws


def prescan2d(
    x: torch.Tensor,
    layout: int,
    spatial_dims: Tuple[int, int],
    kernel_dims: Tuple[int, int],
    stride,
    padding,
    block_dims: Tuple[int, int],
    group_size_c: int,
    threshold: float,
    ag_mask_out: Optional[torch.Tensor] = None,
    tile_class_out: Optional[torch.Tensor] = None,
    active_ids_out: Optional[torch.Tensor] = None,
    active_count_out: Optional[torch.Tensor] = None,
):
    """Run the native prescan on an NCHW (``layout=0``) or NHWC (``layout=1``) tensor.

    Returns (tile_class, ag_mask, active_ids, active_count); the last two are
    None unless buffers for them were passed.
    """
    if x.dim() != 4:
        raise ValueError(f"Expected a 4-D tensor, got {tuple(x.shape)}")
    x = x.contiguous()
    if layout == _lib.SF_LAYOUT_NCHW:
        n, c, h, w = x.shape
    else:
        n, h, w, c = x.shape
    ho, wo = _tuple(spatial_dims, 2)
    kh, kw = _tuple(kernel_dims, 2)
    sh, sw = _tuple(stride, 2)
    ph, pw = _tuple(padding, 2)
    bh, bw = _tuple(block_dims, 2)
    if kh != kw or sh != sw or ph != pw:
        raise ValueError("the native prescan takes square kernels, strides and paddings")
    gh, gw = -(-ho // bh), -(-wo // bw)
    n_tiles = n * gh * gw
    desc = _lib.prescan_desc(n, c, h, w, ho, wo, kh, sh, ph, bh, bw, group_size_c, threshold, x.dtype, layout)
    if ag_mask_out is None:
        ag_mask_out = torch.empty(n_tiles, dtype=torch.int32, device=x.device)
    if tile_class_out is None:
        tile_class_out = torch.empty(n_tiles, dtype=torch.int32, device=x.device)
    for name, buf in (("ag_mask_out", ag_mask_out), ("tile_class_out", tile_class_out),
                      ("active_ids_out", active_ids_out)):
        if buf is not None and (buf.numel() < n_tiles or buf.dtype != torch.int32 or not buf.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous int32 buffer of >= {n_tiles} elements")
    ws = prescan_workspace(x.device, _lib.prescan_workspace_bytes(desc))
    _lib.prescan2d(x, desc, ag_mask_out, tile_class_out, active_ids_out, active_count_out, ws)
    return tile_class_out[:n_tiles], ag_mask_out[:n_tiles], active_ids_out, active_count_out


def _debug_stats(tile_class: torch.Tensor, ag_mask: torch.Tensor, num_groups: int) -> Dict[str, float]:
    # Host-synchronising summary; only built when a caller asks for statistics.
    n_tiles = int(tile_class.numel())
    zero = int((tile_class == TILE_ZERO).sum().item())
    dense = int((tile_class == TILE_DENSEISH).sum().item())
    sparse = int((tile_class == TILE_SPARSE).sum().item())
    bits = 0
    if n_tiles:
        m = ag_mask.to(torch.int64) & 0xFFFFFFFF
        for g in range(num_groups):
            bits += int(((m >> g) & 1).sum().item())
    ratio = bits / max(n_tiles * max(num_groups, 1), 1)
    return {
        "stage1_zero_candidate": zero,
        "stage1_denseish": dense,
        "stage1_uncertain": sparse,
        "stage1_avg_active_group_ratio_lower_bound": float(ratio),
        "final_zero": zero,
        "final_sparse": sparse,
        "final_denseish": dense,
        "stage2_zero_refine_tiles": 0,
        "stage2_uncertain_tiles": 0,
        "total_tiles": n_tiles,
    }


def _build_rf_prescan_metadata_impl(
    x_channels_last: torch.Tensor,
    spatial_dims,
    kernel_dims,
    stride,
    padding,
    block_dims,
    group_size_c: int,
    num_groups: int,
    threshold: float,
    return_debug_stats: bool = False,
    tile_class_out: Optional[torch.Tensor] = None,
    ag_mask_out: Optional[torch.Tensor] = None,
):
    """Reference signature (Kernels/_prescan_common.py:231-275) on a channels-last tensor.

    Returns (tile_class, ag_mask, debug_stats_or_None).
    """
    spatial_ndim = len(_tuple(spatial_dims, len(spatial_dims)))
    if x_channels_last.dim() != spatial_ndim + 2:
        raise ValueError(
            f"Expected channels-last tensor with {spatial_ndim + 2} dims, got {tuple(x_channels_last.shape)}")
    if spatial_ndim != 2:
        raise ValueError(f"Unsupported spatial_ndim={spatial_ndim} on the B200 path (2-D only)")
    c_in = int(x_channels_last.shape[-1])
    if c_in > int(num_groups) * int(group_size_c):
        raise ValueError(f"C_in={c_in} exceeds num_groups*group_size_c={num_groups * group_size_c}")
    tile_class, ag_mask, _, _ = prescan2d(
        x_channels_last, _lib.SF_LAYOUT_NHWC, spatial_dims, kernel_dims, stride, padding, block_dims,
        group_size_c, threshold, ag_mask_out=ag_mask_out, tile_class_out=tile_class_out)
    stats = _debug_stats(tile_class, ag_mask, num_groups) if return_debug_stats else None
    return tile_class, ag_mask, stats


def build_rf_prescan_metadata(
    x_channels_last: torch.Tensor,
    spatial_dims,
    kernel_dims,
    stride,
    padding,
    block_dims,
    group_size_c: int,
    num_groups: int,
    threshold: float,
    tile_class_out: Optional[torch.Tensor] = None,
    ag_mask_out: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Return (tile_class, ag_mask) on device without a host sync (reference :278-306)."""
    tile_class, ag_mask, _ = _build_rf_prescan_metadata_impl(
        x_channels_last, spatial_dims, kernel_dims, stride, padding, block_dims, group_size_c, num_groups,
        threshold, False, tile_class_out, ag_mask_out)
    return tile_class, ag_mask


__all__ = [
    "TILE_ZERO", "TILE_SPARSE", "TILE_DENSEISH",
    "prescan2d", "prescan_workspace", "_build_rf_prescan_metadata_impl", "build_rf_prescan_metadata",
]
