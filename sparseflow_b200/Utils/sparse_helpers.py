"""Tile classes, channel-group sizing and bitmask popcount.

Reference: Utils/sparse_helpers.py:28-76 and Kernels/conv2d.py:64-84.
"""
from __future__ import annotations

import torch

TILE_ZERO = 0
TILE_SPARSE = 1
TILE_DENSEISH = 2


def choose_group_size(c_in: int) -> int:
    """Channels per prescan group: 16 up to 128 channels, else 32, doubled
    until at most 32 groups remain (so one tile's mask fits in 32 bits)."""
    gs = 16 if c_in <= 128 else 32
    while (c_in + gs - 1) // gs > 32:
        gs *= 2
    return gs


def num_groups(c_in: int) -> int:
    gs = choose_group_size(c_in)
    return (c_in + gs - 1) // gs


def select_tile_sizes(h_out: int, w_out: int) -> tuple[int, int]:
    """Output tile of the prescan metadata: 8x16 for maps of >= 3136 pixels, else 8x8."""
    return (8, 16) if h_out * w_out >= 3136 else (8, 8)


def popcount_buf(ag_mask_buf: torch.Tensor, count: int) -> torch.Tensor:
    """Active groups per tile for the first ``count`` masks (int32 result)."""
    v = ag_mask_buf[:count].to(torch.int64) & 0xFFFFFFFF
    out = torch.zeros_like(v)
    for _ in range(32):
        out += v & 1
        v = v >> 1
    return out.to(torch.int32)
