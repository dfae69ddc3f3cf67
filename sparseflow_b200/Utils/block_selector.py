"""Feature-map height -> block size rule.

The reference documents this module (README.md:37-41, Instructions.md:136-144)
but does not ship it; the rule is restated from those documents:
    H >= 32       -> 16
    16 <= H < 32  -> 8
    8 <= H < 16   -> 4
    H < 8         -> None (do not replace)
Like the reference's ``SparseConv2d.block_size`` (Ops/sparse_conv2d.py:114-119,
162) the value is carried on the module and reported, while the kernels pick
their own tiling from the layer geometry.
"""
from __future__ import annotations

from typing import Optional


def select_block_size(h: int) -> Optional[int]:
    h = int(h)
    if h >= 32:
        return 16
    if h >= 16:
        return 8
    if h >= 8:
        return 4
    return None


def should_replace(h: int) -> bool:
    return select_block_size(h) is not None
