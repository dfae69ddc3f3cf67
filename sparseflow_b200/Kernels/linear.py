"""Sparse linear layer of spike inputs (reference: Kernels/linear.py:460-520, sparse_linear_forward).

y = x @ W^T + b for x [M, K] is the 1x1 convolution of M one-pixel images of K
channels, so it runs on the library's 1x1 path (the mask pass + gather kernel,
which touches only the nonzero inputs; exact fp32 accumulation against fp32 or
bf16 weights). Same arguments and variable-arity tuple as the reference.
"""
from __future__ import annotations

import torch

from .conv2d import pack_weight, sparse_conv2d_forward
from ..Utils.config import PRESCAN_ACTIVITY_EPS


def pack_linear_weight(weight: torch.Tensor) -> torch.Tensor:
    """[out, in] -> the packed 1x1 layout sf_sparse_conv2d reads."""
    return pack_weight(weight.reshape(weight.shape[0], weight.shape[1], 1, 1))


def sparse_linear_forward(x, weight, bias=None, threshold=PRESCAN_ACTIVITY_EPS, w_t=None, ag_mask_buf=None,
                          tile_class_buf=None, return_ms=False, fallback_ratio=None,
                          return_avg_active_ratio=False, return_tile_stats=False, return_backend_meta=False,
                          active_tile_ids_buf=None, launch_all_tiles=False, output_dtype=None):
    """x [M, in] CUDA tensor -> (y [M, out], ms[, ratio][, tile_stats][, backend_meta]).

    ``w_t`` is an optional buffer from ``pack_linear_weight``; the metadata
    buffers, ``fallback_ratio`` and ``launch_all_tiles`` are accepted for
    signature compatibility."""
    if not x.is_cuda:
        raise RuntimeError("sparse_linear_forward needs a CUDA tensor (the B200 path has no CPU fallback)")
    if x.dim() != 2:
        raise ValueError(f"sparse_linear_forward expects [M, in_features], got {tuple(x.shape)}")
    m, k = x.shape
    w4 = weight.reshape(weight.shape[0], k, 1, 1)
    wp = w_t if w_t is not None else pack_linear_weight(weight)
    need_ratio = bool(return_avg_active_ratio)
    out = sparse_conv2d_forward(x.contiguous().reshape(m, k, 1, 1), w4, bias, kernel_size=1, stride=1, padding=0,
                                threshold=threshold, w_cl=wp, return_ms=return_ms,
                                return_avg_active_ratio=need_ratio, return_tile_stats=return_tile_stats,
                                return_backend_meta=return_backend_meta, output_dtype=output_dtype)
    y = out[0].reshape(m, weight.shape[0])
    rest = list(out[1:])
    if return_backend_meta:
        meta = dict(rest[-1])
        meta["backend"] = "sparse_b200_linear"
        rest[-1] = meta
    return (y, *rest)
