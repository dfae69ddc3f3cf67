"""Module replacement pass (reference: Core/replacer.py:83-292).

Swaps each conv2d target (conv2d_3x3, conv2d_3x3_s2, conv2d_1x1) in place,
by dotted module name, for ``SparseConv2d.from_dense(conv, block_size, ...)``
and attaches the reference's ``sf_*`` observability attributes
(:122-154). Layers listed in ``static_zero_layers`` become
``StaticZeroConv2d`` (bias-only output, reference Ops/static_zero_conv2d.py).
Linear targets become ``SparseLinear`` (reference Core/replacer.py linear branch).
Targets of other families (conv1d/3d, depthwise, attention, pools)
have no kernel on the B200 path and are kept dense and counted as such.
Returns ``(replaced, sparse_count, static_zero_count, dense_keep_count)``.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Set, Tuple

import torch
import torch.nn as nn

from ..Ops.sparse_conv2d import SparseConv2d
from ..Ops.sparse_linear import SparseLinear
from .analyzer import ReplacementTarget, display_block_info

_CONV2D_OPS = ("conv2d_3x3", "conv2d_1x1", "conv2d_3x3_s2")
_LINEAR_OPS = ("linear",)
_STATIC_ZERO_OPS = ("conv2d_3x3", "conv2d_1x1", "conv2d_3x3_s2")


class StaticZeroConv2d(nn.Module):
    """Conv2d whose input is known to be all zeros: output = bias broadcast."""

    def __init__(self, conv: nn.Conv2d):
        super().__init__()
        self.in_channels, self.out_channels = conv.in_channels, conv.out_channels
        self.kernel_size, self.stride = conv.kernel_size, conv.stride
        self.padding, self.dilation = conv.padding, conv.dilation
        self.weight = conv.weight
        self.bias = conv.bias

    @classmethod
    def from_conv(cls, conv: nn.Conv2d) -> "StaticZeroConv2d":
        return cls(conv)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-3]
        h, w = x.shape[-2:]
        ho = (h + 2 * self.padding[0] - self.dilation[0] * (self.kernel_size[0] - 1) - 1) // self.stride[0] + 1
        wo = (w + 2 * self.padding[1] - self.dilation[1] * (self.kernel_size[1] - 1) - 1) // self.stride[1] + 1
        y = torch.zeros(*lead, self.out_channels, ho, wo, dtype=x.dtype, device=x.device)
        if self.bias is not None:
            y += self.bias.detach().to(x.dtype).view(self.out_channels, 1, 1)
        return y


def _set_module_by_name(model: nn.Module, name: str, new_module: nn.Module) -> None:
    parent = model
    parts = name.split(".")
    for part in parts[:-1]:
        parent = parent[int(part)] if part.isdigit() else getattr(parent, part)
    setattr(parent, parts[-1], new_module)


class ModuleReplacer:
    def __init__(self, verbose: bool = True):
        self.verbose = verbose

    @staticmethod
    def _score_family_from_op(op_type: str) -> str:
        if op_type in ("conv2d_3x3", "conv2d_1x1", "conv2d_3x3_s2", "depthwise_conv2d", "conv1d", "conv3d"):
            return "conv"
        if op_type == "linear":
            return "linear"
        if op_type in ("attention_linear", "attention_proj_linear"):
            return "attn_linear"
        if op_type in ("attention_qkav", "attention_qkmix", "attention_matmul"):
            return "attn_matmul"
        if op_type in ("maxpool2d", "avgpool2d"):
            return "pool"
        return "unknown"

    def _attach_observability(self, module: nn.Module, target: ReplacementTarget, backend_mode: str,
                              backend_family: Optional[str] = None, fallback_reason: str = "") -> nn.Module:
        family = backend_family or ("exact_zero" if backend_mode == "staticzero" else "sparse_kernel")
        score = self._score_family_from_op(str(target.op_type))
        attrs = {
            "sf_layer_name": str(target.conv_name), "sf_operator_type": str(target.op_type),
            "sf_operator_family": score, "sf_spike_source": str(target.spike_name),
            "sf_backend_mode": backend_mode, "sf_dispatch_decision": backend_mode,
            "sf_backend_family": family, "sf_reason_code": "", "sf_meta_source": "measured",
            "sf_diag_source": "measured", "sf_support_status": "supported", "sf_score_family": score,
            "sf_tile_source": "unknown", "sf_fallback_reason": str(fallback_reason),
        }
        for k, v in attrs.items():
            setattr(module, k, v)
        return module

    def replace(self, model: nn.Module, targets: List[ReplacementTarget],
                block_sizes: Optional[Dict[str, int]] = None, static_zero_layers: Optional[Set[str]] = None,
                disable_static_zero: bool = False, only_static_zero: bool = False,
                sparse_kwargs: Optional[Dict[str, Any]] = None) -> Tuple[int, int, int, int]:
        static_zero_layers = set() if (static_zero_layers is None or disable_static_zero) else set(static_zero_layers)
        sparse_kwargs = sparse_kwargs or {}
        replaced = sparse = static_zero = dense_keep = 0
        for t in targets:
            block = block_sizes[t.conv_name] if block_sizes and t.conv_name in block_sizes else t.block_size
            if t.op_type in _STATIC_ZERO_OPS and t.conv_name in static_zero_layers:
                mod = StaticZeroConv2d.from_conv(t.conv_module)
                self._attach_observability(mod, t, "staticzero", "exact_zero")
                _set_module_by_name(model, t.conv_name, mod)
                replaced += 1
                static_zero += 1
                if self.verbose:
                    print(f"  [STATIC ] {t.conv_name} ({t.op_type}) -> StaticZeroConv2d")
                continue
            if only_static_zero or t.op_type not in _CONV2D_OPS + _LINEAR_OPS:
                dense_keep += 1
                if self.verbose:
                    why = "DenseKeep" if only_static_zero else "DenseKeep (no B200 kernel for this op)"
                    print(f"  [KEEP   ] {t.conv_name} ({t.op_type}) -> {why}")
                continue
            mod = self._create_sparse_module(t, block, sparse_kwargs)
            self._attach_observability(mod, t, "sparse", "sparse_kernel")
            _set_module_by_name(model, t.conv_name, mod)
            replaced += 1
            sparse += 1
            if self.verbose:
                print(f"  [SPARSE ] {t.conv_name} ({t.op_type}, {display_block_info(t)}, "
                      f"block={block}) <- spike {t.spike_name}")
        return replaced, sparse, static_zero, dense_keep

    def _create_sparse_module(self, target: ReplacementTarget, block: Optional[int],
                              sparse_kwargs: Dict[str, Any]) -> nn.Module:
        mod = target.conv_module
        if target.op_type in _LINEAR_OPS:
            lin = SparseLinear.from_dense(mod, threshold=float(sparse_kwargs.get("threshold", 1e-6)),
                                          return_ms=bool(sparse_kwargs.get("return_ms", False)))
            return lin.to(mod.weight.device)
        sparse = SparseConv2d.from_dense(mod, block_size=block,
                                         threshold=float(sparse_kwargs.get("threshold", 1e-6)),
                                         return_ms=bool(sparse_kwargs.get("return_ms", False)))
        sparse.collect_diag = bool(sparse_kwargs.get("collect_diag", False))
        sparse.profile_runtime = bool(sparse_kwargs.get("profile_runtime", False))
        return sparse.to(mod.weight.device)
