"""Replacement-target discovery (reference: Core/analyzer.py:52-811).

A target is a module that consumes the output of a spike source (LIF/IF ...)
before the next spike source. Discovery runs in the reference's order, each
mode used only when the previous one finds nothing or fails:

  1. torch.fx symbolic trace, breadth-first from each spike node through its
     users (depth <= 20), stopping at targets and at other spike nodes
     (:347-418);
  2. runtime order: forward hooks under ``sample_input`` record the order in
     which spike sources and targets run; each target pairs with the most
     recent spike source (:424-500);
  3. module order: for each spike module, the next modules in
     ``named_modules()`` order within a window of 15, skipping transparent
     layers (BN, pooling, dropout, activations, ...) and stopping at the
     next spike module (:506-549).

Conv2d targets are classified as conv2d_3x3 (3x3/s1/p1), conv2d_3x3_s2
(3x3/s2/p1), conv2d_1x1 (1x1/s1/p0) or depthwise_conv2d; other grouped or
shaped convs are not targets, and maps smaller than 7 on either side are
skipped (:575-636). ``block_size`` is filled from the H -> block rule of
``Utils.block_selector``.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass
from typing import Dict, List, Optional, Set, Tuple

import torch
import torch.nn as nn

from ..Utils.block_selector import select_block_size
from .registry import SpikeOpRegistry


@dataclass
class ReplacementTarget:
    conv_name: str
    conv_module: nn.Module
    spike_name: str
    op_type: str
    block_size: Optional[int] = None
    input_h: int = 0
    input_w: int = 0
    input_d: int = 0
    extra: Optional[dict] = None


_TRANSPARENT_MODULES = (
    nn.Dropout, nn.Dropout2d, nn.Dropout3d, nn.Identity, nn.Flatten,
    nn.AdaptiveAvgPool1d, nn.AdaptiveAvgPool2d, nn.AdaptiveAvgPool3d,
    nn.AdaptiveMaxPool1d, nn.AdaptiveMaxPool2d, nn.AdaptiveMaxPool3d,
    nn.AvgPool1d, nn.AvgPool2d, nn.AvgPool3d, nn.MaxPool1d, nn.MaxPool2d, nn.MaxPool3d,
    nn.BatchNorm1d, nn.BatchNorm2d, nn.BatchNorm3d,
    nn.ReLU, nn.ReLU6, nn.LeakyReLU, nn.GELU, nn.SiLU, nn.Sequential,
)


def _is_attention_like(module: Optional[nn.Module]) -> bool:
    if module is None:
        return False
    if not all(isinstance(getattr(module, a, None), nn.Linear) for a in ("q", "k", "v", "proj")):
        return False
    return hasattr(module, "attn_lif")


def _target_kind(module: Optional[nn.Module]) -> Optional[str]:
    """Module -> target family, in the reference's precedence."""
    if isinstance(module, nn.Conv1d):
        return "conv1d"
    if isinstance(module, nn.Conv2d):
        return "conv2d"
    if isinstance(module, nn.Conv3d):
        return "conv3d"
    if isinstance(module, nn.Linear):
        return "linear"
    if _is_attention_like(module):
        return "attention"
    return None


def _pair(v) -> Tuple[int, int]:
    if isinstance(v, (tuple, list)):
        return (int(v[0]), int(v[0])) if len(v) == 1 else (int(v[0]), int(v[1]))
    return int(v), int(v)


def display_block_info(target: ReplacementTarget) -> str:
    if target.op_type in ("conv2d_3x3", "conv2d_3x3_s2", "conv2d_1x1"):
        h, w = target.input_h, target.input_w
        if h <= 0 or w <= 0:
            return "H=? BLOCK_M=?"
        from ..Utils.sparse_helpers import select_tile_sizes
        bh, bw = select_tile_sizes(h, w)
        return f"H={h} BLOCK_M={bh * bw}"
    if target.op_type == "depthwise_conv2d":
        return f"DW H={target.input_h or '?'} W={target.input_w or '?'}"
    return ""


def _reset_states(model: nn.Module) -> None:
    try:
        from spikingjelly.activation_based import functional as sj_func
        sj_func.reset_net(model)
        return
    except ImportError:
        pass
    from ..Ops.lif_node import reset_net
    reset_net(model)


_LEAF_LAYERS = (nn.modules.conv._ConvNd, nn.modules.batchnorm._BatchNorm, nn.modules.pooling._MaxPoolNd,
                nn.modules.pooling._AvgPoolNd, nn.Linear)


class NetworkAnalyzer:
    FALLBACK_SEARCH_WINDOW = 15
    MAX_BFS_DEPTH = 20

    def __init__(self, registry: SpikeOpRegistry):
        self.registry = registry

    # -- driver ---------------------------------------------------------------
    def analyze(self, model: nn.Module, sample_input: Optional[torch.Tensor] = None) -> List[ReplacementTarget]:
        shapes = self._infer_input_shapes(model, sample_input) if sample_input is not None else {}
        attention = self._analyze_attention_modules(model, shapes)
        attention_names = {t.conv_name for t in attention}

        fx_failed = False
        try:
            found = self._analyze_fx(model, shapes)
            merged = self._merge_targets(found, attention, attention_names) if found else []
            if merged:
                return merged
        except Exception as err:  # symbolic tracing fails on data-dependent control flow
            fx_failed = True
            warnings.warn(f"[SparseFlow] torch.fx symbolic trace failed: {err}\n"
                          "  Falling back to runtime-order scan mode.")
        if sample_input is not None:
            try:
                found = self._analyze_runtime_fallback(model, shapes, sample_input)
                merged = self._merge_targets(found, attention, attention_names) if found else []
                if merged:
                    return merged
            except Exception as err:
                warnings.warn(f"[SparseFlow] runtime-order fallback failed: {err}\n"
                              "  Falling back to linear module-order scan mode.")
        elif not fx_failed:
            warnings.warn("[SparseFlow] torch.fx produced no targets and no sample input was provided; "
                          "falling back to linear module-order scan mode.")
        return self._merge_targets(self._analyze_fallback(model, shapes), attention, attention_names)

    @staticmethod
    def _merge_targets(base: List[ReplacementTarget], attention: List[ReplacementTarget],
                       attention_names: Set[str]) -> List[ReplacementTarget]:
        out: List[ReplacementTarget] = []
        seen: Set[str] = set()
        for t in base:
            if any(t.conv_name.startswith(a + ".") for a in attention_names) or t.conv_name in seen:
                continue
            out.append(t)
            seen.add(t.conv_name)
        for t in attention:
            if t.conv_name not in seen:
                out.append(t)
                seen.add(t.conv_name)
        return out

    def _analyze_attention_modules(self, model, shapes) -> List[ReplacementTarget]:
        res = []
        for name, mod in model.named_modules():
            if _is_attention_like(mod):
                t = self._make_attention_target(name, mod, f"{name}.attn_lif", shapes)
                if t is not None:
                    res.append(t)
        return res

    # -- mode 1: torch.fx -----------------------------------------------------------
    def _analyze_fx(self, model, shapes) -> List[ReplacementTarget]:
        registry = self.registry

        class _SpikeLeafTracer(torch.fx.Tracer):
            # Spike sources, and subclasses of torch's conv / norm / pool / linear
            # layers (multi-step wrappers that fold T into the batch), are graph
            # leaves: their bodies branch on runtime state (membrane shape, input
            # rank, device), which symbolic tracing cannot follow, and the
            # analyzer only needs their call sites.
            def is_leaf_module(self, m, qualname):
                return (registry.is_spike_op(m) or isinstance(m, _LEAF_LAYERS)
                        or super().is_leaf_module(m, qualname))

        graph = _SpikeLeafTracer().trace(model)
        gm = torch.fx.GraphModule(model, graph)
        modules = dict(gm.named_modules())
        is_spike = lambda node: (node.op == "call_module"  # noqa: E731
                                 and self.registry.is_spike_op(modules.get(node.target)))
        targets: List[ReplacementTarget] = []
        taken: Set[str] = set()
        for spike in [nd for nd in gm.graph.nodes if is_spike(nd)]:
            for name, kind in self._bfs_find_targets(spike, modules, taken, is_spike):
                t = self._make_target(name, modules[name], kind, spike.target, shapes)
                if t is not None:
                    targets.append(t)
                    taken.add(name)
        return targets

    def _bfs_find_targets(self, spike_node, modules, taken, is_spike):
        found = []
        frontier = [(u, 0) for u in spike_node.users]
        visited = set()
        while frontier:
            node, depth = frontier.pop(0)
            if depth > self.MAX_BFS_DEPTH or id(node) in visited:
                continue
            visited.add(id(node))
            kind = _target_kind(modules.get(node.target)) if node.op == "call_module" else None
            if kind is not None:
                if node.target not in taken:
                    found.append((node.target, kind))
                continue
            if is_spike(node):
                continue
            frontier.extend((u, depth + 1) for u in node.users)
        return found

    # -- mode 2: runtime order ------------------------------------------------
    def _analyze_runtime_fallback(self, model, shapes, sample_input) -> List[ReplacementTarget]:
        modules = dict(model.named_modules())
        events: List[Tuple[str, str]] = []
        hooks = []
        for name, mod in model.named_modules():
            if self.registry.is_spike_op(mod):
                hooks.append(mod.register_forward_hook(lambda _m, _i, _o, n=name: events.append(("spike", n))))
            elif _target_kind(mod) is not None:
                hooks.append(mod.register_forward_hook(lambda _m, _i, _o, n=name: events.append(("target", n))))
        try:
            _reset_states(model)
            with torch.no_grad():
                model(sample_input)
        finally:
            for h in hooks:
                h.remove()
        targets, taken, last_spike = [], set(), None
        for kind, name in events:
            if kind == "spike":
                last_spike = name
                continue
            if name in taken or last_spike is None:
                continue
            mod = modules.get(name)
            t = self._make_target(name, mod, _target_kind(mod), last_spike, shapes) if mod is not None else None
            if t is not None:
                targets.append(t)
                taken.add(name)
        return targets

    # -- mode 3: module order ------------------------------------------------------
    def _analyze_fallback(self, model, shapes) -> List[ReplacementTarget]:
        mods = list(model.named_modules())
        targets, taken = [], set()
        for i, (name, mod) in enumerate(mods):
            if not self.registry.is_spike_op(mod):
                continue
            for nxt_name, nxt in mods[i + 1: min(i + self.FALLBACK_SEARCH_WINDOW, len(mods))]:
                if nxt_name in taken:
                    continue
                if self.registry.is_spike_op(nxt):
                    break
                if isinstance(nxt, _TRANSPARENT_MODULES):
                    continue
                kind = _target_kind(nxt)
                if kind is None:
                    continue
                t = self._make_target(nxt_name, nxt, kind, name, shapes)
                if t is not None:
                    targets.append(t)
                    taken.add(nxt_name)
        return targets

    # -- target builders --------------------------------------------------------------
    def _make_target(self, name, module, kind, spike_name, shapes) -> Optional[ReplacementTarget]:
        if kind == "conv2d":
            return self._make_conv2d_target(name, module, spike_name, shapes)
        if kind in ("conv1d", "conv3d", "linear"):
            shp = shapes.get(name)
            h, w = self._extract_hw(shp) if kind == "conv3d" else (0, self._extract_l(shp))
            return ReplacementTarget(name, module, spike_name, kind, None, h if kind == "conv3d" else 0, w)
        if kind == "attention":
            return self._make_attention_target(name, module, spike_name, shapes)
        return None

    def _make_conv2d_target(self, name, conv, spike_name, shapes) -> Optional[ReplacementTarget]:
        if not isinstance(conv, nn.Conv2d):
            return None
        k, s, p = _pair(conv.kernel_size), _pair(conv.stride), _pair(conv.padding)
        h, w = self._extract_hw(shapes.get(name))
        if (conv.groups == conv.in_channels and conv.out_channels == conv.in_channels
                and k[0] == k[1] and s[0] == s[1] and p[0] == p[1]):
            return ReplacementTarget(name, conv, spike_name, "depthwise_conv2d", None, h, w)
        if conv.groups != 1:
            return None
        op = {((3, 3), (1, 1), (1, 1)): "conv2d_3x3", ((3, 3), (2, 2), (1, 1)): "conv2d_3x3_s2",
              ((1, 1), (1, 1), (0, 0)): "conv2d_1x1"}.get((k, s, p))
        if op is None:
            return None
        if h > 0 and w > 0 and min(h, w) < 7:
            return None
        return ReplacementTarget(name, conv, spike_name, op, select_block_size(h) if h > 0 else None, h, w)

    def _make_attention_target(self, name, module, spike_name, shapes) -> Optional[ReplacementTarget]:
        if not _is_attention_like(module):
            return None
        shp = shapes.get(name)
        n, c = (int(shp[-2]), int(shp[-1])) if shp is not None and len(shp) >= 2 else (0, 0)
        cls = type(module).__name__.lower()
        op = "attention_qkmix" if "qkmix" in cls else ("attention_qkav" if hasattr(module, "scale")
                                                       else "attention_linear")
        heads = int(getattr(module, "num_heads", 1))
        extra = {"num_heads": heads, "head_dim": int(getattr(module, "head_dim", max(1, c // max(1, heads))))}
        return ReplacementTarget(name, module, spike_name, op, None, n, c, extra=extra)

    @staticmethod
    def _extract_hw(shape) -> Tuple[int, int]:
        return (int(shape[-2]), int(shape[-1])) if shape is not None and len(shape) >= 2 else (0, 0)

    @staticmethod
    def _extract_l(shape) -> int:
        return int(shape[-1]) if shape is not None and len(shape) >= 1 else 0

    @staticmethod
    def _infer_input_shapes(model: nn.Module, sample_input: torch.Tensor) -> Dict[str, tuple]:
        shapes: Dict[str, tuple] = {}
        hooks = []
        for name, mod in model.named_modules():
            def hook(_m, inp, _o, n=name):
                if isinstance(inp, (tuple, list)) and inp and isinstance(inp[0], torch.Tensor):
                    shapes[n] = tuple(inp[0].shape)
            hooks.append(mod.register_forward_hook(hook))
        try:
            _reset_states(model)
            with torch.no_grad():
                model(sample_input)
        finally:
            for h in hooks:
                h.remove()
        _reset_states(model)
        return shapes
