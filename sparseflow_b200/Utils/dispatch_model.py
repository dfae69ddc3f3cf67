"""Execution-grounded dispatch (EGD): per-layer backend choice "sparse", "dense" or "staticzero".

Restates the reference's policy (Utils/dispatch_model.py:814-1018 of hpcyhr/SparseFlow) on this
build's diagnostics (``SparseConv2d._last_diag`` with ``collect_diag``; same keys). For a layer
whose input is not identically zero, with AGR the active channel-group ratio over all tiles and
TZR the zero-tile ratio measured by the prescan:

    saved work      R = TZR + (1 - TZR) * (1 - AGR_nz),  AGR_nz = min(AGR / (1 - TZR), 1)
    tile intensity  I = dense MACs / tiles per image
    score           S = R * I        (dense MACs the sparse path skips, per tile)

    R >= 0.99                    -> sparse
    R (or 1 - AGR_p90) < R_min   -> dense
    S > tau(kernel family)       -> sparse, else dense

with a confidence product (measured diagnostics / metadata / tile counts) that sends a sparse
choice below ``DISPATCH_MIN_CONFIDENCE`` back to dense. Thresholds are the reference's
(Utils/config.py:50-61), kept as the default so a decision made here equals the reference's on
the same diagnostics; they can be recalibrated for this build's kernels (the crossover against
cuDNN is measured by ``bench.py --sweep``).

Helpers beyond the reference's module (its benchmark script does these steps inline):
``collect_layer_diags`` runs one forward with diagnostics on every SparseConv2d, and
``apply_dispatch`` routes layers dispatched dense to cuDNN inside their SparseConv2d.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from typing import Any, Dict, Optional, Set, Tuple

import torch
import torch.nn as nn

from .config import (
    DISPATCH_MIN_CONFIDENCE,
    DISPATCH_R_MARGIN,
    DISPATCH_R_MIN,
    DISPATCH_TAU_1X1,
    DISPATCH_TAU_3X3,
    DISPATCH_TAU_ATTN_LINEAR,
    DISPATCH_TAU_ATTN_MATMUL,
    DISPATCH_TAU_LINEAR,
    DISPATCH_TAU_MARGIN,
    NUMERIC_EPS,
)

R_NEAR_ONE = 0.99  # saved-work fraction above which a layer is sparse whatever its score


def _two(v) -> Tuple[int, int]:
    if isinstance(v, (tuple, list)):
        return (int(v[0]), int(v[0])) if len(v) == 1 else (int(v[0]), int(v[1]))
    return (int(v), int(v))


def infer_conv_output_hw(h_in: int, w_in: int, kernel_size, stride, padding, dilation=(1, 1)) -> Tuple[int, int]:
    (kh, kw), (sh, sw), (ph, pw), (dh, dw) = _two(kernel_size), _two(stride), _two(padding), _two(dilation)
    return (max((h_in + 2 * ph - dh * (kh - 1) - 1) // sh + 1, 0),
            max((w_in + 2 * pw - dw * (kw - 1) - 1) // sw + 1, 0))


def estimate_conv_macs(batch_size: int, h_out: int, w_out: int, c_out: int, c_in: int, kernel_size,
                       groups: int = 1) -> float:
    kh, kw = _two(kernel_size)
    return float(batch_size * h_out * w_out * c_out * kh * kw * (c_in / max(groups, 1)))


def _block_m_estimate(h_out: int, w_out: int) -> int:
    """Output pixels per tile when the diagnostics carry no tile count (reference :185-202)."""
    px = h_out * w_out
    for lim, m in ((512, 64), (128, 32), (32, 16)):
        if px >= lim:
            return m
    return max(px, 1)


@dataclass
class OpMeta:
    """Static description of one layer (reference :206-229; conv fields used here)."""
    layer_name: str = ""
    op_type: str = "unknown"
    meta_source: str = "measured"
    c_in: int = 0
    c_out: int = 0
    kernel_size: Tuple[int, int] = (3, 3)
    stride: Tuple[int, int] = (1, 1)
    padding: Tuple[int, int] = (1, 1)
    dilation: Tuple[int, int] = (1, 1)
    groups: int = 1
    h_in: int = 0
    w_in: int = 0
    h_out: int = 0
    w_out: int = 0
    batch_size: int = 1
    macs: float = 0.0


ConvMeta = OpMeta


@dataclass
class DispatchDecision:
    """One layer's decision with the quantities behind it (reference :235-290)."""
    backend: str = "dense"
    reason: str = ""
    reason_code: str = "init"
    confidence: float = 1.0
    fallback_reason: str = ""
    meta_source: str = "measured"
    diag_source: str = "measured"
    support_status: str = "supported"
    score_family: str = "unknown"
    tile_source: str = "diag"
    R_l: float = 0.0
    I_l: float = 0.0
    S_l: float = 0.0
    agr_nz: float = 0.0
    n_tiles: float = 0.0
    tau: float = 0.0
    agr_p90: float = -1.0
    r_worst: float = -1.0
    score_sparse: float = 0.0
    agr: float = -1.0
    tzr: float = -1.0
    macs: float = 0.0
    denseish_ratio: float = -1.0
    sparse_tile_ratio: float = -1.0
    active_groups: float = 0.0
    total_groups: float = 0.0
    layer_name: str = ""
    groups: int = 1

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


def conv_meta_from_module(conv: nn.Module, sample_x_shape: Optional[Tuple] = None, layer_name: str = "") -> OpMeta:
    """OpMeta of a Conv2d (or SparseConv2d) for an input of ``sample_x_shape`` (4-D, or 5-D T,N,...)."""
    ks, st, pad, dil = _two(conv.kernel_size), _two(conv.stride), _two(conv.padding), _two(conv.dilation)
    h_in = w_in = 0
    batch = 1
    if sample_x_shape is not None:
        shp = tuple(sample_x_shape)
        if len(shp) == 5:
            batch, h_in, w_in = shp[0] * shp[1], shp[3], shp[4]
        elif len(shp) == 4:
            batch, h_in, w_in = shp[0], shp[2], shp[3]
        elif len(shp) == 3:
            batch, h_in, w_in = shp[0], shp[2], 1
    h_out, w_out = infer_conv_output_hw(h_in, w_in, ks, st, pad, dil)
    return OpMeta(layer_name=layer_name, op_type="conv", meta_source="measured", c_in=int(conv.in_channels),
                  c_out=int(conv.out_channels), kernel_size=ks, stride=st, padding=pad, dilation=dil,
                  groups=int(conv.groups), h_in=h_in, w_in=w_in, h_out=h_out, w_out=w_out, batch_size=batch,
                  macs=estimate_conv_macs(batch, h_out, w_out, int(conv.out_channels), int(conv.in_channels), ks,
                                          int(conv.groups)))


def _field(target: Any, key: str, default=None):
    return target.get(key, default) if isinstance(target, dict) else getattr(target, key, default)


def _layer_name(target: Any) -> str:
    return str(_field(target, "name", "") or _field(target, "conv_name", ""))


def op_meta_from_target(target: Any) -> OpMeta:
    """OpMeta from a replacement target (``Core.analyzer.ReplacementTarget`` or a dict).

    The module's geometry counts as measured; the input size comes from ``input_shape`` when the
    target carries one, else from the analyzer's ``input_h``/``input_w`` (then "estimated"), and a
    missing batch size counts as 1 ("fallback"), as in the reference (:589-662).
    """
    name = _layer_name(target)
    module = _field(target, "module") or _field(target, "conv_module")
    shape = _field(target, "input_shape")
    if module is not None and hasattr(module, "kernel_size"):
        meta = conv_meta_from_module(module, shape, name)  # batch 1 when no shape is known
        src = "measured"
    else:
        meta = OpMeta(layer_name=name, op_type="conv",
                      kernel_size=_two(_field(target, "kernel_size", (3, 3))),
                      stride=_two(_field(target, "stride", (1, 1))), padding=_two(_field(target, "padding", (1, 1))),
                      dilation=_two(_field(target, "dilation", (1, 1))), groups=int(_field(target, "groups", 1)),
                      c_in=int(_field(target, "cin", _field(target, "c_in", 0))),
                      c_out=int(_field(target, "cout", _field(target, "c_out", 0))), batch_size=0)
        src = "fallback"
    if meta.h_in <= 0 or meta.w_in <= 0:
        h, w = int(_field(target, "input_h", 0) or 0), int(_field(target, "input_w", 0) or 0)
        if h > 0 and w > 0:
            meta.h_in, meta.w_in = h, w
            if src == "measured":
                src = "estimated"
    if meta.batch_size <= 0:
        shp = tuple(int(v) for v in shape) if shape is not None else ()
        meta.batch_size = (max(shp[0] * shp[1], 1) if len(shp) == 5 else max(shp[0], 1) if len(shp) in (3, 4) else 0)
        if meta.batch_size <= 0:
            meta.batch_size = int(_field(target, "batch_size", 0) or 0)
        if meta.batch_size > 0:
            src = "estimated" if src == "fallback" else src
        else:
            meta.batch_size, src = 1, "fallback"
    meta.h_out, meta.w_out = infer_conv_output_hw(meta.h_in, meta.w_in, meta.kernel_size, meta.stride,
                                                  meta.padding, meta.dilation)
    meta.macs = (estimate_conv_macs(meta.batch_size, meta.h_out, meta.w_out, meta.c_out, meta.c_in,
                                    meta.kernel_size, meta.groups)
                 if meta.c_in > 0 and meta.c_out > 0 and meta.h_out > 0 and meta.w_out > 0 else 0.0)
    hint = str(_field(target, "op_type", "conv"))
    meta.op_type = hint if hint in ("depthwise_conv2d", "grouped_conv2d") else "conv"
    meta.meta_source = src
    return meta


def _tau_for(meta: OpMeta, diag: Dict[str, Any]) -> Tuple[float, str]:
    """Threshold and score family by operator (reference :775-808)."""
    op = str(meta.op_type).lower()
    kt = str(diag.get("kernel_type", "")).lower()
    if op in ("matmul", "bmm") or kt in ("matmul", "bmm"):
        return DISPATCH_TAU_ATTN_MATMUL, (op if op in ("matmul", "bmm") else kt)
    table = {"linear": (DISPATCH_TAU_LINEAR, "linear"),
             "attention_proj_linear": (DISPATCH_TAU_ATTN_LINEAR, "attn_linear"),
             "attention_matmul": (DISPATCH_TAU_ATTN_MATMUL, "attn_matmul")}
    if op in table:
        return table[op]
    if "attention" in kt:
        return (DISPATCH_TAU_ATTN_LINEAR, "attn_linear") if "linear" in kt else (DISPATCH_TAU_ATTN_MATMUL, "attn_matmul")
    if kt == "linear":
        return DISPATCH_TAU_LINEAR, "linear"
    return (DISPATCH_TAU_1X1 if _two(meta.kernel_size) == (1, 1) else DISPATCH_TAU_3X3), "conv"


def _fallback(dec: DispatchDecision, code: str, reason: str, confidence: float) -> DispatchDecision:
    dec.backend, dec.reason_code, dec.reason, dec.fallback_reason, dec.confidence = "dense", code, reason, code, confidence
    return dec


def make_dispatch_decision(diag: Dict[str, Any], meta: OpMeta) -> DispatchDecision:
    """Decision for one layer whose input is not identically zero."""
    agr = float(diag.get("active_group_ratio", -1.0))
    tzr = float(diag.get("tile_zero_ratio", -1.0))
    act_g = diag.get("nonzero_group_count", -1.0)
    tot_g = diag.get("total_group_count", -1.0)
    if agr < 0 and tot_g > 0 and act_g >= 0:
        agr = act_g / tot_g
    tiles_diag = diag.get("total_tile_count", -1.0)
    if tzr < 0:
        zc = diag.get("tile_zero_count", -1.0)
        if tiles_diag > 0 and zc >= 0:
            tzr = zc / tiles_diag
    dense_r = sparse_r = -1.0
    if tiles_diag and tiles_diag > 0:
        if diag.get("denseish_tiles", -1.0) >= 0:
            dense_r = diag["denseish_tiles"] / tiles_diag
        if diag.get("sparse_tiles", -1.0) >= 0:
            sparse_r = diag["sparse_tiles"] / tiles_diag
    op = str(meta.op_type)
    dec = DispatchDecision(layer_name=meta.layer_name, agr=agr, tzr=tzr, macs=meta.macs, active_groups=act_g,
                           total_groups=tot_g, denseish_ratio=dense_r, sparse_tile_ratio=sparse_r,
                           groups=meta.groups, meta_source=str(meta.meta_source))

    if meta.groups != 1 and op not in ("grouped_conv2d", "depthwise_conv2d"):
        dec.support_status = "unsupported_groups"
        return _fallback(dec, "unsupported_groups", "unsupported_groups!=1", 1.0)
    if op == "unknown":
        dec.support_status = "unsupported_op"
        return _fallback(dec, "unsupported_op", "unsupported_op_fallback_dense", 0.7)
    if agr < 0 or tzr < 0:
        dec.diag_source = "missing"
        return _fallback(dec, "missing_diag", "missing_diag_fallback_dense", 0.2)

    nz = max(1.0 - tzr, NUMERIC_EPS)
    agr_nz = min(agr / nz, 1.0)
    r_exec = tzr + nz * (1.0 - agr_nz)
    r_mismatch = abs(r_exec - (1.0 - agr))
    agr_p90 = float(diag.get("active_group_ratio_p90", -1.0))
    r_worst = 1.0 - agr_p90 if agr_p90 >= 0 else -1.0

    # Tile count: measured, else the output geometry over an estimated tile size.
    if tiles_diag > 0:
        n_tiles, dec.tile_source = float(tiles_diag), "diag"
    elif meta.h_out <= 0 or meta.w_out <= 0:
        n_tiles, dec.tile_source = 1.0, "estimated_default"
    else:
        bm = _block_m_estimate(meta.h_out, meta.w_out)
        n_tiles = float(max(int(meta.batch_size), 1) * max(-(-(meta.h_out * meta.w_out) // bm), 1))
        dec.tile_source = "meta_geometry"

    macs, estimated = float(meta.macs), False
    if macs <= 0 and meta.c_in > 0 and meta.c_out > 0:
        kt = str(diag.get("kernel_type", "")).lower()
        linear_like = _two(meta.kernel_size) == (1, 1) and meta.h_out <= 1 and meta.w_out <= 1 and meta.groups == 1
        bm_diag = float(diag.get("block_m", -1))
        if kt == "linear" and linear_like:
            macs = float(max(n_tiles * (bm_diag if bm_diag > 0 else 32.0), 1.0) * meta.c_in * meta.c_out)
            estimated = True
        elif meta.h_out > 0 and meta.w_out > 0:
            bm = bm_diag if bm_diag > 0 else float(_block_m_estimate(meta.h_out, meta.w_out))
            per_img_tiles = max(math.ceil(meta.h_out * meta.w_out / max(bm, 1.0)), 1.0)
            kh, kw = _two(meta.kernel_size)
            macs = float(max(n_tiles / per_img_tiles, 1.0) * meta.h_out * meta.w_out * meta.c_out * kh * kw
                         * (meta.c_in / max(meta.groups, 1)))
            estimated = True
    if estimated and dec.meta_source == "measured":
        dec.meta_source = "estimated"
    dec.macs = macs
    if macs <= 0:
        if dec.meta_source == "measured":
            dec.meta_source = "fallback"
        return _fallback(dec, "missing_meta", "missing_meta_fallback_dense", 0.2)

    # Per-image intensity: batched tile counts against per-image MACs when the meta has no batch.
    batch = max(int(meta.batch_size), 1)
    if op in ("conv", "depthwise_conv2d", "grouped_conv2d") and batch <= 1 and n_tiles > 0:
        per_img = max(math.ceil(meta.h_out * meta.w_out / max(float(diag.get("block_m", 64)), 1.0)), 1.0)
        batch = max(int(round(n_tiles / per_img)), 1)
    I_l = macs / max(n_tiles / batch, 1.0)
    S_l = r_exec * I_l
    tau, family = _tau_for(meta, diag)
    tau_gate, r_gate = tau * (1.0 + DISPATCH_TAU_MARGIN), DISPATCH_R_MIN + DISPATCH_R_MARGIN
    dec.score_family, dec.R_l, dec.I_l, dec.S_l, dec.agr_nz = family, r_exec, I_l, S_l, agr_nz
    dec.agr_p90, dec.r_worst, dec.n_tiles, dec.tau = agr_p90, r_worst, n_tiles, tau
    dec.score_sparse = S_l / tau if tau > 0 else 0.0
    suffix = ("|macs_estimated" if estimated else "") + ("|R_mismatch_check" if r_mismatch > 1e-4 else "")

    if r_exec >= R_NEAR_ONE:
        dec.backend, dec.reason_code, dec.fallback_reason = "sparse", "R_near_one", ""
        dec.reason = f"R={r_exec:.4f}>={R_NEAR_ONE}{suffix}"
        dec.confidence = max(dec.confidence, 0.95)
        return dec
    if 0 <= r_worst < r_gate:
        dec.backend, dec.reason_code = "dense", "R_guard_worst"
        dec.reason = f"R_worst={r_worst:.3f}<R_min={r_gate:.3f}{suffix}"
    elif r_exec < r_gate:
        dec.backend, dec.reason_code = "dense", "R_guard"
        dec.reason = f"R={r_exec:.3f}<R_min={r_gate:.3f}{suffix}"
    elif S_l > tau_gate:
        dec.backend, dec.reason_code = "sparse", "score_pass"
        dec.reason = f"S={S_l:.0f}>tau={tau_gate:.0f}{suffix}"
    else:
        dec.backend, dec.reason_code = "dense", "score_fail"
        dec.reason = f"S={S_l:.0f}<=tau={tau_gate:.0f}{suffix}"
    dec.fallback_reason = "" if dec.backend == "sparse" else dec.reason_code

    conf = 1.0
    conf *= 0.5 if dec.diag_source != "measured" else 1.0
    conf *= 0.75 if dec.meta_source != "measured" else 1.0
    conf *= 0.9 if dec.tile_source != "diag" else 1.0
    conf *= 0.8 if r_mismatch > 1e-4 else 1.0
    dec.confidence = max(0.0, min(1.0, conf))
    if dec.backend == "sparse" and dec.confidence < DISPATCH_MIN_CONFIDENCE:
        dec.backend, dec.reason_code, dec.fallback_reason = "dense", "low_confidence", "low_confidence"
        dec.reason = f"low_confidence<{DISPATCH_MIN_CONFIDENCE:.2f}{suffix}"
    return dec


def _staticzero_decision(name: str) -> DispatchDecision:
    """A layer whose input is identically zero: all work saved (reference :1021-1046)."""
    return DispatchDecision(layer_name=name, backend="staticzero", reason="exact_zero_input_shortcut",
                            reason_code="exact_zero", fallback_reason="exact_zero_shortcut", meta_source="shortcut",
                            diag_source="shortcut", support_status="exact_zero_shortcut", score_family="none",
                            tile_source="unknown", confidence=1.0, agr=0.0, tzr=1.0, R_l=1.0, agr_nz=0.0,
                            score_sparse=float("inf"), denseish_ratio=0.0, sparse_tile_ratio=0.0)


def _pool_decision(name: str, op_type: str, module: Optional[nn.Module]) -> DispatchDecision:
    """Pools stay dense: sparse pools are out of this build's scope (reference :1049-1138 defaults to dense)."""
    code, reason = "pool_replacement_disabled", f"pool_replacement_disabled_{op_type}"
    if module is not None and bool(getattr(module, "ceil_mode", False)):
        code, reason = "unsupported_pool_ceil_mode", f"unsupported_pool_ceil_mode_{op_type}"
    elif module is not None and op_type == "maxpool2d" and bool(getattr(module, "return_indices", False)):
        code, reason = "unsupported_pool_return_indices", "unsupported_pool_return_indices_maxpool2d"
    return DispatchDecision(layer_name=name, backend="dense", reason=reason, reason_code=code, fallback_reason=code,
                            meta_source="shortcut", diag_source="shortcut", support_status="unsupported_op",
                            score_family="pool", tile_source="unknown", confidence=1.0, agr=0.0, tzr=0.0, R_l=0.0,
                            agr_nz=0.0, score_sparse=0.0, denseish_ratio=0.0, sparse_tile_ratio=0.0)


def dispatch_all_layers(targets, group_sparsity_data: Dict[str, Dict], zero_layers=None) -> Dict[str, DispatchDecision]:
    """Decisions for every target: layer name -> DispatchDecision (reference :1141-1182)."""
    zero_layers = set(zero_layers or ())
    out: Dict[str, DispatchDecision] = {}
    for t in targets:
        name = _layer_name(t)
        if not name:
            continue
        op = str(_field(t, "op_type", ""))
        if op in ("maxpool2d", "avgpool2d"):
            out[name] = _pool_decision(name, op, _field(t, "module") or _field(t, "conv_module"))
        elif name in zero_layers:
            out[name] = _staticzero_decision(name)
        else:
            out[name] = make_dispatch_decision(group_sparsity_data.get(name, {}), op_meta_from_target(t))
    return out


def decisions_to_sets(decisions: Dict[str, DispatchDecision]) -> Tuple[Set[str], Set[str]]:
    """(staticzero layer names, sparse layer names)."""
    return ({n for n, d in decisions.items() if d.backend == "staticzero"},
            {n for n, d in decisions.items() if d.backend == "sparse"})


def collect_layer_diags(model: nn.Module, sample_input: torch.Tensor) -> Dict[str, Dict[str, Any]]:
    """One forward of ``model`` with diagnostics on every SparseConv2d: layer name -> ``_last_diag``.

    Diagnostics read the prescan's tile statistics back to the host (one sync per layer), so this is a
    calibration step, not part of the timed path. Inference mode is suspended for the pass.
    """
    from ..Ops.sparse_conv2d import SparseConv2d
    saved = {}
    for name, m in model.named_modules():
        if isinstance(m, SparseConv2d):
            saved[name] = (m.collect_diag, m._inference_mode)
            m.collect_diag = True
            m._inference_mode = False
    try:
        with torch.no_grad():
            model(sample_input)
    finally:
        for name, m in model.named_modules():
            if name in saved:
                m.collect_diag, m._inference_mode = saved[name]
    return {name: dict(m._last_diag) for name, m in model.named_modules()
            if name in saved and m._last_diag}


def apply_dispatch(model: nn.Module, decisions: Dict[str, DispatchDecision]) -> int:
    """Route each SparseConv2d dispatched "dense" to cuDNN (``dispatch_backend = "dense"``).

    The module keeps its parameters, state_dict keys and 4-D / 5-D input handling; "sparse" and
    "staticzero" layers are set back to the sparse path. Returns the number of layers routed dense.
    """
    from ..Ops.sparse_conv2d import SparseConv2d
    n = 0
    for name, dec in decisions.items():
        if not name:
            continue
        try:
            mod = model.get_submodule(name)
        except AttributeError:
            continue
        if not isinstance(mod, SparseConv2d):
            continue
        mod.dispatch_backend = "dense" if dec.backend == "dense" else "sparse"
        n += dec.backend == "dense"
    return n
