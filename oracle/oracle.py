"""Python side of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

* ``prescan2d`` / ``conv2d`` / ``conv_lif`` call the plain-C restatement in
  sf_oracle.c (built into liboracle_sf.so by the Makefile next to it).
* ``reference_cpu_conv2d`` / ``reference_cpu_conv_bn_lif`` restate the
  reference's own CPU path: SparseConv2d on a CPU tensor is F.conv2d
  (Ops/sparse_conv2d.py:557, 595-596, 819-834) and the conv+LIF module's CPU
  path is F.conv2d followed by the LIF update (Ops/sparse_fused_conv_lif.py:
  271-293). These are what bench.py times as the CPU baseline.

Pinned by tests/test_oracle_golden.py against fixtures generated from the
reference itself (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle_sf.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def _load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = ctypes.CDLL(str(LIB))
        f = ctypes.c_void_p
        i = ctypes.c_int
        lib.oracle_prescan2d.restype = i
        lib.oracle_prescan2d.argtypes = [f, i, i, i, i, i, i, i, i, i, i, i, i, i, ctypes.c_float, f, f, f, f]
        lib.oracle_conv2d.restype = None
        lib.oracle_conv2d.argtypes = [f, i, i, i, i, f, f, i, i, i, i, f]
        lib.oracle_lif_step.restype = None
        lib.oracle_lif_step.argtypes = [f, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_float, i, i, f, f]
        lib.oracle_conv_lif.restype = None
        lib.oracle_conv_lif.argtypes = [f, i, i, i, i, i, f, f, i, i, i, i, ctypes.c_float, ctypes.c_float,
                                        ctypes.c_float, i, i, f, f]
        _lib = lib
    return _lib


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def choose_group_size(c_in: int) -> int:
    """Kernels/conv2d.py:64-73."""
    gs = 16 if c_in <= 128 else 32
    while (c_in + gs - 1) // gs > 32:
        gs *= 2
    return gs


def tile_sizes(h_out: int, w_out: int):
    """Kernels/conv2d.py:80-84."""
    return (8, 16) if h_out * w_out >= 3136 else (8, 8)


def half_round(x: np.ndarray) -> np.ndarray:
    """x -> nearest IEEE half (ties to even), back as float32 (x.half() in the reference)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def prescan2d(x: np.ndarray, layout: int, ho: int, wo: int, k: int, s: int, p: int, bh: int, bw: int, gs: int,
              threshold: float):
    """Returns (ag_mask int32[n_tiles], tile_class int32[n_tiles], active_ids int32[count])."""
    xh = np.ascontiguousarray(half_round(x))
    if layout == 0:
        n, c, h, w = xh.shape
    else:
        n, h, w, c = xh.shape
    thr = float(np.float16(threshold))
    gh, gw = -(-ho // bh), -(-wo // bw)
    nt = n * gh * gw
    ag = np.zeros(nt, np.int32)
    tc = np.zeros(nt, np.int32)
    ids = np.zeros(max(nt, 1), np.int32)
    cnt = np.zeros(1, np.int32)
    rc = _load().oracle_prescan2d(_p(xh), layout, n, c, h, w, ho, wo, k, s, p, bh, bw, gs, thr, _p(ag), _p(tc),
                                  _p(ids), _p(cnt))
    if rc != 0:
        raise ValueError(f"oracle_prescan2d failed ({rc})")
    return ag, tc, ids[: int(cnt[0])].copy()


def conv2d(x: np.ndarray, w: np.ndarray, b: Optional[np.ndarray], stride: int, padding: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    b = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    n, c, h, wd = x.shape
    co, _, k, _ = w.shape
    ho, wo = (h + 2 * padding - k) // stride + 1, (wd + 2 * padding - k) // stride + 1
    y = np.empty((n, co, ho, wo), np.float32)
    _load().oracle_conv2d(_p(x), n, c, h, wd, _p(w), _p(b), co, k, stride, padding, _p(y))
    return y


def lif_step(current: np.ndarray, v: np.ndarray, tau: float, v_threshold: float, v_reset: Optional[float],
             decay_input: bool):
    """One LIF step; returns (spikes, v_next) as new float32 arrays."""
    cur = np.ascontiguousarray(current, dtype=np.float32)
    vv = np.array(v, dtype=np.float32, copy=True)
    sp = np.empty_like(cur)
    _load().oracle_lif_step(_p(cur), cur.size, tau, v_threshold, 0.0 if v_reset is None else v_reset,
                            int(v_reset is not None), int(decay_input), _p(vv), _p(sp))
    return sp, vv


def conv_lif(x5: np.ndarray, w: np.ndarray, b: Optional[np.ndarray], v0: np.ndarray, stride: int, padding: int,
             tau: float, v_threshold: float, v_reset: Optional[float], decay_input: bool,
             bn: Optional[dict] = None):
    """Multi-step conv (+ eval BN given as dict mean/var/gamma/beta/eps) + LIF.

    Returns (spikes [T, N, Co, Ho, Wo], v_final)."""
    v = np.array(v0, dtype=np.float32, copy=True)
    outs = []
    for t in range(x5.shape[0]):
        cur = conv2d(x5[t], w, b, stride, padding)
        if bn is not None:
            scale = (bn["gamma"] / np.sqrt(bn["var"].astype(np.float32) + np.float32(bn["eps"]))).astype(np.float32)
            cur = ((cur - bn["mean"].reshape(1, -1, 1, 1)) * scale.reshape(1, -1, 1, 1)
                   + bn["beta"].reshape(1, -1, 1, 1)).astype(np.float32)
        sp, v = lif_step(cur, v, tau, v_threshold, v_reset, decay_input)
        outs.append(sp)
    return np.stack(outs, 0), v


def conv_lif_near(x5: np.ndarray, w: np.ndarray, b: Optional[np.ndarray], v0: np.ndarray, stride: int,
                  padding: int, tau: float, v_threshold: float, v_reset: Optional[float], decay_input: bool,
                  bn: Optional[dict] = None):
    """conv_lif plus the near-threshold mask: (spikes, near, v_final), near[t] marking
    where the pre-spike membrane (Ops/sparse_fused_conv_lif.py:271-293, v_tmp) lies
    within 1e-5 of v_threshold -- the only places a spike may differ from the
    reference, whose conv sums run in another order."""
    v = np.array(v0, dtype=np.float32, copy=True)
    vr = np.float32(0.0 if v_reset is None else v_reset)
    sps, near = [], []
    for t in range(x5.shape[0]):
        cur = conv2d(x5[t], w, b, stride, padding)
        if bn is not None:
            scale = (bn["gamma"] / np.sqrt(bn["var"].astype(np.float32) + np.float32(bn["eps"]))).astype(np.float32)
            cur = ((cur - bn["mean"].reshape(1, -1, 1, 1)) * scale.reshape(1, -1, 1, 1)
                   + bn["beta"].reshape(1, -1, 1, 1)).astype(np.float32)
        tau32 = np.float32(tau)
        vt = v + (cur - (v - vr)) / tau32 if decay_input else v - (v - vr) / tau32 + cur
        near.append(np.abs(vt - np.float32(v_threshold)) < 1e-5)
        sp, v = lif_step(cur, v, tau, v_threshold, v_reset, decay_input)
        sps.append(sp)
    return np.stack(sps, 0), np.stack(near, 0), v


def spikes_match(got: np.ndarray, ref: np.ndarray, near: np.ndarray) -> bool:
    """The fused-LIF parity rule: spikes [T, ...] identical except where |v - v_th| < 1e-5.
    Once a near-tie spike flips, that neuron's later trajectory legitimately
    differs, so only the first mismatch of each neuron is held to the rule."""
    diff = np.asarray(got) != np.asarray(ref)
    first = diff & (np.cumsum(diff, axis=0) == 1)
    return not bool(np.any(first & ~np.asarray(near)))


# ---------------------------------------------------------------------------
# The reference's CPU path, timed as the CPU baseline.
# ---------------------------------------------------------------------------

def reference_cpu_conv2d(x, weight, bias, stride, padding):
    """SparseConv2d's CPU path: F.conv2d on the (folded T*N) input (Ops/sparse_conv2d.py:819-834)."""
    import torch.nn.functional as F
    lead = None
    if x.dim() == 5:
        lead = x.shape[:2]
        x = x.reshape(-1, *x.shape[2:])
    y = F.conv2d(x, weight.to(x.dtype), None if bias is None else bias.to(x.dtype), stride, padding)
    return y if lead is None else y.reshape(*lead, *y.shape[1:])


def reference_cpu_conv_bn_lif(x5, weight, bias, bn_params, tau, v_threshold, v_reset, decay_input):
    """conv -> eval BN -> LIF over T on CPU, as the reference's modules compute it
    (Ops/sparse_fused_conv_lif.py:271-293 per step; BN by F.batch_norm)."""
    import torch
    import torch.nn.functional as F
    v = None
    outs = []
    vr = 0.0 if v_reset is None else float(v_reset)
    for t in range(x5.shape[0]):
        conv = F.conv2d(x5[t], weight, bias, 1, weight.shape[-1] // 2).float()
        if bn_params is not None:
            conv = F.batch_norm(conv, bn_params["mean"], bn_params["var"], bn_params["gamma"], bn_params["beta"],
                                False, 0.0, bn_params["eps"])
        if v is None:
            v = torch.zeros_like(conv)
        if decay_input:
            vt = v + (conv - (v - vr)) / tau
        else:
            vt = v - (v - vr) / tau + conv
        sp = (vt >= v_threshold).to(vt.dtype)
        v = vt - sp * v_threshold if v_reset is None else torch.where(sp.bool(), torch.full_like(vt, vr), vt)
        outs.append(sp)
    return torch.stack(outs, 0), v
