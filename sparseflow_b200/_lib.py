"""ctypes binding of ``libsparseflow_b200.so`` (the C ABI in include/sparseflow_b200.h).

This module is the only place Python touches the native library. It converts
torch CUDA tensors to raw pointers, passes torch's current CUDA stream, and
turns a non-zero status into an exception. There is no fallback: if the
library is missing or a call fails, the error propagates to the caller.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading
from pathlib import Path
from typing import Optional

import torch

import os

# SPARSEFLOW_B200_LIB may point at another build of the same ABI (e.g. an
# instrumented one); by default the in-tree library is used.
LIB_PATH = Path(os.environ.get("SPARSEFLOW_B200_LIB", Path(__file__).resolve().parent / "libsparseflow_b200.so"))

SF_OK = 0
SF_ERR_INVALID_ARG = 1
SF_ERR_UNSUPPORTED = 2
SF_ERR_ALIGNMENT = 3
SF_ERR_WORKSPACE = 4
SF_ERR_CUDA = 5
SF_ERR_DEVICE_TIMEOUT = 6

SF_DTYPE_F32, SF_DTYPE_F16, SF_DTYPE_BF16 = 0, 1, 2
SF_LAYOUT_NCHW, SF_LAYOUT_NHWC = 0, 1
# Path policy keys (sf_set_path_policy).
SF_POLICY_CONV1X1_PATH, SF_POLICY_CONV1X1_TC_MIN_HW, SF_POLICY_CONV3X3_PATH, SF_POLICY_LIF_EVENTS_GENERAL = 0, 1, 2, 3
SF_POLICY_LIF_TC_EPILOGUE = 4

_TORCH2SF = {torch.float32: SF_DTYPE_F32, torch.float16: SF_DTYPE_F16, torch.bfloat16: SF_DTYPE_BF16}


class SparseFlowError(RuntimeError):
    """A native entry point returned a non-OK status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: {msg} (status {status})")
        self.status = status


class PrescanDesc(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int32), ("c", ctypes.c_int32), ("h", ctypes.c_int32), ("w", ctypes.c_int32),
        ("h_out", ctypes.c_int32), ("w_out", ctypes.c_int32),
        ("kernel", ctypes.c_int32), ("stride", ctypes.c_int32), ("padding", ctypes.c_int32),
        ("block_h", ctypes.c_int32), ("block_w", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("threshold", ctypes.c_double),
        ("dtype", ctypes.c_int32), ("layout", ctypes.c_int32),
    ]


class ConvDesc(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int32), ("c_in", ctypes.c_int32), ("h", ctypes.c_int32), ("w", ctypes.c_int32),
        ("c_out", ctypes.c_int32), ("h_out", ctypes.c_int32), ("w_out", ctypes.c_int32),
        ("kernel", ctypes.c_int32), ("stride", ctypes.c_int32), ("padding", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32), ("w_dtype", ctypes.c_int32), ("has_bias", ctypes.c_int32),
    ]


class LifDesc(ctypes.Structure):
    _fields_ = [
        ("t_steps", ctypes.c_int32), ("n", ctypes.c_int32), ("c_in", ctypes.c_int32),
        ("h", ctypes.c_int32), ("w", ctypes.c_int32),
        ("c_out", ctypes.c_int32), ("h_out", ctypes.c_int32), ("w_out", ctypes.c_int32),
        ("kernel", ctypes.c_int32), ("stride", ctypes.c_int32), ("padding", ctypes.c_int32),
        ("tau", ctypes.c_float), ("v_threshold", ctypes.c_float), ("v_reset", ctypes.c_float),
        ("hard_reset", ctypes.c_int32), ("decay_input", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32), ("w_dtype", ctypes.c_int32), ("has_bias", ctypes.c_int32),
    ]


class LifMsDesc(ctypes.Structure):
    _fields_ = [
        ("numel", ctypes.c_int64), ("t_steps", ctypes.c_int32),
        ("tau", ctypes.c_float), ("v_threshold", ctypes.c_float), ("v_reset", ctypes.c_float),
        ("hard_reset", ctypes.c_int32), ("decay_input", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32), ("s_dtype", ctypes.c_int32),
    ]


# Every symbol declared in include/sparseflow_b200.h, with its ctypes signature.
_VP = ctypes.c_void_p
_SIGNATURES = {
    "sf_abi_version": (ctypes.c_int32, []),
    "sf_status_string": (ctypes.c_char_p, [ctypes.c_int32]),
    "sf_prescan2d_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(PrescanDesc)]),
    "sf_prescan2d": (ctypes.c_int32, [_VP, ctypes.POINTER(PrescanDesc), _VP, _VP, _VP, _VP, _VP,
                                      ctypes.c_size_t, _VP]),
    "sf_prescan2d_status": (ctypes.c_int32, [_VP, _VP]),
    "sf_prescan2d_static_ws": (ctypes.c_int32, [_VP, ctypes.POINTER(PrescanDesc), _VP, _VP, _VP, _VP, _VP]),
    "sf_prescan2d_static_ws_status": (ctypes.c_int32, [_VP]),
    "sf_packed_weight_bytes": (ctypes.c_size_t, [ctypes.c_int32] * 4),
    "sf_pack_weights": (ctypes.c_int32, [_VP, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_int32, _VP, _VP]),
    "sf_sparse_conv2d_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(ConvDesc)]),
    "sf_sparse_conv2d": (ctypes.c_int32, [_VP, _VP, _VP, _VP, ctypes.POINTER(ConvDesc), _VP, ctypes.c_size_t, _VP]),
    "sf_sparse_conv2d_status": (ctypes.c_int32, [_VP]),
    "sf_fused_conv_lif_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(LifDesc)]),
    "sf_fused_conv_lif": (ctypes.c_int32, [_VP, _VP, _VP, _VP, _VP, _VP, ctypes.POINTER(LifDesc), _VP, ctypes.c_size_t,
                                           _VP]),
    "sf_lif_multistep": (ctypes.c_int32, [_VP, _VP, _VP, ctypes.POINTER(LifMsDesc), _VP]),
    "sf_lif_multistep_events": (ctypes.c_int32, [_VP, _VP, _VP, _VP, ctypes.POINTER(LifMsDesc), ctypes.c_int32,
                                                 ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _VP]),
    "sf_event_masks_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "sf_selftest_bounded_wait": (ctypes.c_int32, [ctypes.c_uint64, _VP]),
    "sf_set_path_policy": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_int64]),
    "sf_get_path_policy": (ctypes.c_int64, [ctypes.c_int32]),
    "sf_sparse_conv2d_from_masks": (ctypes.c_int32, [_VP, _VP, _VP, _VP, ctypes.POINTER(ConvDesc), _VP]),
    "sf_sparse_conv2d_masks_or_x_workspace_size": (ctypes.c_size_t, []),
    "sf_sparse_conv2d_masks_or_x": (ctypes.c_int32, [_VP, _VP, _VP, _VP, _VP, ctypes.POINTER(ConvDesc), _VP,
                                                     ctypes.c_size_t, _VP]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the native library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m sparseflow_b200.build` "
                    "(the sparse path has no CPU or dense fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.sf_abi_version() != 1:
                raise RuntimeError("libsparseflow_b200.so ABI version mismatch")
            _lib = lib
    return _lib


def declared_symbols() -> list[str]:
    return list(_SIGNATURES)


def _check(fn: str, status: int) -> None:
    if status != SF_OK:
        msg = load().sf_status_string(status).decode()
        raise SparseFlowError(fn, status, msg)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return raw_stream(idx)


def sf_dtype(dt: torch.dtype) -> int:
    try:
        return _TORCH2SF[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16") from None


def _require_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("sparseflow_b200 kernels need CUDA tensors (there is no CPU path)")


# ----------------------------------------------------------------------------
# Prescan
# ----------------------------------------------------------------------------

def prescan_desc(n, c, h, w, h_out, w_out, kernel, stride, padding, block_h, block_w, group_size,
                 threshold, dtype: torch.dtype, layout: int) -> PrescanDesc:
    return PrescanDesc(n, c, h, w, h_out, w_out, kernel, stride, padding, block_h, block_w, group_size,
                       float(threshold), sf_dtype(dtype), layout)


def prescan_workspace_bytes(desc: PrescanDesc) -> int:
    nbytes = load().sf_prescan2d_workspace_size(ctypes.byref(desc))
    if nbytes == 0:
        raise SparseFlowError("sf_prescan2d_workspace_size", SF_ERR_INVALID_ARG, "invalid descriptor")
    return int(nbytes)


def prescan2d(x: torch.Tensor, desc: PrescanDesc, ag_mask: torch.Tensor, tile_class: torch.Tensor,
              active_ids: Optional[torch.Tensor], active_count: Optional[torch.Tensor],
              workspace: torch.Tensor) -> None:
    _require_cuda(x, ag_mask, tile_class, active_ids, active_count, workspace)
    st = load().sf_prescan2d(_ptr(x), ctypes.byref(desc), _ptr(ag_mask), _ptr(tile_class), _ptr(active_ids),
                             _ptr(active_count), _ptr(workspace), workspace.numel() * workspace.element_size(),
                             _stream(x.device))
    _check("sf_prescan2d", st)


def prescan_status(workspace: torch.Tensor) -> int:
    return int(load().sf_prescan2d_status(_ptr(workspace), _stream(workspace.device)))


def conv_status(device: torch.device) -> int:
    return int(load().sf_sparse_conv2d_status(_stream(device)))


# ----------------------------------------------------------------------------
# Weights and convolution
# ----------------------------------------------------------------------------

def pack_weights(weight: torch.Tensor, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """[C_out, C_in, k, k] -> packed [block][C_in][k*k][32][cpl], block = 32*cpl output channels
    (zero padded past C_out; cpl chosen by the library so one block fits shared memory)."""
    _require_cuda(weight)
    w = weight.detach().contiguous()
    co, ci, kh, kw = w.shape
    if kh != kw:
        raise ValueError("only square kernels are packed")
    dst = sf_dtype(out_dtype)
    nbytes = load().sf_packed_weight_bytes(co, ci, kh, dst)
    out = torch.empty(nbytes // torch.tensor([], dtype=out_dtype).element_size(), dtype=out_dtype, device=w.device)
    st = load().sf_pack_weights(_ptr(w), sf_dtype(w.dtype), co, ci, kh, dst, _ptr(out), _stream(w.device))
    _check("sf_pack_weights", st)
    return out


_ws_lock = threading.Lock()
_workspaces: dict = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-(device, stream) scratch buffer for the conv entry points, grown on demand.

    Calls on one stream run in order, so they can share it; another stream
    gets its own.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return workspace_on(idx, torch.cuda.current_stream(device).cuda_stream, nbytes)


def workspace_on(idx: int, stream: int, nbytes: int) -> torch.Tensor:
    """workspace() for a device index and a raw stream handle the caller already has."""
    key = (idx, stream)
    buf = _workspaces.get(key)
    if buf is not None and buf.numel() >= nbytes:
        return buf
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[key] = buf
    return buf


def raw_stream(idx: int) -> int:
    """Handle of the current stream of device idx (what torch.cuda.current_stream(idx).cuda_stream
    returns, without building the Stream object)."""
    return torch._C._cuda_getCurrentRawStream(idx)


def sparse_conv2d(x: torch.Tensor, w_packed: torch.Tensor, bias: Optional[torch.Tensor], y: torch.Tensor,
                  c_out: int, kernel: int, stride: int, padding: int) -> None:
    _require_cuda(x, w_packed, bias, y)
    n, c, h, w = x.shape
    _, co, ho, wo = y.shape
    desc = ConvDesc(n, c, h, w, co, ho, wo, kernel, stride, padding, sf_dtype(x.dtype), sf_dtype(w_packed.dtype),
                    int(bias is not None))
    lib = load()
    nbytes = lib.sf_sparse_conv2d_workspace_size(ctypes.byref(desc))
    ws = workspace(x.device, nbytes)
    st = lib.sf_sparse_conv2d(_ptr(x), _ptr(w_packed), _ptr(bias), _ptr(y), ctypes.byref(desc), _ptr(ws),
                              ws.numel(), _stream(x.device))
    _check("sf_sparse_conv2d", st)


def event_masks_bytes(n_images: int, channels: int, h: int, w: int) -> int:
    return int(load().sf_event_masks_bytes(n_images, channels, h, w))


def sparse_conv2d_from_masks(masks: torch.Tensor, x_shape, x_dtype: torch.dtype, w_packed: torch.Tensor,
                             bias: Optional[torch.Tensor], y: torch.Tensor, kernel: int, stride: int,
                             padding: int) -> None:
    """Convolution of binary spikes of shape x_shape = (n, c, h, w) given their event masks."""
    _require_cuda(masks, w_packed, bias, y)
    n, c, h, w = x_shape
    _, co, ho, wo = y.shape
    desc = ConvDesc(n, c, h, w, co, ho, wo, kernel, stride, padding, sf_dtype(x_dtype), sf_dtype(w_packed.dtype),
                    int(bias is not None))
    st = load().sf_sparse_conv2d_from_masks(_ptr(masks), _ptr(w_packed), _ptr(bias), _ptr(y), ctypes.byref(desc),
                                            _stream(y.device))
    _check("sf_sparse_conv2d_from_masks", st)


def sparse_conv2d_masks_or_x(x: torch.Tensor, masks: torch.Tensor, w_packed: torch.Tensor,
                             bias: Optional[torch.Tensor], y: torch.Tensor, kernel: int, stride: int,
                             padding: int) -> None:
    """Convolution of binary spikes x given x and its event masks: a sampled density picks the
    gather kernel from the masks or the tensor cores from x on the device."""
    _require_cuda(x, masks, w_packed, bias, y)
    n, c, h, w = x.shape
    _, co, ho, wo = y.shape
    desc = ConvDesc(n, c, h, w, co, ho, wo, kernel, stride, padding, sf_dtype(x.dtype), sf_dtype(w_packed.dtype),
                    int(bias is not None))
    lib = load()
    ws = torch.empty(int(lib.sf_sparse_conv2d_masks_or_x_workspace_size()), dtype=torch.uint8, device=x.device)
    st = lib.sf_sparse_conv2d_masks_or_x(_ptr(x), _ptr(masks), _ptr(w_packed), _ptr(bias), _ptr(y),
                                         ctypes.byref(desc), _ptr(ws), ws.numel(), _stream(y.device))
    _check("sf_sparse_conv2d_masks_or_x", st)


def fused_conv_lif(x5: torch.Tensor, w_packed: torch.Tensor, bias: Optional[torch.Tensor], v: torch.Tensor,
                   spikes: torch.Tensor, kernel: int, stride: int, padding: int, tau: float, v_threshold: float,
                   v_reset: Optional[float], decay_input: bool, masks_out: Optional[torch.Tensor] = None) -> None:
    _require_cuda(x5, w_packed, bias, v, spikes, masks_out)
    t, n, c, h, w = x5.shape
    _, _, co, ho, wo = spikes.shape
    desc = LifDesc(t, n, c, h, w, co, ho, wo, kernel, stride, padding, float(tau), float(v_threshold),
                   0.0 if v_reset is None else float(v_reset), int(v_reset is not None), int(bool(decay_input)),
                   sf_dtype(x5.dtype), sf_dtype(w_packed.dtype), int(bias is not None))
    lib = load()
    nbytes = lib.sf_fused_conv_lif_workspace_size(ctypes.byref(desc))
    ws = workspace(x5.device, nbytes)
    st = lib.sf_fused_conv_lif(_ptr(x5), _ptr(w_packed), _ptr(bias), _ptr(v), _ptr(spikes), _ptr(masks_out),
                               ctypes.byref(desc), _ptr(ws), ws.numel(), _stream(x5.device))
    _check("sf_fused_conv_lif", st)


def lif_multistep(x: torch.Tensor, v: torch.Tensor, spikes: torch.Tensor, tau: float, v_threshold: float,
                  v_reset: Optional[float], decay_input: bool) -> None:
    """x, spikes: [T, ...] contiguous; v: fp32 [...] contiguous, updated in place."""
    _require_cuda(x, v, spikes)
    if v.dtype != torch.float32 or not (x.is_contiguous() and v.is_contiguous() and spikes.is_contiguous()):
        raise ValueError("lif_multistep needs contiguous tensors and an fp32 membrane")
    t = x.shape[0]
    numel = x.numel() // t if t > 0 else v.numel()
    if v.numel() != numel or spikes.shape != x.shape:
        raise ValueError("shape mismatch between x, v and spikes")
    desc = LifMsDesc(numel, t, float(tau), float(v_threshold), 0.0 if v_reset is None else float(v_reset),
                     int(v_reset is not None), int(bool(decay_input)), sf_dtype(x.dtype), sf_dtype(spikes.dtype))
    st = load().sf_lif_multistep(_ptr(x), _ptr(v), _ptr(spikes), ctypes.byref(desc), _stream(x.device))
    _check("sf_lif_multistep", st)


def lif_multistep_events(x: torch.Tensor, v: torch.Tensor, spikes: torch.Tensor, masks: torch.Tensor, tau: float,
                         v_threshold: float, v_reset: Optional[float], decay_input: bool) -> None:
    """lif_multistep on x = [T, N, C, H, W] that also writes the spikes' event masks into ``masks``
    (sf_event_masks_bytes(T*N, C, H, W) bytes, 8-byte aligned)."""
    _require_cuda(x, v, spikes, masks)
    if v.dtype != torch.float32 or not (x.is_contiguous() and v.is_contiguous() and spikes.is_contiguous()):
        raise ValueError("lif_multistep_events needs contiguous tensors and an fp32 membrane")
    if x.dim() != 5:
        raise ValueError(f"lif_multistep_events needs a 5-D [T, N, C, H, W] input, got {x.dim()}-D")
    t, n, c, h, w = x.shape
    if tuple(v.shape) != (n, c, h, w) or spikes.shape != x.shape:
        raise ValueError("shape mismatch between x, v and spikes")
    if masks.numel() * masks.element_size() < event_masks_bytes(t * n, c, h, w):
        raise ValueError("event-mask buffer too small")
    desc = LifMsDesc(n * c * h * w, t, float(tau), float(v_threshold), 0.0 if v_reset is None else float(v_reset),
                     int(v_reset is not None), int(bool(decay_input)), sf_dtype(x.dtype), sf_dtype(spikes.dtype))
    st = load().sf_lif_multistep_events(_ptr(x), _ptr(v), _ptr(spikes), _ptr(masks), ctypes.byref(desc), n, c, h, w,
                                        _stream(x.device))
    _check("sf_lif_multistep_events", st)


def set_path_policy(key: int, value: int) -> int:
    """Sets a process-wide path policy value; returns the previous one."""
    lib = load()
    prev = int(lib.sf_get_path_policy(key))
    _check("sf_set_path_policy", lib.sf_set_path_policy(key, int(value)))
    return prev


@contextlib.contextmanager
def path_policy(key: int, value: int):
    """with path_policy(SF_POLICY_CONV3X3_PATH, 1): ... -- the policy applies inside the block only."""
    prev = set_path_policy(key, value)
    try:
        yield
    finally:
        set_path_policy(key, prev)
