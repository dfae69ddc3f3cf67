"""SparseConv2d: drop-in ``nn.Conv2d`` on the B200 sparse kernels.

Reference: Ops/sparse_conv2d.py:109-848. Kept from the reference:
  * constructor arguments and defaults (:134-145), ``from_dense`` (:498-513);
  * parameters ``weight``/``bias`` registered exactly as ``nn.Conv2d`` does,
    so ``state_dict`` keys are interchangeable;
  * 4-D NCHW and 5-D (T, N, C, H, W) inputs, the output keeping the input's
    rank and dtype (:544-547, :622-627); other ranks raise ValueError (:551);
  * ``block_size`` is stored and reported but does not steer the kernels
    (:114-119, :162);
  * ``_last_sparse_ms`` (CUDA-event time of the sparse launch when
    ``return_ms`` is set, :726-741), ``_last_dense_ms``, ``_last_diag`` when
    ``collect_diag`` is set (:752-816), ``profile_runtime`` statistics
    (:255-289), ``set_inference_mode`` / ``set_launch_all_tiles`` (:234-250).
Changed: there is no silent ``F.conv2d`` fallback. A CPU tensor raises, and
the only dense path is the reference's own one for conv patterns the sparse
kernels do not cover (never chosen by the analyzer).
"""
from __future__ import annotations

import ctypes

import math
import time
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _lib
from ..Kernels.fused_conv_lif import event_masks_of
from ..Kernels.conv2d import (SUPPORTED_PATTERNS, choose_group_size, output_hw, pack_weight,
                              sparse_conv2d_forward)
from ..Utils.sparse_helpers import TILE_DENSEISH, TILE_SPARSE, TILE_ZERO, select_tile_sizes


@dataclass
class _ProfileStats:
    calls: int = 0
    zero_path_hits: int = 0
    sparse_path_hits: int = 0
    dense_path_hits: int = 0
    triton_supported_calls: int = 0
    total_ms: float = 0.0
    policy_ms: float = 0.0
    reshape_ms: float = 0.0
    buffer_ms: float = 0.0
    sparse_kernel_ms: float = 0.0
    dense_fallback_ms: float = 0.0
    output_pack_ms: float = 0.0
    last_path: str = "none"
    last_total_ms: float = 0.0
    last_avg_active_ratio: float = -1.0


class SparseConv2d(nn.Module):
    """Conv2d over spike tensors that skips exact-zero inputs on the GPU."""

    def __init__(
        self,
        in_channels, out_channels, kernel_size,
        stride=1, padding=0, dilation=1, groups=1, bias=True,
        block_size=None, threshold=1e-6, return_ms=False,
        dense_threshold: float = 0.85,
        warmup_steps: int = 8, calib_every: int = 32,
        ema_decay: float = 0.9, zero_streak_needed: int = 2,
        profile_runtime: bool = False,
        allow_sparse_1x1: bool = True,
        launch_all_tiles: bool = False,
    ):
        super().__init__()
        pair = lambda v: (v, v) if isinstance(v, int) else tuple(v)  # noqa: E731
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = pair(kernel_size)
        self.stride = pair(stride)
        self.padding = pair(padding)
        self.dilation = pair(dilation)
        self.groups = groups
        self.block_size = block_size
        self.threshold = threshold
        self.return_ms = return_ms
        self.allow_sparse_1x1 = bool(allow_sparse_1x1)
        self.launch_all_tiles = bool(launch_all_tiles)

        self.weight = nn.Parameter(torch.empty(out_channels, in_channels // groups, *self.kernel_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in = self.in_channels * self.kernel_size[0] * self.kernel_size[1]
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

        # Caches (plain attributes, not buffers: state_dict matches nn.Conv2d).
        self._w_packed = None
        self._w_packed_key = None
        self._fast = None  # plain-call cache (_plain_call)
        self._bias_key = None
        self._bias32 = None
        self._ag_mask_buf = None
        self._tile_class_buf = None
        self._active_tile_ids_buf = None
        self._last_sparse_ms = 0.0
        self._last_dense_ms = 0.0
        self._last_avg_active_ratio = -1.0
        self._dense_threshold = float(dense_threshold)
        self._warmup_left = int(max(0, warmup_steps))
        self._calib_every = int(max(1, calib_every))
        self._inference_mode = False

        self.collect_diag = False
        self._last_diag = {}
        # "dense" when a dispatch decision (Utils.dispatch_model.apply_dispatch) routes this layer to
        # cuDNN: the module keeps its parameters and 4-D / 5-D handling and runs F.conv2d.
        self.dispatch_backend = "sparse"
        self.profile_runtime = profile_runtime
        self._profile = _ProfileStats()
        self.backend_family = "sparse_kernel"
        self.diag_path = "conv2d_b200_gather"
        self.fallback_reason = ""

    # -- switches kept from the reference ---------------------------------
    def set_launch_all_tiles(self, enabled: bool):
        """Kept for API compatibility; the persistent kernel always visits every tile."""
        self.launch_all_tiles = bool(enabled)

    def set_inference_mode(self, enabled: bool):
        """Disable diagnostics and profiling so forward never synchronises."""
        self._inference_mode = bool(enabled)
        if enabled:
            self.collect_diag = False
            self.profile_runtime = False

    @classmethod
    def from_dense(cls, conv: nn.Conv2d, block_size=None, threshold=1e-6, return_ms=False, **kwargs):
        sparse = cls(
            in_channels=conv.in_channels, out_channels=conv.out_channels,
            kernel_size=conv.kernel_size, stride=conv.stride, padding=conv.padding,
            dilation=conv.dilation, groups=conv.groups, bias=conv.bias is not None,
            block_size=block_size, threshold=threshold, return_ms=return_ms, **kwargs,
        )
        sparse = sparse.to(device=conv.weight.device, dtype=conv.weight.dtype)
        sparse.weight.data.copy_(conv.weight.data)
        if conv.bias is not None:
            sparse.bias.data.copy_(conv.bias.data)
        return sparse

    # -- helpers ------------------------------------------------------------
    def _pattern(self):
        return (self.kernel_size[0], self.stride[0], self.padding[0])

    def _supports_sparse(self) -> bool:
        k, s, p = self.kernel_size, self.stride, self.padding
        if k[0] != k[1] or s[0] != s[1] or p[0] != p[1] or self.dilation != (1, 1) or self.groups != 1:
            return False
        if k == (1, 1) and not self.allow_sparse_1x1:
            return False
        return self._pattern() in SUPPORTED_PATTERNS

    def _get_w_packed(self):
        key = (self.weight._version, self.weight.data_ptr())  # .to() gives the parameter new storage
        if self._w_packed is None or self._w_packed_key != key:
            self._w_packed = pack_weight(self.weight.data)
            self._w_packed_key = key
        return self._w_packed

    def _output_hw(self, h_in: int, w_in: int):
        return output_hw(h_in, w_in, self.kernel_size[0], self.stride[0], self.padding[0], self.dilation[0])

    def _stamp(self):
        if self.profile_runtime and self.weight.is_cuda:
            torch.cuda.synchronize(self.weight.device)
        return time.perf_counter()

    def get_profile_summary(self) -> str:
        p = self._profile
        if p.calls == 0:
            return "SparseConv2d runtime profile: no calls"
        avg = lambda v: v / max(1, p.calls)  # noqa: E731
        return (f"SparseConv2d runtime profile\n  calls={p.calls}, last_path={p.last_path}\n"
                f"  hits: sparse={p.sparse_path_hits}, dense={p.dense_path_hits}\n"
                f"  avg: total={avg(p.total_ms):.3f}, sparse_kernel={avg(p.sparse_kernel_ms):.3f}, "
                f"dense_fallback={avg(p.dense_fallback_ms):.3f}\n  last: total={p.last_total_ms:.3f}")

    # -- forward --------------------------------------------------------------
    def forward(self, x: torch.Tensor):
        y = self._plain_call(x)
        if y is not None:
            return y
        self.fallback_reason = ""
        if self.profile_runtime:
            self._profile.calls += 1
            t_total = self._stamp()
        event_masks = event_masks_of(x)  # set when x came straight from a FusedSparseConvLIF
        if x.dim() == 5:
            t, b, c, h, w = x.shape
            x4 = x.reshape(t * b, c, h, w)
        elif x.dim() == 4:
            x4 = x
        else:
            raise ValueError(f"Expected 4D or 5D input, got {x.dim()}D")
        if not x4.is_cuda:
            raise RuntimeError("SparseConv2d runs on CUDA tensors only; the B200 path has no CPU fallback")

        self._last_used_event_masks = False
        if self._supports_sparse() and self.dispatch_backend != "dense":
            y4, backend = self._sparse_forward(x4, event_masks)
        else:
            y4 = F.conv2d(x4, self.weight, self.bias, self.stride, self.padding, self.dilation, self.groups)
            backend = "dense_fallback"
            self.fallback_reason = "dispatch_dense" if self.dispatch_backend == "dense" else "unsupported_pattern"
            self._last_sparse_ms = 0.0
        if self.profile_runtime:
            if backend == "dense_fallback":
                self._profile.dense_path_hits += 1
            else:
                self._profile.sparse_path_hits += 1
            self._profile.sparse_kernel_ms += self._last_sparse_ms
            self._profile.last_path = "sparse" if backend != "dense_fallback" else "dense"
            tot = (self._stamp() - t_total) * 1000.0
            self._profile.total_ms += tot
            self._profile.last_total_ms = tot
        if x.dim() == 5:
            _, co, ho, wo = y4.shape
            return y4.reshape(t, b, co, ho, wo)
        return y4

    def _ensure_buffers(self, x4):
        ho, wo = self._output_hw(x4.shape[2], x4.shape[3])
        bh, bw = select_tile_sizes(ho, wo)
        n_tiles = x4.shape[0] * (-(-ho // bh)) * (-(-wo // bw))
        for name in ("_ag_mask_buf", "_tile_class_buf", "_active_tile_ids_buf"):
            buf = getattr(self, name)
            if buf is None or buf.numel() < n_tiles or buf.device != x4.device:
                setattr(self, name, torch.empty(n_tiles, dtype=torch.int32, device=x4.device))
        return n_tiles

    def _plain_call(self, x):
        """The plain call, on 4-D or 5-D input: no statistics, timing, handed-over event masks or
        dense dispatch. Descriptor, output shape and workspace size are cached per input shape,
        the packed weights and fp32 bias per parameter version; then one library call on the
        current stream. Host time per call matters for small layers (C1: ~10 us of device time).
        None when the call is not a plain one."""
        if (self.profile_runtime or self.return_ms or (self.collect_diag and not self._inference_mode)
                or self.dispatch_backend != "sparse" or getattr(x, "_sf_event_masks", None) is not None):
            return None
        key = (x.shape, x.dtype, x.get_device(), self.allow_sparse_1x1)
        c = self._fast
        if c is None or c[0] != key:
            c = self._plain_setup(x, key)
            self._fast = c
        if c[1] is None or not x.is_contiguous():
            return None
        _, fn, _desc, dref, nbytes, out_shape, idx = c
        w = self.weight
        if self._w_packed is None or self._w_packed_key != (w._version, w.data_ptr()):
            self._get_w_packed()
        b = self.bias
        bp = None
        if b is not None:
            bkey = (b._version, b.data_ptr())
            if self._bias_key != bkey:
                self._bias32 = b.detach().to(torch.float32).contiguous()
                self._bias_key = bkey
            bp = self._bias32.data_ptr()
        st = _lib.raw_stream(idx)
        ws = _lib.workspace_on(idx, st, nbytes)
        y = torch.empty(out_shape, dtype=x.dtype, device=x.device)
        status = fn(x.data_ptr(), self._w_packed.data_ptr(), bp, y.data_ptr(), dref, ws.data_ptr(), ws.numel(), st)
        if status != 0:
            _lib._check("sf_sparse_conv2d", status)
        self.fallback_reason = ""
        self._last_used_event_masks = False
        self._last_sparse_ms = 0.0
        self._last_dense_ms = 0.0
        return y

    def _plain_setup(self, x, key):
        none = (key, None, None, None, None, None, None)
        if not x.is_cuda or x.dim() not in (4, 5) or x.dtype not in (torch.float32, torch.float16, torch.bfloat16) \
                or not self._supports_sparse():
            return none
        if x.dim() == 5:
            t, bsz, c, h, w = x.shape
            n = t * bsz
        else:
            n, c, h, w = x.shape
        ho, wo = self._output_hw(h, w)
        wp = self._get_w_packed()
        desc = _lib.ConvDesc(n, c, h, w, self.out_channels, ho, wo, self.kernel_size[0], self.stride[0],
                             self.padding[0], _lib.sf_dtype(x.dtype), _lib.sf_dtype(wp.dtype),
                             int(self.bias is not None))
        lib = _lib.load()
        nbytes = int(lib.sf_sparse_conv2d_workspace_size(ctypes.byref(desc)))
        out_shape = (t, bsz, self.out_channels, ho, wo) if x.dim() == 5 else (n, self.out_channels, ho, wo)
        return (key, lib.sf_sparse_conv2d, desc, ctypes.byref(desc), nbytes, out_shape, x.get_device())

    def _sparse_forward(self, x4, event_masks=None):
        diag = self.collect_diag and not self._inference_mode
        kw = {}
        if event_masks is not None and not diag:
            kw["event_masks"] = event_masks
        if diag:
            self._ensure_buffers(x4)
            kw = dict(ag_mask_buf=self._ag_mask_buf, tile_class_buf=self._tile_class_buf,
                      return_avg_active_ratio=True, return_tile_stats=True)
        res = sparse_conv2d_forward(
            x4, self.weight, self.bias, kernel_size=self.kernel_size[0], stride=self.stride[0],
            padding=self.padding[0], dilation=self.dilation[0], groups=self.groups, threshold=self.threshold,
            w_cl=self._get_w_packed(), return_ms=self.return_ms, return_backend_meta=True,
            launch_all_tiles=self.launch_all_tiles, output_dtype=x4.dtype, **kw)
        y, ms = res[0], res[1]
        meta = res[-1]
        self._last_used_event_masks = bool(meta.get("event_masks", False))
        self._last_sparse_ms = float(ms)
        self._last_dense_ms = 0.0
        if diag:
            ratio, stats = res[2], res[3]
            self._last_avg_active_ratio = ratio
            gs = choose_group_size(self.in_channels)
            zt = stats["zero_tiles"]
            n_tiles = stats["total_tiles"]
            self._last_diag = {
                "sparse_path_executed": True,
                "metadata_kind": "b200_single_pass",
                "group_size": gs, "num_groups": -(-self.in_channels // gs),
                "active_group_ratio": ratio, "effective_k_ratio": ratio,
                "tile_zero_count": zt, "total_tile_count": n_tiles,
                "tile_zero_ratio": zt / max(n_tiles, 1),
                "zero_tiles": zt, "sparse_tiles": stats["sparse_tiles"], "denseish_tiles": stats["denseish_tiles"],
                "active_tiles": stats["active_tiles"],
                "sparse_compute_ms": float(ms), "sparse_total_ms": float(ms),
                "backend": meta.get("backend"), "backend_reason": meta.get("reason"),
                "kernel_type": f"{self.kernel_size[0]}x{self.kernel_size[0]}/s{self.stride[0]}",
                "backend_family": self.backend_family, "diag_path": self.diag_path,
                "fallback_reason": self.fallback_reason,
            }
        return y, meta.get("backend", "sparse_b200")

    def extra_repr(self):
        bs = self.block_size if self.block_size is not None else "auto"
        return (f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, "
                f"stride={self.stride}, padding={self.padding}, block_size={bs}, "
                f"return_ms={self.return_ms}, sparse=True, backend=b200_gather, "
                f"allow_sparse_1x1={self.allow_sparse_1x1}, inference_mode={self._inference_mode}")


__all__ = ["SparseConv2d", "TILE_ZERO", "TILE_SPARSE", "TILE_DENSEISH"]
