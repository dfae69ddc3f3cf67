"""Generate golden vectors from the reference implementation itself.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/SparseFlow

It imports the reference read-only and records, for seeded inputs:
  * prescan.npz -- ``Kernels._prescan_common._build_rf_prescan_metadata_impl``
    outputs (ag_mask, tile_class) and the active tile ids of
    ``Kernels.conv2d._build_active_tile_ids``, on the reference's fp16 NHWC
    input, for both tile geometries (the kernel's 8x8/8x16 tiles and square
    block_selector blocks), strides 1 and 2, ragged shapes, threshold edge
    values and NaN;
  * conv.npz -- ``Ops.sparse_conv2d.SparseConv2d.from_dense(conv, block)`` on
    CPU tensors (its F.conv2d path), 4-D and 5-D inputs;
  * lif.npz -- ``Ops.sparse_fused_conv_lif.FusedSparseConvLIF`` on CPU tensors
    (its LIF fallback) over T steps, hard and soft reset, decay_input on/off.

The reference's LIF module subclasses spikingjelly's ``MemoryModule``;
spikingjelly is not installed here, so a minimal stand-in providing only the
names it needs (``MemoryModule.register_memory``, ``neuron.LIFNode``,
``functional.reset_net``) is registered in ``sys.modules`` first. It contains
no spikingjelly code.

The fixtures are small (each a few hundred KB at most) and committed; the
tests never need the reference checkout.
"""
from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

OUT = Path(__file__).resolve().parent


def _install_spikingjelly_standin() -> None:
    if "spikingjelly" in sys.modules:
        return

    class MemoryModule(nn.Module):
        def __init__(self):
            super().__init__()
            self._memories = {}

        def register_memory(self, name, value):
            self._memories[name] = value
            setattr(self, name, value)

        def reset(self):
            for k, v in self._memories.items():
                setattr(self, k, v)

    class LIFNode(nn.Module):
        def __init__(self, tau=2.0, v_threshold=1.0, v_reset=0.0, decay_input=True, detach_reset=False):
            super().__init__()
            self.tau, self.v_threshold, self.v_reset = tau, v_threshold, v_reset
            self.decay_input, self.detach_reset = decay_input, detach_reset

    root = types.ModuleType("spikingjelly")
    ab = types.ModuleType("spikingjelly.activation_based")
    base = types.ModuleType("spikingjelly.activation_based.base")
    neuron = types.ModuleType("spikingjelly.activation_based.neuron")
    functional = types.ModuleType("spikingjelly.activation_based.functional")
    base.MemoryModule = MemoryModule
    neuron.LIFNode = LIFNode
    neuron.IFNode = type("IFNode", (LIFNode,), {})
    neuron.ParametricLIFNode = type("ParametricLIFNode", (LIFNode,), {})
    functional.reset_net = lambda m: [x.reset() for x in m.modules() if hasattr(x, "reset")]
    ab.base, ab.neuron, ab.functional = base, neuron, functional
    root.activation_based = ab
    for name, mod in [("spikingjelly", root), ("spikingjelly.activation_based", ab),
                      ("spikingjelly.activation_based.base", base),
                      ("spikingjelly.activation_based.neuron", neuron),
                      ("spikingjelly.activation_based.functional", functional)]:
        sys.modules[name] = mod


def _bernoulli(g, shape, p):
    return (torch.rand(shape, generator=g) < p).float()


def _clustered(g, shape, block, p_block, p_in):
    """Block-clustered spikes: independent block x block masks per (n, c) plane (ceil tiling)."""
    n, c, h, w = shape
    bh, bw = -(-h // block), -(-w // block)
    blk = (torch.rand(n, c, bh, bw, generator=g) < p_block).float()
    mask = blk.repeat_interleave(block, 2).repeat_interleave(block, 3)[:, :, :h, :w]
    return mask * _bernoulli(g, shape, p_in)


def prescan_cases(g):
    from Kernels._prescan_common import _build_rf_prescan_metadata_impl
    from Kernels.conv2d import _build_active_tile_ids, _select_tile_sizes, choose_group_size

    cases = []
    # (name, x NCHW float32, k, s, p, block or None for the kernel's own tile)
    cases.append(("c1_p02", _bernoulli(g, (4, 64, 32, 32), 0.02), 3, 1, 1, None))
    cases.append(("c1_p002", _bernoulli(g, (4, 64, 32, 32), 0.002), 3, 1, 1, None))
    cases.append(("c1_block16", _bernoulli(g, (4, 64, 32, 32), 0.0005), 3, 1, 1, 16))
    cases.append(("ragged_c40", _bernoulli(g, (3, 40, 13, 30), 0.003), 3, 1, 1, None))
    cases.append(("s2_c48", _bernoulli(g, (2, 48, 17, 17), 0.004), 3, 2, 1, None))
    cases.append(("s2_block4", _bernoulli(g, (2, 48, 17, 17), 0.004), 3, 2, 1, 4))
    cases.append(("c2_1x1_clustered", _clustered(g, (2, 256, 56, 56), 16, 0.05, 0.3), 1, 1, 0, None))
    cases.append(("c512_1x1", _bernoulli(g, (2, 512, 14, 14), 0.0008), 1, 1, 0, None))
    cases.append(("c1100_3x3", _bernoulli(g, (1, 1100, 9, 9), 0.0003), 3, 1, 1, None))
    cases.append(("h7_block8", _bernoulli(g, (2, 64, 7, 7), 0.01), 3, 1, 1, 8))
    cases.append(("empty", torch.zeros(2, 32, 16, 16), 3, 1, 1, None))
    cases.append(("dense_vals", torch.randn(2, 16, 12, 20, generator=g), 3, 1, 1, None))
    # Threshold edge values (half ulps around 1e-6), negatives, overflow to inf, NaN.
    edge = torch.zeros(2, 32, 24, 24)
    vals = [16 * 2.0 ** -24, 17 * 2.0 ** -24, 18 * 2.0 ** -24, 1.0e-6, 1.03e-6, -1.1e-6, 1e-7, 7.0e4, -3.0]
    flat = edge.view(-1)
    idx = torch.randperm(flat.numel(), generator=g)[: 3 * len(vals)]
    for j, i in enumerate(idx.tolist()):
        flat[i] = vals[j % len(vals)]
    cases.append(("threshold_edges", edge.clone(), 3, 1, 1, None))
    nan_x = edge.clone()
    nan_x.view(-1)[idx[:4]] = float("nan")
    cases.append(("nan_poison", nan_x, 3, 1, 1, None))

    out = {}
    for name, x, k, s, p, block in cases:
        n, c, h, w = x.shape
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        bh, bw = (block, block) if block else _select_tile_sizes(ho, wo)
        gs = choose_group_size(c)
        ng = -(-c // gs)
        x16 = x.half()
        tc, ag, _ = _build_rf_prescan_metadata_impl(
            x16.permute(0, 2, 3, 1), (ho, wo), (k, k), s, p, (bh, bw), gs, ng, 1e-6)
        ids, cnt = _build_active_tile_ids(tc, tc.numel())
        out[f"{name}__x"] = x.numpy()
        out[f"{name}__geom"] = np.array([k, s, p, bh, bw, gs, ho, wo], np.int32)
        out[f"{name}__ag_mask"] = ag.numpy().astype(np.int32)
        out[f"{name}__tile_class"] = tc.numpy().astype(np.int32)
        out[f"{name}__active_ids"] = ids.numpy().astype(np.int32)[:cnt]
    return out


def conv_cases(g):
    from Ops.sparse_conv2d import SparseConv2d

    specs = [
        # name, x shape (5-D T,N,C,H,W or 4-D), p, cout, k, s, pad, bias, weight kind, block
        ("c1_small", (2, 2, 64, 32, 32), 0.02, 64, 3, 1, 1, True, "kaiming", 16),
        ("s2", (3, 32, 15, 15), 0.05, 64, 3, 2, 1, True, "kaiming", 4),
        ("ragged", (2, 40, 9, 13), 0.1, 24, 3, 1, 1, False, "kaiming", 4),
        ("c2_1x1_bf16w", (2, 2, 256, 14, 14), 0.02, 64, 1, 1, 0, False, "bf16", 4),
        ("values", (2, 16, 12, 12), 0.3, 32, 3, 1, 1, True, "kaiming", 4),
    ]
    out = {}
    for name, shape, p, co, k, s, pad, bias, wkind, block in specs:
        c = shape[-3]
        conv = nn.Conv2d(c, co, k, s, pad, bias=bias)
        if wkind == "bf16":
            w = (torch.randn(co, c, k, k, generator=g) * 0.02).bfloat16().float()
        else:
            w = torch.empty(co, c, k, k)
            nn.init.kaiming_normal_(w, mode="fan_out", nonlinearity="relu", generator=g)
        conv.weight.data.copy_(w)
        if bias:
            conv.bias.data.copy_(torch.randn(co, generator=g) * 0.1)
        x = _bernoulli(g, shape, p)
        if name == "values":
            x = x * torch.randn(shape, generator=g)
        sp = SparseConv2d.from_dense(conv, block_size=block)
        with torch.no_grad():
            y = sp(x)
        out[f"{name}__x"] = x.numpy()
        out[f"{name}__w"] = conv.weight.detach().numpy()
        if bias:
            out[f"{name}__b"] = conv.bias.detach().numpy()
        out[f"{name}__geom"] = np.array([k, s, pad], np.int32)
        out[f"{name}__y"] = y.numpy()
    return out


def lif_cases(g):
    _install_spikingjelly_standin()
    from Ops.sparse_fused_conv_lif import FusedSparseConvLIF

    specs = [
        # name, T, N, C, Co, H, p, bias, v_reset, decay_input, tau, vth
        ("hard_decay", 4, 2, 32, 32, 12, 0.05, True, 0.0, True, 2.0, 1.0),
        ("soft_decay", 4, 2, 32, 32, 12, 0.05, True, None, True, 2.0, 0.5),
        ("hard_nodecay", 3, 2, 16, 32, 10, 0.1, False, 0.0, False, 3.0, 0.7),
    ]
    out = {}
    for name, T, N, C, Co, H, p, bias, v_reset, decay, tau, vth in specs:
        conv = nn.Conv2d(C, Co, 3, 1, 1, bias=bias)
        w = torch.empty(Co, C, 3, 3)
        nn.init.kaiming_normal_(w, mode="fan_out", nonlinearity="relu", generator=g)
        conv.weight.data.copy_(w * 2.0)
        if bias:
            conv.bias.data.copy_(torch.randn(Co, generator=g) * 0.2)
        lif = types.SimpleNamespace(tau=tau, v_threshold=vth, v_reset=v_reset, decay_input=decay,
                                    detach_reset=False, backend="torch")
        mod = FusedSparseConvLIF.from_conv_and_lif(conv, lif)
        x = _bernoulli(g, (T, N, C, H, H), p)
        with torch.no_grad():
            spikes = mod(x)
        out[f"{name}__x"] = x.numpy()
        out[f"{name}__w"] = conv.weight.detach().numpy()
        if bias:
            out[f"{name}__b"] = conv.bias.detach().numpy()
        out[f"{name}__params"] = np.array([tau, vth, 0.0 if v_reset is None else v_reset,
                                           float(v_reset is not None), float(decay)], np.float32)
        out[f"{name}__spikes"] = spikes.numpy()
        out[f"{name}__v"] = mod.v.numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the SparseFlow checkout to import")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    torch.manual_seed(0)
    g = torch.Generator().manual_seed(20261201)
    np.savez_compressed(OUT / "prescan.npz", **prescan_cases(g))
    np.savez_compressed(OUT / "conv.npz", **conv_cases(g))
    np.savez_compressed(OUT / "lif.npz", **lif_cases(g))
    for f in ("prescan.npz", "conv.npz", "lif.npz"):
        print(f, (OUT / f).stat().st_size)


if __name__ == "__main__":
    main()
