"""Benchmark of the spike-sparse conv path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (one line of JSON on rank 0): the reference's headline
layer shape, a SparseConv2d 3x3/s1/p1 64->64 on a 5-D spike tensor
T=16, N=64, 56x56, Bernoulli(0.01) fp32 spikes (99% sparsity), kaiming-normal
fp32 weights + bias -- BASELINE.json's sweep cell (C=64, H=56, density 0.01,
block 16 per the H->block rule), i.e. layer1.x.conv2 of Spiking-ResNet50.
A step is one ``SparseConv2d.forward`` over the whole batch.

* ``value``: GB/s of algorithmic traffic (x read + y written + weights + bias,
  once each) over the timed device time, inputs resident in HBM; x and y are
  822 MB each, larger than L2, so no flush is needed between steps.
* ``e2e``: the same metric through the public module call with all of a
  step's spikes copied from pinned host memory and all of its output copied
  back, every step; the batch runs in chunks so uploads, convolutions and
  downloads of neighbouring chunks overlap (three streams, full-duplex PCIe).
* ``roofline``: the sparse-conv kernel against the measured HBM copy peak.
* ``cpu_baseline``: the reference's CPU path (F.conv2d, all host threads) on
  a bounded sample of the same workload.
* ``extra``: the other hot-path kernels on their BASELINE.json configs
  (prescan GB/s on the same input; C2 1x1 with bf16 weights; C3 fused
  conv+BN+LIF over T=16) and cuDNN dense time for the speedup figures.

Multi-GPU (torchrun): every rank runs the same per-GPU workload on its own
shard of the batch (weak scaling, no collective in the data path); the
timed region is bracketed by barriers and the max over ranks is reported.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.nn as nn  # noqa: E402

T_STEPS, N_BATCH, C, H, W = 16, 64, 64, 56, 56
DENSITY = 0.01
E2E_CHUNKS = 8  # pipeline depth of the end-to-end measurement
METRIC = "sparse conv3x3 GB/s (layer1.x.conv2 shape, 99% spike sparsity)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extra", action="store_true", help="skip the C2/C3/prescan side measurements")
    ap.add_argument("--only-timed", action="store_true",
                    help="run only the warm-up and timed steps (no cuDNN, e2e, extras or CPU baseline); for ncu")
    ap.add_argument("--kernel", choices=["conv", "prescan", "c2", "c2masks", "c3", "lif", "lif_events", "c4"],
                    default="conv",
                    help="with --only-timed: time the sparse conv (default), the prescan on the same input, "
                         "the C2 1x1 cell (--images = T*N of C2, default 512; c2masks: fed by the producer's "
                         "event masks), the C3 fused conv+LIF or the "
                         "standalone LIF, without or with the event masks (--images = T*N, default 1024), or "
                         "the C4 Spiking-ResNet50 forward after optimize()")
    ap.add_argument("--sweep", action="store_true",
                    help="C5 grid: C x H x density, sparse conv3x3 vs cuDNN and the HBM roofline (one JSON line per cell)")
    ap.add_argument("--sweep-images", type=int, default=T_STEPS * N_BATCH,
                    help="T*N images per sweep cell (BASELINE: T16 N64 = 1024)")
    ap.add_argument("--cell", default=None,
                    help="with --only-timed --kernel conv: 'C,H,density' times that C5 grid cell (C->C 3x3/s1/p1, "
                         "HxH maps, Bernoulli spikes) instead of the headline cell; an ncu-sized case with --images")
    ap.add_argument("--images", type=int, default=T_STEPS * N_BATCH,
                    help="T*N images per step (multiple of 16); smaller values make an ncu-sized case")
    ap.add_argument("--path3x3", type=int, choices=[0, 1, 2], default=0,
                    help="with --only-timed: SF_POLICY_CONV3X3_PATH (0 the density gate, 1 gather kernel, "
                         "2 tensor cores), to profile one route of a gated cell")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


def conv_bytes(n_img, c, h, w, co, ho, wo, k, esz=4, wsz=4, bias=True):
    return esz * n_img * c * h * w + esz * n_img * co * ho * wo + wsz * co * c * k * k + (4 * co if bias else 0)


def make_conv(c, co, k, s, p, bias, seed, wdtype=torch.float32, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    conv = nn.Conv2d(c, co, k, s, p, bias=bias)
    w = torch.empty(co, c, k, k)
    nn.init.kaiming_normal_(w, mode="fan_out", nonlinearity="relu", generator=g)
    conv.weight.data.copy_(w)
    if bias:
        conv.bias.data.copy_(torch.randn(co, generator=g) * 0.1)
    conv = conv.to(device)
    if wdtype != torch.float32:
        conv = conv.to(wdtype)
    return conv


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML every 5 ms while the GPU works
    (reading only; nothing is set)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self.thread = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 -- no NVML: the line reports clocks as null
            return

        def run():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    util = pynvml.nvmlDeviceGetUtilizationRates(h).gpu
                    self.samples.append((float(mhz), int(reasons), int(util)))
                except Exception:  # noqa: BLE001
                    pass
                time.sleep(0.005)
        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()

    def stop(self):
        if self.thread is None:
            return None
        self._stop.set()
        self.thread.join(timeout=2)
        if not self.samples:
            return None
        busy = [smp for smp in self.samples if smp[2] > 0] or self.samples
        reasons = sorted(nm for nm, bit in self.REASONS.items() if any(smp[1] & bit for smp in busy))
        return {"sm_mhz": statistics.median(smp[0] for smp in busy), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(busy), "source": "NVML, 5 ms"}


def cuda_time(fn, steps, warmup, dist=None):
    """Device time of `steps` calls of fn, CUDA events on the current stream, max over ranks."""
    for _ in range(warmup):
        fn()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = s.elapsed_time(e)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def time_reference_cpu(steps, warmup, n_img=T_STEPS * N_BATCH):
    """The reference's own CPU path for this layer (SparseConv2d on a CPU tensor = F.conv2d,
    Ops/sparse_conv2d.py:819-834) on the headline workload (same shapes, density, weight init),
    all host threads. Returns (GB/s, threads, seconds per step, steps)."""
    from oracle import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    conv = make_conv(C, C, 3, 1, 1, True, 1, device="cpu")
    x = (torch.rand(n_img, C, H, W, generator=g) < DENSITY).float()
    nbytes = conv_bytes(n_img, C, H, W, C, H, W, 3)
    with torch.no_grad():
        for _ in range(max(1, warmup)):
            oracle.reference_cpu_conv2d(x, conv.weight, conv.bias, 1, 1)
        t0 = time.perf_counter()
        for _ in range(steps):
            oracle.reference_cpu_conv2d(x, conv.weight, conv.bias, 1, 1)
        sec = (time.perf_counter() - t0) / steps
    return nbytes / sec / 1e9, threads, sec, steps


def run_reference(args):
    """--impl reference: rank 0 times the reference's CPU path on the full per-GPU workload; under
    torchrun the other ranks wait at a gloo barrier (idle, not competing for the host cores) and exit."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    pg = None
    if world > 1:
        import torch.distributed as tdist
        tdist.init_process_group("gloo")
        pg = tdist
        pg.barrier()  # every rank has started (imports done) before rank 0 times
    if rank == 0:
        steps = max(1, min(args.steps, 20))
        val, cores, sec, steps = time_reference_cpu(steps, min(args.warmup, 3))
        sample = (f"the full step: {T_STEPS * N_BATCH} images (T*N) of C64 56x56, same shapes/density/weight init; "
                  "torch F.conv2d = the reference SparseConv2d CPU path (Ops/sparse_conv2d.py:819-834)")
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C5 cell: SparseConv2d 3x3/s1/p1 C64->64, T16 N64 56x56, Bernoulli(0.01) fp32 "
                                   "spikes, block 16 (per GPU)", "sample": sample,
                       "note": "one host CPU for all N: the reference's CPU path does not shard across GPUs"},
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def masks_of(x4):
    """Event masks of a binary NCHW tensor in the layout a spike producer writes:
    [n][h][w][ceil(C/64)] 64-bit words, bit c % 64 of word c // 64 set iff channel c is nonzero."""
    n, c, h, w = x4.shape
    nw = (c + 63) // 64
    pad = torch.zeros(n, nw * 64, h, w, dtype=torch.bool, device=x4.device)
    pad[:, :c] = x4 != 0
    out = torch.zeros(n, h, w, nw, dtype=torch.int64, device=x4.device)
    for b in range(64):
        out |= pad[:, b::64].permute(0, 2, 3, 1).to(torch.int64) << b
    return out.contiguous()


def extras(dev, hbm_peak, steps):
    """Side measurements: prescan GB/s, C2 1x1 bf16, C3 fused conv+BN+LIF, cuDNN comparisons."""
    from sparseflow_b200.Kernels._prescan_common import prescan2d
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    from sparseflow_b200.Ops.sparse_fused_conv_lif import FusedSparseConvLIF
    from sparseflow_b200.Ops.lif_node import LIFNode
    out = {}
    steps = max(3, min(steps, 50))
    g = torch.Generator(device=dev).manual_seed(17)

    # Prescan on the headline input (fp32 NCHW, 3x3 RF, 8x16 tiles, gs 16).
    x = (torch.rand(T_STEPS * N_BATCH, C, H, W, device=dev, generator=g) < DENSITY).float()
    nt = T_STEPS * N_BATCH * 7 * 4
    ag = torch.empty(nt, dtype=torch.int32, device=dev)
    tc = torch.empty_like(ag)
    ids = torch.empty_like(ag)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    fn = lambda: prescan2d(x, 0, (H, W), (3, 3), 1, 1, (8, 16), 16, 1e-6, ag, tc, ids, cnt)  # noqa: E731
    ms = cuda_time(fn, steps, 3) / steps
    pb = x.numel() * 4 + nt * 12
    out["prescan_c5"] = {"GBps": round(pb / ms / 1e6, 1), "frac_of_measured_hbm": round(pb / ms / 1e6 / hbm_peak, 3),
                         "ms": round(ms, 4), "bytes": pb}
    del x

    # The headline layer with bf16 activations in and out (spikes are exact in bf16; fp32 weights,
    # fp32 accumulation; outputs rounded to bf16): half the bytes of the fp32 cell, against cuDNN
    # on the same bf16 tensors.
    xb = (torch.rand(T_STEPS * N_BATCH, C, H, W, device=dev, generator=g) < DENSITY).to(torch.bfloat16)
    convb = make_conv(C, C, 3, 1, 1, True, 1, device=dev)
    mb = SparseConv2d.from_dense(convb, block_size=16)
    mb.set_inference_mode(True)
    ms_b = cuda_time(lambda: mb(xb), steps, 3) / steps
    wb, bb = convb.weight.to(torch.bfloat16), convb.bias.to(torch.bfloat16)
    cud_b = cuda_time(lambda: torch.nn.functional.conv2d(xb, wb, bb, 1, 1), steps, 3) / steps
    bytes_b = conv_bytes(T_STEPS * N_BATCH, C, H, W, C, H, W, 3, esz=2)
    out["c5_bf16_io"] = {"ms": round(ms_b, 4), "GBps": round(bytes_b / ms_b / 1e6, 1),
                         "frac_of_measured_hbm": round(bytes_b / ms_b / 1e6 / hbm_peak, 3),
                         "cudnn_bf16_ms": round(cud_b, 4), "speedup_vs_cudnn_bf16": round(cud_b / ms_b, 2)}
    del xb

    # C2: 1x1 256->64, T16 N32 56x56 block-clustered spikes, bf16 weights.
    n2 = 16 * 32
    blk = (torch.rand(n2, 256, 4, 4, device=dev, generator=g) < 0.05).float()
    mask = blk.repeat_interleave(16, 2).repeat_interleave(16, 3)[:, :, :56, :56]
    x2 = (mask * (torch.rand(n2, 256, 56, 56, device=dev, generator=g) < 0.3).float()).reshape(16, 32, 256, 56, 56)
    del blk, mask
    conv2 = nn.Conv2d(256, 64, 1, bias=False)
    conv2.weight.data = (torch.randn(64, 256, 1, 1, generator=torch.Generator().manual_seed(2)) * 0.02)
    conv2 = conv2.to(dev).to(torch.bfloat16)
    m2 = SparseConv2d.from_dense(conv2, block_size=16)
    m2.set_inference_mode(True)
    ms = cuda_time(lambda: m2(x2), steps, 3) / steps
    b2 = conv_bytes(n2, 256, 56, 56, 64, 56, 56, 1, wsz=2, bias=False)
    x2f = x2.reshape(n2, 256, 56, 56)
    wf = conv2.weight.float()
    cud = cuda_time(lambda: torch.nn.functional.conv2d(x2f, wf), steps, 3) / steps
    out["c2_conv1x1_bf16w"] = {"GBps": round(b2 / ms / 1e6, 1), "frac_of_measured_hbm": round(b2 / ms / 1e6 / hbm_peak, 3),
                               "ms": round(ms, 4), "cudnn_ms": round(cud, 4), "speedup_vs_cudnn": round(cud / ms, 2),
                               "density": round(float((x2 != 0).float().mean()), 5)}
    # The same layer as it runs inside a network: its input spikes come from a LIF node that hands
    # over their event masks (LIFNode.emit_event_masks), so the tcgen05 kernel builds its A operand
    # from the masks (32 bytes per pixel) instead of reading 1 KB of fp32 spikes. The masks are
    # built here, outside the timed region, as that producer would have written them.
    from sparseflow_b200 import _lib
    m2 = masks_of(x2f)
    y2 = torch.empty(n2, 64, 56, 56, device=dev)
    wp2 = _lib.pack_weights(conv2.weight, torch.bfloat16)
    msk = cuda_time(lambda: _lib.sparse_conv2d_from_masks(m2, tuple(x2f.shape), x2f.dtype, wp2, None, y2, 1, 1, 0),
                    steps, 3) / steps
    ref2 = torch.nn.functional.conv2d(x2f, wf)
    bm = m2.numel() * 8 + n2 * 64 * 56 * 56 * 4 + 64 * 256 * 2
    out["c2_conv1x1_bf16w_from_producer_masks"] = {
        "ms": round(msk, 4), "cudnn_ms": round(cud, 4), "speedup_vs_cudnn": round(cud / msk, 2),
        "GBps": round(bm / msk / 1e6, 1), "frac_of_measured_hbm": round(bm / msk / 1e6 / hbm_peak, 3),
        "bytes": bm, "max_rel_err_vs_cudnn_fp32": float((y2 - ref2).abs().max() / ref2.abs().max())}
    del m2, y2, ref2
    del x2, x2f

    # C3: fused conv3x3 + BN-fold + LIF, T16 N64 C128 28x28, Bernoulli(0.005).
    x3 = (torch.rand(16, 64, 128, 28, 28, device=dev, generator=g) < 0.005).float()
    conv3 = make_conv(128, 128, 3, 1, 1, False, 3, device=dev)
    bn = nn.BatchNorm2d(128).to(dev).eval()
    gg = torch.Generator(device=dev).manual_seed(4)
    bn.weight.data = torch.rand(128, device=dev, generator=gg) + 0.5
    bn.bias.data = torch.randn(128, device=dev, generator=gg) * 0.1
    bn.running_mean = torch.randn(128, device=dev, generator=gg) * 0.1
    bn.running_var = torch.rand(128, device=dev, generator=gg) + 0.5
    m3 = FusedSparseConvLIF.from_conv_bn_lif(conv3, bn, LIFNode(tau=2.0, v_threshold=1.0, v_reset=0.0))

    def c3_step():
        m3.reset()
        return m3(x3)
    ms = cuda_time(c3_step, steps, 3) / steps
    b3 = 4 * x3.numel() * 2 + 4 * 64 * 128 * 28 * 28 * 2 + 4 * 128 * 128 * 9

    # What the reference runs for this layer on a GPU without its (dead) fused kernel:
    # cuDNN conv over all T*N images, eval BN, then the LIF formula step by step in torch.
    lif_ref = LIFNode(tau=2.0, v_threshold=1.0, v_reset=0.0)

    def c3_torch():
        y = bn(torch.nn.functional.conv2d(x3.flatten(0, 1), conv3.weight, None, 1, 1)).reshape(16, 64, 128, 28, 28)
        lif_ref.reset()
        return torch.stack([lif_ref._step(y[t]) for t in range(16)], 0)
    ms_ref = cuda_time(c3_torch, max(3, steps // 5), 2) / max(3, steps // 5)
    out["c3_fused_conv_bn_lif"] = {"GBps": round(b3 / ms / 1e6, 1), "frac_of_measured_hbm": round(b3 / ms / 1e6 / hbm_peak, 3),
                                   "ms": round(ms, 4), "cudnn_conv_bn_torch_lif_ms": round(ms_ref, 4),
                                   "speedup_vs_cudnn_path": round(ms_ref / ms, 2)}
    # The same layer at higher firing rates, where the density gate sends it to the tensor-core
    # route (conv into the spike buffer, LIF in place); the cuDNN path does not depend on density.
    by_density = {}
    for dd in (0.02, 0.1):
        x3 = (torch.rand(16, 64, 128, 28, 28, device=dev, generator=g) < dd).float()
        by_density[str(dd)] = {"ms": round(cuda_time(c3_step, steps, 3) / steps, 4)}
        by_density[str(dd)]["speedup_vs_cudnn_path"] = round(ms_ref / by_density[str(dd)]["ms"], 2)
    out["c3_fused_conv_bn_lif"]["by_density"] = by_density
    del x3
    # LIF -> SparseConv2d on the headline layer shape (T16 N64 C64 56x56, ~1 % spikes): the LIF
    # writing the next convolution's event masks (LIFNode.emit_event_masks) against the plain
    # LIF followed by the convolution's own mask pass over the spikes.
    xl = torch.randn(T_STEPS, N_BATCH, C, H, W, device=dev, generator=g) * 0.8
    convl = make_conv(C, C, 3, 1, 1, True, 5, device=dev)
    scl = SparseConv2d.from_dense(convl, block_size=16)
    scl.set_inference_mode(True)
    chain = {}
    for emit in (False, True):
        lifl = LIFNode(tau=2.0, v_threshold=1.0, v_reset=0.0)
        lifl.emit_event_masks = emit

        def lif_conv():
            lifl.reset()
            return scl(lifl(xl))
        chain["emit_ms" if emit else "plain_ms"] = round(cuda_time(lif_conv, steps, 3) / steps, 4)
    lifl.reset()
    chain["spike_density"] = round(float(lifl(xl).float().mean()), 4)
    chain["speedup"] = round(chain["plain_ms"] / chain["emit_ms"], 3)
    chain["note"] = ("the C64 3x3 convolution runs on the tensor cores from the spikes and ignores the masks, "
                     "so optimize() leaves emission off for such layers; this times the emission cost alone")
    out["lif_events_to_conv"] = chain
    del xl
    out["c1_conv3x3_small"] = c1_small(dev, hbm_peak, steps)
    out["c4_spiking_resnet50"] = c4_resnet(dev)
    return out


def c1_small(dev, hbm_peak, steps, sets=8):
    """C1: SparseConv2d 3x3/s1/p1 64->64 with bias on [T=4, N=8, 64, 32, 32]
    Bernoulli(0.02) fp32 spikes, kaiming weights, block 16. One call is 16.9 MB, so `sets` input /
    output pairs (135 MB, larger than L2) rotate between calls; cuDNN on the same rotation; the
    reference CPU path (F.conv2d, all host threads) on the full C1 step."""
    from oracle import oracle
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    g = torch.Generator(device=dev).manual_seed(41)
    conv = make_conv(64, 64, 3, 1, 1, True, 41, device=dev)
    mod = SparseConv2d.from_dense(conv, block_size=16)
    mod.set_inference_mode(True)
    xs = [(torch.rand(4, 8, 64, 32, 32, device=dev, generator=g) < 0.02).float() for _ in range(sets)]
    k = [0]

    def step():
        k[0] = (k[0] + 1) % sets
        return mod(xs[k[0]])
    n = max(steps, 50)
    ms = cuda_time(step, n, 5) / n
    x4 = [x.reshape(32, 64, 32, 32) for x in xs]

    def cudnn_step():
        k[0] = (k[0] + 1) % sets
        return torch.nn.functional.conv2d(x4[k[0]], conv.weight, conv.bias, 1, 1)
    cud = cuda_time(cudnn_step, n, 5) / n
    nbytes = conv_bytes(32, 64, 32, 32, 64, 32, 32, 3)

    def graph_ms(fn):
        # One graph holds a call on each of the rotating sets; replay time / sets = device time per
        # call with the host's per-call launch overhead removed (both arms alike).
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(sets):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(sets):
                fn()
        reps = max(5, n // sets)
        return cuda_time(graph.replay, reps, 2) / (reps * sets)
    with torch.no_grad():
        ms_g = graph_ms(step)
        cud_g = graph_ms(cudnn_step)
    conv_cpu = make_conv(64, 64, 3, 1, 1, True, 41, device="cpu")
    xc = xs[0].reshape(32, 64, 32, 32).cpu()
    torch.set_num_threads(os.cpu_count() or 1)
    with torch.no_grad():
        oracle.reference_cpu_conv2d(xc, conv_cpu.weight, conv_cpu.bias, 1, 1)
        t0 = time.perf_counter()
        for _ in range(20):
            oracle.reference_cpu_conv2d(xc, conv_cpu.weight, conv_cpu.bias, 1, 1)
        cpu_ms = (time.perf_counter() - t0) / 20 * 1e3
    return {"ms": round(ms, 4), "GBps": round(nbytes / ms / 1e6, 1),
            "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm_peak, 3), "cudnn_ms": round(cud, 4),
            "speedup_vs_cudnn": round(cud / ms, 2), "cpu_reference_ms": round(cpu_ms, 3),
            "speedup_vs_cpu_reference": round(cpu_ms / ms, 1), "bytes": nbytes,
            "ms_cuda_graph": round(ms_g, 4), "cudnn_ms_cuda_graph": round(cud_g, 4),
            "speedup_vs_cudnn_cuda_graph": round(cud_g / ms_g, 2),
            "GBps_cuda_graph": round(nbytes / ms_g / 1e6, 1),
            "note": f"{sets} rotating input/output sets (135 MB > L2); eager calls are bound by host launch "
                    "overhead at this size, the CUDA-graph figures by the device"}


def c4_resnet(dev, iters=3):
    """C4: Spiking-ResNet50 inference, T16 N128 3x32x32 N(0,1) direct-encoded, random init;
    the same model timed dense and after sparseflow_b200.optimize (img/s = N / s per forward)."""
    import copy
    import sparseflow_b200
    from sparseflow_b200.snn import spiking_resnet50
    from sparseflow_b200.Ops.lif_node import reset_net
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    torch.manual_seed(5)
    T, N = 16, 128
    dense = spiking_resnet50().to(dev).eval()
    img = torch.randn(N, 3, 32, 32, generator=torch.Generator().manual_seed(6)).to(dev)
    x = img.unsqueeze(0).repeat(T, 1, 1, 1, 1)
    sparse = copy.deepcopy(dense)
    sparseflow_b200.optimize(sparse, sample_input=x[:, :2], verbose=False)
    n_sparse = sum(isinstance(m, SparseConv2d) for m in sparse.modules())

    def run(model):
        reset_net(model)
        return model(x)
    res = {}
    with torch.no_grad():
        for name, model in (("dense", dense), ("sparse", sparse)):
            ms = cuda_time(lambda: run(model), iters, 2) / iters
            res[name] = ms
        # The same forwards replayed from CUDA graphs (one launch of the whole captured forward;
        # about 700 kernels per forward otherwise leave the step partly bound by host launches).
        for name, model in (("dense", dense), ("sparse", sparse)):
            try:
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    run(model)  # warm every lazily built buffer outside the capture
                torch.cuda.current_stream().wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    run(model)
                res[name + "_graph"] = cuda_time(graph.replay, iters, 2) / iters
            except Exception as e:  # noqa: BLE001 -- reported, never silently replaced
                res[name + "_graph_error"] = str(e)[:200]
        reset_net(dense)
        reset_net(sparse)
        ref = dense(x)
        reset_net(sparse)
        got = sparse(x)
        err = float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-12))
    return {"img_per_s_sparse": round(N / (res["sparse"] / 1e3), 1), "img_per_s_dense": round(N / (res["dense"] / 1e3), 1),
            "ms_sparse": round(res["sparse"], 2), "ms_dense": round(res["dense"], 2), "sparse_layers": n_sparse,
            "logits_rel_err_vs_dense": err,
            **{f"img_per_s_{k[:-6]}_cuda_graph": round(N / (v / 1e3), 1) for k, v in res.items()
               if k.endswith("_graph") and isinstance(v, float)},
            **{k: v for k, v in res.items() if k.endswith("_graph_error")},
            "note": "same random-init model and input; every LIF node is one launch of the multi-step LIF kernel (with event masks where it feeds a replaced convolution)"}


def c4_sharded(dev, dist, world, iters=5):
    """C4 N-sharded: every rank runs Spiking-ResNet50 (after optimize()) on its own 128 images,
    T16 3x32x32 N(0,1); img/s = 128 * world / (max over ranks of the device time per forward)."""
    import sparseflow_b200
    from sparseflow_b200.snn import spiking_resnet50
    from sparseflow_b200.Ops.lif_node import reset_net
    torch.manual_seed(5)
    model = spiking_resnet50().to(dev).eval()
    rank = dist.get_rank() if dist is not None else 0
    img = torch.randn(128, 3, 32, 32, generator=torch.Generator().manual_seed(6 + rank)).to(dev)
    x = img.unsqueeze(0).repeat(16, 1, 1, 1, 1)
    sparseflow_b200.optimize(model, sample_input=x[:, :2], verbose=False)

    def fwd():
        reset_net(model)
        return model(x)
    with torch.no_grad():
        ms = cuda_time(fwd, iters, 2, dist) / iters
    return {"img_per_s": round(128 * world / (ms / 1e3), 1), "ms_per_forward_max_over_ranks": round(ms, 3),
            "images_per_rank": 128, "ranks": world, "scaling": "weak", "eager": True}


def run_sweep(args):
    """C5: conv3x3/s1/p1 C->C over C in {64,128,256,512}, H=W in {14,28,56}, density in
    {0.001,0.01,0.05,0.2}; block size per the H->block rule (inert in the kernels). Bytes = x + y + w + b."""
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    from sparseflow_b200.Utils.block_selector import select_block_size
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm_peak, _, peak_kind = peaks()
    n_img = args.sweep_images
    for c in (64, 128, 256, 512):
        conv = make_conv(c, c, 3, 1, 1, True, c, device=dev)
        for h in (14, 28, 56):
            mod = SparseConv2d.from_dense(conv, block_size=select_block_size(h))
            mod.set_inference_mode(True)
            for dens in (0.001, 0.01, 0.05, 0.2):
                g = torch.Generator(device=dev).manual_seed(c * 1000 + h)
                x = (torch.rand(n_img, c, h, h, device=dev, generator=g) < dens).float()
                steps = 10
                with torch.no_grad():
                    ms = cuda_time(lambda: mod(x), steps, 3) / steps
                    cud = cuda_time(lambda: torch.nn.functional.conv2d(x, conv.weight, conv.bias, 1, 1), steps, 3) / steps
                nbytes = conv_bytes(n_img, c, h, h, c, h, h, 3)
                gbps = nbytes / ms / 1e6
                flops = 2.0 * n_img * c * c * 9 * h * h
                print(json.dumps({"cell": f"C{c}_H{h}_p{dens}", "c": c, "h": h, "density": dens, "images": n_img,
                                  "block": select_block_size(h), "ms": round(ms, 4), "cudnn_ms": round(cud, 4),
                                  "speedup_vs_cudnn": round(cud / ms, 2), "GBps": round(gbps, 1),
                                  "hbm_frac": round(gbps / hbm_peak, 3), "peak": f"{hbm_peak} GB/s ({peak_kind})",
                                  "hbm_floor_ms": round(nbytes / hbm_peak / 1e6, 4),
                                  "dense_equiv_tflops_cudnn": round(flops / cud / 1e9, 1)}), flush=True)
                del x


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.only_timed and args.path3x3:
        from sparseflow_b200 import _lib
        _lib.set_path_policy(_lib.SF_POLICY_CONV3X3_PATH, args.path3x3)
    if args.sweep:
        run_sweep(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as tdist
        tdist.init_process_group("nccl", device_id=dev)
        dist = tdist

    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d

    hbm_peak, _, peak_kind = peaks()
    n_img = args.images
    n_batch = n_img // T_STEPS
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    cc, hh, dd = C, H, DENSITY
    if args.cell:
        if not (args.only_timed and args.kernel == "conv"):
            raise SystemExit("--cell needs --only-timed --kernel conv")
        cc, hh, dd = int(args.cell.split(",")[0]), int(args.cell.split(",")[1]), float(args.cell.split(",")[2])
    x = (torch.rand(T_STEPS, n_batch, cc, hh, hh, device=dev, generator=g) < dd).float()
    conv = make_conv(cc, cc, 3, 1, 1, True, 1, device=dev)
    mod = SparseConv2d.from_dense(conv, block_size=16)
    mod.set_inference_mode(True)
    step_bytes = conv_bytes(n_img, cc, hh, hh, cc, hh, hh, 3)

    if args.only_timed and args.kernel in ("c2", "c2masks"):
        from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
        n2 = args.images if args.images != T_STEPS * N_BATCH else 512
        g2 = torch.Generator(device=dev).manual_seed(17 + rank)
        blk = (torch.rand(n2, 256, 4, 4, device=dev, generator=g2) < 0.05).float()
        mask = blk.repeat_interleave(16, 2).repeat_interleave(16, 3)[:, :, :56, :56]
        x2 = (mask * (torch.rand(n2, 256, 56, 56, device=dev, generator=g2) < 0.3).float()).contiguous()
        del blk, mask
        conv2 = nn.Conv2d(256, 64, 1, bias=False)
        conv2.weight.data = torch.randn(64, 256, 1, 1, generator=torch.Generator().manual_seed(2)) * 0.02
        m2 = SparseConv2d.from_dense(conv2.to(dev).to(torch.bfloat16), block_size=16)
        m2.set_inference_mode(True)
        with torch.no_grad():
            if args.kernel == "c2masks":
                from sparseflow_b200 import _lib
                m2m = masks_of(x2)
                y2 = torch.empty(n2, 64, 56, 56, device=dev)
                wp2 = _lib.pack_weights(conv2.weight, torch.bfloat16)
                ms = cuda_time(lambda: _lib.sparse_conv2d_from_masks(m2m, tuple(x2.shape), x2.dtype, wp2, None, y2,
                                                                     1, 1, 0), args.steps, args.warmup, dist) / args.steps
            else:
                ms = cuda_time(lambda: m2(x2), args.steps, args.warmup, dist) / args.steps
        b2 = conv_bytes(n2, 256, 56, 56, 64, 56, 56, 1, wsz=2, bias=False)
        if args.kernel == "c2masks":
            b2 = m2m.numel() * 8 + n2 * 64 * 56 * 56 * 4 + 64 * 256 * 2
        if rank == 0:
            print(json.dumps({"kernel": args.kernel, "ms_per_step": round(ms, 4), "GBps": round(b2 / ms / 1e6, 1),
                              "frac_of_measured_hbm": round(b2 / ms / 1e6 / hbm_peak, 3), "images": n2}))
        if dist is not None:
            dist.destroy_process_group()
        return

    if args.only_timed and args.kernel == "c4":
        # C4: one forward of the optimize()d Spiking-ResNet50 (T16 N128 3x32x32) per step.
        import sparseflow_b200
        from sparseflow_b200.snn import spiking_resnet50
        from sparseflow_b200.Ops.lif_node import reset_net
        torch.manual_seed(5)
        model = spiking_resnet50().to(dev).eval()
        img = torch.randn(128, 3, 32, 32, generator=torch.Generator().manual_seed(6)).to(dev)
        x = img.unsqueeze(0).repeat(16, 1, 1, 1, 1)
        sparseflow_b200.optimize(model, sample_input=x[:, :2], verbose=False)

        def fwd():
            reset_net(model)
            return model(x)
        with torch.no_grad():
            ms = cuda_time(fwd, args.steps, args.warmup, dist) / args.steps
        if rank == 0:
            print(json.dumps({"kernel": "c4", "ms_per_step": round(ms, 3), "img_per_s": round(128 / (ms / 1e3), 1)}))
        if dist is not None:
            dist.destroy_process_group()
        return

    if args.only_timed and args.kernel in ("c3", "lif", "lif_events"):
        # C3 fused conv3x3 + BN-fold + LIF (T16, C128 28x28, Bernoulli(0.005)
        # spikes), or the standalone multi-step LIF on the same shape with
        # real-valued input currents N(0,1). --images sets T*N (default 16*64).
        from sparseflow_b200.Ops.sparse_fused_conv_lif import FusedSparseConvLIF
        from sparseflow_b200.Ops.lif_node import LIFNode
        n3 = (args.images if args.images != T_STEPS * N_BATCH else 16 * 64) // 16
        g3 = torch.Generator(device=dev).manual_seed(23 + rank)
        if args.kernel == "c3":
            x3 = (torch.rand(16, n3, 128, 28, 28, device=dev, generator=g3) < 0.005).float()
            conv3 = make_conv(128, 128, 3, 1, 1, False, 3, device=dev)
            bn = nn.BatchNorm2d(128).to(dev).eval()
            m3 = FusedSparseConvLIF.from_conv_bn_lif(conv3, bn, LIFNode(tau=2.0, v_threshold=1.0, v_reset=0.0))

            def step():
                m3.reset()
                return m3(x3)
            nb = 4 * x3.numel() * 2 + 4 * n3 * 128 * 28 * 28 * 2 + 4 * 128 * 128 * 9
        else:
            x3 = torch.randn(16, n3, 128, 28, 28, device=dev, generator=g3)
            lif = LIFNode(tau=2.0, v_threshold=1.0, v_reset=0.0, step_mode="m")
            lif.emit_event_masks = args.kernel == "lif_events"

            def step():
                lif.reset()
                return lif(x3)
            nb = 4 * x3.numel() * 2 + 4 * n3 * 128 * 28 * 28
            if lif.emit_event_masks:
                nb += 16 * n3 * 28 * 28 * 16  # event masks: 2 words of 8 bytes per pixel
        with torch.no_grad():
            ms = cuda_time(step, args.steps, args.warmup, dist) / args.steps
        if rank == 0:
            print(json.dumps({"kernel": args.kernel, "ms_per_step": round(ms, 4), "GBps": round(nb / ms / 1e6, 1),
                              "frac_of_measured_hbm": round(nb / ms / 1e6 / hbm_peak, 3), "images": 16 * n3,
                              "bytes": nb}))
        if dist is not None:
            dist.destroy_process_group()
        return

    if args.only_timed and args.kernel == "prescan":
        from sparseflow_b200.Kernels._prescan_common import prescan2d
        x4 = x.reshape(n_img, C, H, W)
        nt = n_img * 7 * 4
        ag = torch.empty(nt, dtype=torch.int32, device=dev)
        tc, ids = torch.empty_like(ag), torch.empty_like(ag)
        cnt = torch.zeros(1, dtype=torch.int32, device=dev)
        ms = cuda_time(lambda: prescan2d(x4, 0, (H, W), (3, 3), 1, 1, (8, 16), 16, 1e-6, ag, tc, ids, cnt),
                       args.steps, args.warmup, dist) / args.steps
        pb = x4.numel() * 4 + nt * 12
        if rank == 0:
            print(json.dumps({"kernel": "prescan", "ms_per_step": round(ms, 4), "GBps": round(pb / ms / 1e6, 1),
                              "frac_of_measured_hbm": round(pb / ms / 1e6 / hbm_peak, 3), "images": n_img}))
        if dist is not None:
            dist.destroy_process_group()
        return

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = int(vis.split(",")[local]) if vis and vis.split(",")[local].strip().isdigit() else local
    sampler = ClockSampler(phys)  # NVML index (CUDA_VISIBLE_DEVICES maps local ranks to physical GPUs)
    sampler.start()
    with torch.no_grad():
        ms_total = cuda_time(lambda: mod(x), args.steps, args.warmup, dist)
    clocks = sampler.stop()
    ms_step = ms_total / args.steps
    value = world * step_bytes * args.steps / (ms_total / 1e3) / 1e9
    achieved = step_bytes / (ms_step / 1e3) / 1e9
    if args.only_timed:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
                              "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
                              "images": n_img, "only_timed": True, "clocks": clocks}))
        if dist is not None:
            dist.destroy_process_group()
        return

    # cuDNN dense on the same input (fp32, torch defaults: TF32 allowed for convs).
    x4 = x.reshape(n_img, C, H, W)
    with torch.no_grad():
        cud_ms = cuda_time(lambda: torch.nn.functional.conv2d(x4, conv.weight, conv.bias, 1, 1),
                           max(3, min(args.steps, 20)), 3) / max(3, min(args.steps, 20))
        tf32 = torch.backends.cudnn.allow_tf32
        torch.backends.cudnn.allow_tf32 = False
        cud32_ms = cuda_time(lambda: torch.nn.functional.conv2d(x4, conv.weight, conv.bias, 1, 1), 3, 1) / 3
        torch.backends.cudnn.allow_tf32 = tf32

    # End to end through the module: every step copies all of its spikes in from pinned host
    # memory and all of its output back. The batch goes in E2E_CHUNKS chunks on three streams
    # (upload of chunk i+1, convolution of chunk i, download of chunk i-1 overlap; PCIe is full
    # duplex), timed on the device from the first upload to the last download.
    e2e_steps = max(2, min(args.steps, 5))
    n4 = T_STEPS * n_batch
    x_host = x.reshape(n4, C, H, W).cpu().pin_memory()
    y_host = torch.empty((n4, C, H, W), dtype=torch.float32).pin_memory()
    x_dev = torch.empty((n4, C, H, W), dtype=torch.float32, device=dev)
    chunks = [(i * n4 // E2E_CHUNKS, (i + 1) * n4 // E2E_CHUNKS) for i in range(E2E_CHUNKS)]
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in chunks]
    ev_cmp = [torch.cuda.Event() for _ in chunks]
    ev_out = [torch.cuda.Event() for _ in chunks]

    # Each chunk's output stays referenced until the next step's output of that chunk replaces it;
    # that allocation is ordered after the wait for the chunk's previous download, so reusing the
    # memory is safe without record_stream (whose deferred frees made the allocator take fresh
    # blocks from the driver every step: 88 ms instead of 18 ms per step).
    ys = [None] * len(chunks)

    def e2e_step():
        for c, (a, b) in enumerate(chunks):
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_cmp[c])  # the previous step's convolution of this chunk has read x_dev
                x_dev[a:b].copy_(x_host[a:b], non_blocking=True)
                ev_in[c].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[c])
                s_cmp.wait_event(ev_out[c])  # the previous step's download of this chunk is done
                ys[c] = mod(x_dev[a:b])
                ev_cmp[c].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp[c])
                y_host[a:b].copy_(ys[c], non_blocking=True)
                ev_out[c].record(s_out)

    with torch.no_grad():
        e2e_step()  # warm-up
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_start.record(s_in)
        for _ in range(e2e_steps):
            e2e_step()
        s_in.wait_stream(s_out)
        t_end.record(s_in)
        torch.cuda.synchronize()
        e2e_ms = t_start.elapsed_time(t_end)
        if dist is not None:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e_ms /= e2e_steps
        # The downloaded output is the module's output (spot check of one chunk).
        assert torch.equal(y_host[:8].to(dev), mod(x_dev[:8]))
    e2e_val = world * step_bytes / (e2e_ms / 1e3) / 1e9
    # The host-side ceiling of that figure: every rank copying its 822 MB of pinned spikes to its
    # GPU at once (all ranks' copies share the host's memory and PCIe), max over ranks.
    with torch.no_grad():
        h2d_ms = cuda_time(lambda: x_dev.copy_(x_host, non_blocking=True), 3, 1, dist) / 3
    h2d_agg = world * x_host.numel() * 4 / (h2d_ms / 1e3) / 1e9
    del x_host, y_host, x_dev
    c4 = c4_sharded(dev, dist, world)

    extra = None
    if not args.no_extra and rank == 0:
        with torch.no_grad():
            extra = extras(dev, hbm_peak, args.steps)

    cpu = None
    if rank == 0 and world == 1:
        val, cores, sec, nsteps = time_reference_cpu(3, 1)
        cpu = {"value": round(val, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"the full step ({T_STEPS * N_BATCH} images), {nsteps} calls, {sec * 1e3:.0f} ms each; "
                         "torch F.conv2d on CPU = the reference SparseConv2d CPU path (Ops/sparse_conv2d.py:819-834); "
                         "the same helper as --impl reference"}

    traffic = None
    tf = ROOT / "profiles" / "conv3x3_tc_c5.traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Bernoulli spikes, kaiming weights)",
            "config": {"workload": f"C5 cell: SparseConv2d 3x3/s1/p1 C64->64, T16 N{n_batch} 56x56, Bernoulli(0.01) "
                                   "fp32 spikes, block 16 (per GPU)", "global_batch": n_batch * world,
                       "seq_len": T_STEPS, "parallelism": f"N-shard x{world}",
                       "l2": "inputs (822 MB) and outputs larger than L2; no flush"},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": x.numel() * 4,
                    "d2h_bytes_per_step": x.numel() * 4, "ms_per_step": round(e2e_ms, 3),
                    "pipeline": f"{E2E_CHUNKS} chunks on upload / compute / download streams",
                    "h2d_copy_GBps_all_ranks": round(h2d_agg, 1),
                    "h2d_copy_GBps_per_rank": round(h2d_agg / world, 1)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                         "frac_of_nominal_8TBps": round(achieved / 8000.0, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s",
                         "kernel": "one sf_sparse_conv2d call = conv3x3_tc_kernel<float,float,true> "
                                   "(tcgen05 kind::i8 implicit GEMM, x read once, y written once)",
                         "algorithmic_bytes_per_launch": step_bytes,
                         "bytes_model": "x read once + y written once + weights + bias"},
            "speedup_vs_cudnn": {"cudnn_default_ms": round(cud_ms, 4), "cudnn_fp32_no_tf32_ms": round(cud32_ms, 4),
                                 "ours_ms": round(ms_step, 4), "vs_default": round(cud_ms / ms_step, 2),
                                 "vs_fp32": round(cud32_ms / ms_step, 2)},
            "gpu_launches": args.steps,  # one conv3x3_tc_kernel launch per step
            "clocks": clocks,
            "cpu_baseline": cpu,
            "extra": extra,
            "c4_spiking_resnet50_sharded": c4,
        }
        print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
