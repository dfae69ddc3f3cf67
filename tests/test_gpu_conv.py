"""Stage-2 sparse conv on the GPU vs the reference golden outputs and the CPU oracle."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import load_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

CONV = load_cases("conv")
RTOL = 1e-5  # fp32 weights: rel 1e-5 of the output scale


def _assert_close(y, ref, rtol=RTOL):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 1e-6)
    err = np.abs(y - ref).max()
    assert err <= rtol * scale, f"max abs err {err} > {rtol} * {scale}"


@pytest.mark.parametrize("case", sorted(CONV))
def test_conv_matches_reference_golden(case):
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    c = CONV[case]
    k, s, p = (int(v) for v in c["geom"])
    w = torch.from_numpy(c["w"])
    conv = nn.Conv2d(w.shape[1], w.shape[0], k, s, p, bias="b" in c)
    conv.weight.data.copy_(w)
    if "b" in c:
        conv.bias.data.copy_(torch.from_numpy(c["b"]))
    sp = SparseConv2d.from_dense(conv.cuda(), block_size=8)
    y = sp(torch.from_numpy(c["x"]).cuda())
    assert tuple(y.shape) == c["y"].shape and y.dtype == torch.float32
    _assert_close(y.cpu().numpy(), c["y"])


GRID = [
    # n, c, h, w, co, k, s, p, density
    (2, 64, 32, 32, 64, 3, 1, 1, 0.02),
    (3, 3, 17, 9, 8, 3, 1, 1, 1.0),
    (2, 40, 13, 30, 24, 3, 1, 1, 0.1),
    (2, 130, 14, 14, 100, 3, 1, 1, 0.05),
    (2, 64, 56, 56, 64, 3, 1, 1, 0.01),
    (1, 256, 56, 56, 64, 1, 1, 0, 0.02),
    (2, 256, 28, 28, 200, 1, 1, 0, 0.05),
    (2, 32, 15, 15, 64, 3, 2, 1, 0.1),
    (2, 64, 56, 56, 128, 3, 2, 1, 0.02),
    (4, 64, 7, 7, 64, 3, 1, 1, 0.2),
    (2, 16, 57, 57, 32, 3, 1, 1, 0.05),
    (2, 32, 1, 1, 16, 3, 1, 1, 1.0),
    (1, 64, 20, 250, 32, 3, 1, 1, 0.01),
    (3, 512, 7, 7, 512, 1, 1, 0, 0.01),
    (2, 48, 12, 12, 256, 3, 1, 1, 0.0),
    # 1x1 (one-pass pointwise kernel): H*W not a multiple of 4, real values, ragged C and C_out,
    # stride 2 (the downsample), more channels than one mask word row holds
    (2, 40, 13, 30, 24, 1, 1, 0, 0.1),
    (3, 3, 17, 9, 8, 1, 1, 0, 1.0),
    (2, 64, 15, 15, 96, 1, 2, 0, 0.1),
    (2, 256, 28, 28, 512, 1, 2, 0, 0.02),
    (1, 1000, 7, 7, 40, 1, 1, 0, 0.05),
    (2, 64, 56, 56, 256, 1, 1, 0, 1.0),
    # 3x3 sweep corners: weights past shared memory (read from L2, 4 slices per lane),
    # dense (0.2) and nearly empty (0.001) inputs
    (2, 256, 14, 14, 256, 3, 1, 1, 0.2),
    (1, 256, 28, 28, 256, 3, 1, 1, 0.001),
    (1, 512, 14, 14, 512, 3, 1, 1, 0.2),
    (1, 512, 28, 28, 512, 3, 1, 1, 0.001),
    (2, 64, 56, 56, 64, 3, 1, 1, 0.2),
    (2, 128, 28, 28, 128, 3, 1, 1, 0.2),
    # every shared-memory weight block width: CPL 1 (C128->128), 2 (C64->128), 4 (C32->128)
    (2, 128, 28, 28, 128, 3, 1, 1, 0.01),
    (2, 64, 28, 28, 128, 3, 1, 1, 0.05),
    (2, 32, 28, 28, 128, 3, 1, 1, 0.05),
]


@pytest.mark.parametrize("n,c,h,w,co,k,s,p,density", GRID)
def test_conv_vs_oracle(n, c, h, w, co, k, s, p, density):
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator().manual_seed(c * 31 + co + h)
    x = (torch.rand(n, c, h, w, generator=g) < density).float()
    if density == 1.0:
        x = torch.randn(n, c, h, w, generator=g) * (torch.rand(n, c, h, w, generator=g) < 0.5)
    wt = torch.randn(co, c, k, k, generator=g) * (2.0 / (c * k * k)) ** 0.5
    b = torch.randn(co, generator=g) * 0.1
    y, _ = sparse_conv2d_forward(x.cuda(), wt.cuda(), b.cuda(), kernel_size=k, stride=s, padding=p)
    ref = oracle.conv2d(x.numpy(), wt.numpy(), b.numpy(), s, p)
    _assert_close(y.cpu().numpy(), ref)


@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_conv_dtypes_vs_oracle(xdt, wdt):
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator().manual_seed(11)
    x = ((torch.rand(4, 64, 28, 28, generator=g) < 0.03).float()).to(xdt)
    wt = (torch.randn(96, 64, 3, 3, generator=g) * 0.05).to(wdt)
    y, _ = sparse_conv2d_forward(x.cuda(), wt.cuda(), None, kernel_size=3, stride=1, padding=1)
    assert y.dtype == xdt
    ref = oracle.conv2d(x.float().numpy(), wt.float().numpy(), None, 1, 1)
    # fp32 accumulation; the only rounding is the final cast to the 16-bit output dtype
    _assert_close(y.float().cpu().numpy(), ref, rtol=1e-2)


def test_conv_bf16_weights_c2_like():
    """C2-style 1x1 bottleneck with bf16 weights and fp32 spikes: within 1e-2 (bf16-weight bound)."""
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    g = torch.Generator().manual_seed(5)
    conv = nn.Conv2d(256, 64, 1, bias=False)
    conv.weight.data = (torch.randn(64, 256, 1, 1, generator=g) * 0.02).bfloat16()
    blk = (torch.rand(2, 4, 256, 4, 4, generator=g) < 0.05).float()
    mask = blk.repeat_interleave(16, 3).repeat_interleave(16, 4)[..., :56, :56]
    x = mask * (torch.rand(2, 4, 256, 56, 56, generator=g) < 0.3).float()
    w_ref = conv.weight.detach().float().numpy().copy()
    sp = SparseConv2d.from_dense(conv.cuda(), block_size=16)
    y = sp(x.cuda())
    ref = oracle.conv2d(x.reshape(8, 256, 56, 56).numpy(), w_ref, None, 1, 0)
    _assert_close(y.reshape(8, 64, 56, 56).cpu().numpy(), ref, rtol=1e-5)


def test_c1_full_shape_through_sparse_conv2d():
    """BASELINE config C1 at full shape: [T=4, N=8, 64, 32, 32], Bernoulli(0.02), kaiming weights,
    bias, block 16, through SparseConv2d (5-D in, 5-D out) against the oracle."""
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    g = torch.Generator().manual_seed(2024)
    conv = nn.Conv2d(64, 64, 3, 1, 1, bias=True)
    w = torch.empty(64, 64, 3, 3)
    nn.init.kaiming_normal_(w, generator=g)
    conv.weight.data.copy_(w)
    conv.bias.data.copy_(torch.randn(64, generator=g) * 0.1)
    x = (torch.rand(4, 8, 64, 32, 32, generator=g) < 0.02).float()
    sp = SparseConv2d.from_dense(conv.cuda(), block_size=16)
    y = sp(x.cuda())
    assert y.shape == (4, 8, 64, 32, 32)
    ref = oracle.conv2d(x.reshape(32, 64, 32, 32).numpy(), w.numpy(), conv.bias.detach().cpu().numpy(), 1, 1)
    _assert_close(y.reshape(32, 64, 32, 32).cpu().numpy(), ref)


def test_conv_deterministic_and_5d_shape():
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    conv = nn.Conv2d(64, 64, 3, 1, 1).cuda()
    sp = SparseConv2d.from_dense(conv, block_size=16)
    g = torch.Generator(device="cuda").manual_seed(1)
    x = (torch.rand(4, 8, 64, 32, 32, device="cuda", generator=g) < 0.02).float()
    y1 = sp(x)
    y2 = sp(x)
    assert y1.shape == (4, 8, 64, 32, 32)
    assert torch.equal(y1, y2)


def test_conv_full_size_c5_cell_vs_cudnn_fp32():
    """Full bench workload (T=16, N=64, C=64, 56x56, p=0.01): against cuDNN with TF32 off."""
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator(device="cuda").manual_seed(2)
    x = (torch.rand(1024, 64, 56, 56, device="cuda", generator=g) < 0.01).float()
    w = torch.randn(64, 64, 3, 3, device="cuda", generator=g) * 0.06
    b = torch.randn(64, device="cuda", generator=g) * 0.1
    y, _ = sparse_conv2d_forward(x, w, b, kernel_size=3, stride=1, padding=1)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        ref = torch.nn.functional.conv2d(x, w, b, 1, 1)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    err = (y - ref).abs().max().item()
    assert err <= RTOL * ref.abs().max().item()
    y2, _ = sparse_conv2d_forward(x, w, b, kernel_size=3, stride=1, padding=1)
    assert torch.equal(y, y2)


def test_conv_metadata_buffers_match_prescan():
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator().manual_seed(9)
    x = (torch.rand(4, 64, 32, 32, generator=g) < 0.0005).float()
    w = torch.randn(64, 64, 3, 3, generator=g) * 0.05
    nt = 4 * 4 * 4
    agb = torch.empty(nt, dtype=torch.int32, device="cuda")
    tcb = torch.empty(nt, dtype=torch.int32, device="cuda")
    y, ms, ratio, stats, meta = sparse_conv2d_forward(
        x.cuda(), w.cuda(), None, kernel_size=3, stride=1, padding=1, ag_mask_buf=agb, tile_class_buf=tcb,
        return_ms=True, return_avg_active_ratio=True, return_tile_stats=True, return_backend_meta=True)
    oag, otc, oids = oracle.prescan2d(x.numpy(), 0, 32, 32, 3, 1, 1, 8, 8, 16, 1e-6)
    np.testing.assert_array_equal(agb.cpu().numpy(), oag)
    assert stats["zero_tiles"] == int((otc == 0).sum())
    assert ms > 0 and meta["backend"] == "sparse_b200"


@pytest.mark.parametrize("s", [1, 2])
def test_conv1x1_one_pass_matches_two_stage(s):
    """The one-pass 1x1 kernel, the two-stage (mask pass + gather) path and the tcgen05 kernel agree."""
    from sparseflow_b200 import _lib
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator().manual_seed(21)
    x = (torch.rand(4, 128, 28, 28, generator=g) < 0.03).float().cuda()
    wt = (torch.randn(64, 128, 1, 1, generator=g) * 0.1).cuda()
    y1, _ = sparse_conv2d_forward(x, wt, None, kernel_size=1, stride=1, padding=0)
    with _lib.path_policy(_lib.SF_POLICY_CONV1X1_PATH, 2):
        y2, _ = sparse_conv2d_forward(x, wt, None, kernel_size=1, stride=1, padding=0)
    with _lib.path_policy(_lib.SF_POLICY_CONV1X1_PATH, 1):
        y4, _ = sparse_conv2d_forward(x, wt, None, kernel_size=1, stride=1, padding=0)
    torch.testing.assert_close(y1, y2, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(y1, y4, rtol=1e-6, atol=1e-6)
    if s == 2:
        y3, _ = sparse_conv2d_forward(x, wt, None, kernel_size=1, stride=2, padding=0)
        torch.testing.assert_close(y3, y1[:, :, ::2, ::2], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("h,w", [(8, 8), (3, 12), (8, 16)])
def test_conv1x1_small_images_both_paths(h, w):
    """Images of fewer than 128 pixels take the gather kernels by default; forced onto the
    tensor-core kernel (SF_POLICY_CONV1X1_TC_MIN_HW = 1) its padded single sub-tile gives the same result."""
    from sparseflow_b200 import _lib
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator().manual_seed(h * w)
    x = (torch.rand(40, 64, h, w, generator=g) < 0.05).float()
    wt = torch.randn(256, 64, 1, 1, generator=g) * 0.1
    b = torch.randn(256, generator=g) * 0.1
    ref = oracle.conv2d(x.numpy(), wt.numpy(), b.numpy(), 1, 0)
    y_default, _ = sparse_conv2d_forward(x.cuda(), wt.cuda(), b.cuda(), kernel_size=1, stride=1, padding=0)
    with _lib.path_policy(_lib.SF_POLICY_CONV1X1_TC_MIN_HW, 1):
        y_tc, _ = sparse_conv2d_forward(x.cuda(), wt.cuda(), b.cuda(), kernel_size=1, stride=1, padding=0)
    _assert_close(y_default.cpu().numpy(), ref)
    _assert_close(y_tc.cpu().numpy(), ref)


@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_conv1x1_bf16_exact_values_on_tensor_cores(wdt):
    """Small integers and powers of two are exact in bf16, so the tensor-core 1x1 path keeps
    them (not only 0/1 spikes); real values in other images take the exact CUDA-core path."""
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator().manual_seed(23)
    x = torch.randint(-3, 4, (3, 96, 24, 24), generator=g).float() * (torch.rand(3, 96, 24, 24, generator=g) < 0.1)
    x[1] *= 0.25                                   # powers of two stay exact
    x[2] = torch.randn(96, 24, 24, generator=g) * (torch.rand(96, 24, 24, generator=g) < 0.1)
    wt = (torch.randn(80, 96, 1, 1, generator=g) * 0.1).to(wdt)
    b = torch.randn(80, generator=g) * 0.1
    y, _ = sparse_conv2d_forward(x.cuda(), wt.cuda(), b.cuda(), kernel_size=1, stride=1, padding=0)
    ref = oracle.conv2d(x.numpy(), wt.float().numpy(), b.numpy(), 1, 0)
    _assert_close(y.cpu().numpy(), ref)


@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("co", [48, 300])
def test_conv1x1_16bit_inputs_vs_oracle(xdt, co):
    """1x1 with 16-bit activations: the tensor-core kernel for C_out <= 256 (f16 values that are
    not bf16-exact take its CUDA-core tiles), the gather kernels above."""
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator().manual_seed(co)
    x = (torch.rand(3, 128, 20, 20, generator=g) < 0.05).float()
    x[2] *= torch.randn(128, 20, 20, generator=g)  # one image with real values
    x = x.to(xdt)
    wt = torch.randn(co, 128, 1, 1, generator=g) * 0.1
    y, _ = sparse_conv2d_forward(x.cuda(), wt.cuda(), None, kernel_size=1, stride=1, padding=0)
    assert y.dtype == xdt
    ref = oracle.conv2d(x.float().numpy(), wt.numpy(), None, 1, 0)
    _assert_close(y.float().cpu().numpy(), ref, rtol=1e-2)


def test_conv1x1_full_size_c2_cell_vs_cudnn_fp32():
    """Full C2 workload (T=16, N=32, 256->64, 56x56, block-clustered spikes, bf16 weights) on the
    tensor-core path: against cuDNN fp32 (TF32 off) on the same bf16-valued weights, and
    deterministic across runs."""
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    g = torch.Generator(device="cuda").manual_seed(17)
    blk = (torch.rand(512, 256, 4, 4, device="cuda", generator=g) < 0.05).float()
    mask = blk.repeat_interleave(16, 2).repeat_interleave(16, 3)[:, :, :56, :56]
    x = (mask * (torch.rand(512, 256, 56, 56, device="cuda", generator=g) < 0.3).float()).contiguous()
    del blk, mask
    w = (torch.randn(64, 256, 1, 1, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    y, _ = sparse_conv2d_forward(x, w, None, kernel_size=1, stride=1, padding=0)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        ref = torch.nn.functional.conv2d(x, w.float())
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    assert (y - ref).abs().max().item() <= RTOL * ref.abs().max().item()
    y2, _ = sparse_conv2d_forward(x, w, None, kernel_size=1, stride=1, padding=0)
    assert torch.equal(y, y2)
