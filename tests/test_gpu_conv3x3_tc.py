"""The tcgen05 3x3 convolution (integer MMA over 0/1 spikes, 3-digit weights) vs the oracle,
against the gather kernel, and on the fallback for inputs that are not 0/1."""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def _close(y, ref, rtol=RTOL):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 1e-6)
    err = np.abs(y - ref).max()
    assert err <= rtol * scale, f"max abs err {err} > {rtol} * {scale}"


def _run(x, w, b, path):
    from sparseflow_b200 import _lib
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    with _lib.path_policy(_lib.SF_POLICY_CONV3X3_PATH, path):
        y, _ = sparse_conv2d_forward(x, w, b, kernel_size=3, stride=1, padding=1)
    return y


GEOM = [
    # n, c, h, w, co, density
    (2, 64, 56, 56, 64, 0.01),
    (3, 64, 32, 32, 64, 0.2),
    (4, 16, 8, 8, 32, 0.1),
    (2, 3, 17, 9, 8, 0.5),
    (2, 40, 13, 30, 24, 0.1),
    (1, 64, 20, 250, 64, 0.05),
    (5, 32, 7, 7, 100, 0.3),
    (2, 64, 28, 28, 128, 0.05),
    (3, 48, 1, 1, 16, 0.5),
    (2, 64, 15, 3, 64, 0.0),
    (64, 64, 8, 8, 64, 0.02),
    (1, 33, 57, 57, 65, 0.03),
    # C_in > 64: weight stages stream past the resident input (32-channel output blocks)
    (2, 128, 28, 28, 128, 0.05),
    (2, 96, 13, 30, 40, 0.1),
    (1, 130, 9, 9, 200, 0.2),
    (1, 256, 14, 14, 256, 0.2),
    (1, 512, 14, 14, 512, 0.01),
    (1, 512, 56, 56, 32, 0.01),
    (3, 256, 7, 7, 64, 0.3),
    # weight stages of 5 and 6 slice pairs (C_in 160 and 192; 384 takes two 6-pair stages a tap)
    (1, 160, 12, 12, 64, 0.1),
    (2, 192, 10, 11, 96, 0.15),
    (1, 384, 9, 9, 64, 0.05),
]


@pytest.mark.parametrize("n,c,h,w,co,density", GEOM)
def test_tc3x3_vs_oracle_and_gather(n, c, h, w, co, density):
    g = torch.Generator().manual_seed(n * 1000 + c * 7 + co + h)
    x = (torch.rand(n, c, h, w, generator=g) < density).float()
    wt = torch.randn(co, c, 3, 3, generator=g) * (2.0 / (c * 9)) ** 0.5
    b = torch.randn(co, generator=g) * 0.1
    ref = oracle.conv2d(x.numpy(), wt.numpy(), b.numpy(), 1, 1)
    y_tc = _run(x.cuda(), wt.cuda(), b.cuda(), 2)
    y_g = _run(x.cuda(), wt.cuda(), b.cuda(), 1)
    _close(y_tc.cpu().numpy(), ref)
    _close(y_g.cpu().numpy(), ref)
    # deterministic: integer sums, fixed combine order
    assert torch.equal(y_tc, _run(x.cuda(), wt.cuda(), b.cuda(), 2))


@pytest.mark.parametrize("xdt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_tc3x3_dtypes(xdt, wdt):
    g = torch.Generator().manual_seed(17)
    x = (torch.rand(4, 64, 28, 28, generator=g) < 0.05).float().to(xdt)
    wt = (torch.randn(64, 64, 3, 3, generator=g) * 0.06).to(wdt)
    y = _run(x.cuda(), wt.cuda(), None, 2)
    assert y.dtype == xdt
    ref = oracle.conv2d(x.float().numpy(), wt.float().numpy(), None, 1, 1)
    _close(y.float().cpu().numpy(), ref, rtol=RTOL if xdt == torch.float32 else 1e-2)


def test_tc3x3_non_binary_units_take_the_fp32_path():
    """Real values in some images: their units are recomputed with fp32 FMAs, the rest stay on the MMA."""
    g = torch.Generator().manual_seed(5)
    x = (torch.rand(6, 32, 20, 20, generator=g) < 0.1).float()
    x[2] *= torch.randn(32, 20, 20, generator=g)
    x[5, 3, 7, 7] = 0.5
    x[0, 0, 0, 0] = 2.0  # an integer that is not 0/1
    wt = torch.randn(48, 32, 3, 3, generator=g) * 0.1
    b = torch.randn(48, generator=g)
    ref = oracle.conv2d(x.numpy(), wt.numpy(), b.numpy(), 1, 1)
    _close(_run(x.cuda(), wt.cuda(), b.cuda(), 2).cpu().numpy(), ref)


def test_tc3x3_extreme_weight_ranges():
    """Per-channel fixed point: channels of very different scale, an all-zero channel, tiny weights."""
    g = torch.Generator().manual_seed(8)
    x = (torch.rand(2, 64, 16, 16, generator=g) < 0.2).float()
    wt = torch.randn(64, 64, 3, 3, generator=g)
    wt[0] *= 1e-30
    wt[1] = 0
    wt[2] *= 1e6
    wt[3, :, 1, 1] = 1e-3  # one large weight per input channel dominates the scale
    wt[3, 0, 0, 0] = 5.0
    ref = oracle.conv2d(x.numpy(), wt.numpy(), None, 1, 1)
    y = _run(x.cuda(), wt.cuda(), None, 2).cpu().numpy()
    for co in range(64):
        _close(y[:, co], ref[:, co])


def test_tc3x3_full_size_c5_cell_vs_cudnn_fp32():
    """Headline workload (1024 images, C64 56x56, p=0.01) on the tensor-core path vs cuDNN fp32."""
    g = torch.Generator(device="cuda").manual_seed(2)
    x = (torch.rand(1024, 64, 56, 56, device="cuda", generator=g) < 0.01).float()
    w = torch.randn(64, 64, 3, 3, device="cuda", generator=g) * 0.06
    b = torch.randn(64, device="cuda", generator=g) * 0.1
    y = _run(x, w, b, 2)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        ref = torch.nn.functional.conv2d(x, w, b, 1, 1)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    assert (y - ref).abs().max().item() <= RTOL * ref.abs().max().item()
    from sparseflow_b200 import _lib
    assert _lib.conv_status(x.device) == 0


@pytest.mark.parametrize("c,density,expect", [(128, 0.0005, 1), (128, 0.05, 2), (256, 0.005, 1), (256, 0.1, 2),
                                               (512, 0.003, 1), (512, 0.05, 2)])
def test_density_gate_picks_one_path(c, density, expect):
    """For C_in > 64 a sampled nonzero count picks the gather kernel (sparse inputs) or the
    tensor-core kernel on the device; the automatic result equals that path's bit for bit."""
    g = torch.Generator().manual_seed(c + int(density * 1e4))
    x = (torch.rand(8, c, 14, 14, generator=g) < density).float().cuda()
    wt = (torch.randn(c, c, 3, 3, generator=g) * 0.05).cuda()
    b = torch.randn(c, generator=g).cuda()
    auto = _run(x, wt, b, 0)
    forced = _run(x, wt, b, expect)
    other = _run(x, wt, b, 3 - expect)
    assert torch.equal(auto, forced)
    _close(auto.cpu().numpy(), other.cpu().numpy())


def test_tc3x3_streamed_weights_non_binary_and_16bit():
    """C_in > 64 (weights streamed): units holding values other than 0/1 take the fp32 path for
    every output block; bf16 and fp16 inputs convert through the scalar converter."""
    g = torch.Generator().manual_seed(12)
    x = (torch.rand(5, 96, 12, 20, generator=g) < 0.1).float()
    x[3] *= torch.randn(96, 12, 20, generator=g)
    wt = torch.randn(80, 96, 3, 3, generator=g) * 0.05
    b = torch.randn(80, generator=g)
    ref = oracle.conv2d(x.numpy(), wt.numpy(), b.numpy(), 1, 1)
    _close(_run(x.cuda(), wt.cuda(), b.cuda(), 2).cpu().numpy(), ref)
    xs = (torch.rand(3, 160, 9, 13, generator=g) < 0.2).float()
    for dt in (torch.bfloat16, torch.float16):
        y = _run(xs.to(dt).cuda(), wt[:, :1].repeat(1, 160, 1, 1).cuda() * 0.5, None, 2)
        ref = oracle.conv2d(xs.numpy(), (wt[:, :1].repeat(1, 160, 1, 1) * 0.5).numpy(), None, 1, 1)
        _close(y.float().cpu().numpy(), ref, rtol=1e-2)


def test_tc3x3_unaligned_input_takes_scalar_converter():
    """x not 16-byte aligned (a view at an odd element offset): the scalar converter path."""
    g = torch.Generator().manual_seed(13)
    base = (torch.rand(2 * 64 * 20 * 20 + 1, generator=g) < 0.05).float()
    x = base[1:].reshape(2, 64, 20, 20)
    wt = torch.randn(64, 64, 3, 3, generator=g) * 0.05
    xd = base.cuda()[1:].reshape(2, 64, 20, 20)
    assert xd.data_ptr() % 16 != 0
    ref = oracle.conv2d(x.numpy(), wt.numpy(), None, 1, 1)
    _close(_run(xd, wt.cuda(), None, 2).cpu().numpy(), ref)


@pytest.mark.parametrize("fresh_thread", [False, True])
def test_gated_routes_under_cuda_graph_capture(fresh_thread):
    """A gated 3x3 call (C_in > 64, both routes launched) captured into a CUDA graph replays to the
    eager result bit for bit: with a side stream already made (fork and join captured) and from a
    thread that has none yet (both routes in order on the captured stream)."""
    import threading
    g = torch.Generator().manual_seed(41)
    res = {}
    for density in (0.001, 0.05):
        x = (torch.rand(8, 128, 14, 14, generator=g) < density).float().cuda()
        wt = (torch.randn(128, 128, 3, 3, generator=g) * 0.05).cuda()
        eager = _run(x, wt, None, 0)

        def capture():
            from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward, pack_weight
            wp = pack_weight(wt)
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                if not fresh_thread:
                    sparse_conv2d_forward(x, wt, None, kernel_size=3, stride=1, padding=1, w_cl=wp)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    y, _ = sparse_conv2d_forward(x, wt, None, kernel_size=3, stride=1, padding=1, w_cl=wp)
                graph.replay()
            torch.cuda.synchronize()
            res[density] = y.clone()

        if fresh_thread:
            th = threading.Thread(target=capture)
            th.start()
            th.join()
        else:
            capture()
        assert torch.equal(res[density], eager)
