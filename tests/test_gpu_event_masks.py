"""Fused conv + LIF emits the next layer's event masks; a following SparseConv2d runs from them."""
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


def _masks_from_spikes(s4):
    """[N, C, H, W] -> int64 [N, H, W, ceil(C/64)] with bit c%64 of word c//64 = (s != 0)."""
    n, c, h, w = s4.shape
    nw = (c + 63) // 64
    pad = torch.zeros(n, nw * 64, h, w, dtype=torch.bool, device=s4.device)
    pad[:, :c] = s4 != 0
    bits = pad.reshape(n, nw, 64, h, w).permute(0, 3, 4, 1, 2).to(torch.int64)
    weights = torch.ones(64, dtype=torch.int64, device=s4.device) << torch.arange(64, device=s4.device)
    return (bits * weights).sum(-1)  # wraps into int64 like the kernel's uint64 words


def _fused(c_in, c_out, k, seed):
    from sparseflow_b200.Ops.sparse_fused_conv_lif import FusedSparseConvLIF
    from sparseflow_b200.Ops.lif_node import LIFNode
    g = torch.Generator().manual_seed(seed)
    conv = nn.Conv2d(c_in, c_out, k, 1, k // 2, bias=True)
    conv.weight.data = torch.randn(c_out, c_in, k, k, generator=g) * (3.0 / (c_in * k * k)) ** 0.5
    conv.bias.data = torch.randn(c_out, generator=g) * 0.3
    m = FusedSparseConvLIF.from_conv_and_lif(conv.cuda(), LIFNode(tau=2.0, v_threshold=0.5, v_reset=0.0))
    m.emit_event_masks = True
    return m


@pytest.mark.parametrize("c_in,c_out,k", [(64, 64, 3), (32, 40, 3), (48, 130, 1)])
def test_fused_lif_masks_match_spikes(c_in, c_out, k):
    g = torch.Generator().manual_seed(c_out)
    x = (torch.rand(4, 3, c_in, 14, 15, generator=g) < 0.2).float().cuda()
    m = _fused(c_in, c_out, k, 7)
    s = m(x)
    masks = s._sf_event_masks[0]
    want = _masks_from_spikes(s.reshape(12, c_out, 14, 15))
    assert float(s.mean()) > 0.01  # the layer does fire
    assert torch.equal(masks.reshape(want.shape), want)


@pytest.mark.parametrize("c_mid,k2,hw", [(64, 3, 12), (40, 3, 12), (72, 1, 10)])
def test_next_conv_runs_from_masks(c_mid, k2, hw):
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    g = torch.Generator().manual_seed(c_mid + k2)
    x = (torch.rand(4, 2, 32, hw, hw, generator=g) < 0.1).float().cuda()
    first = _fused(32, c_mid, 3, 9)
    conv2 = nn.Conv2d(c_mid, 48, k2, 1, k2 // 2)
    conv2.weight.data = torch.randn(48, c_mid, k2, k2, generator=g) * 0.1
    second = SparseConv2d.from_dense(conv2.cuda())
    s = first(x)
    # The gather kernel on both runs (3x3 with C_in <= 64 would otherwise take the tensor-core
    # kernel from the spikes, and 1x1 on images below one 128-pixel MMA tile is gathered anyway).
    from sparseflow_b200 import _lib
    with _lib.path_policy(_lib.SF_POLICY_CONV3X3_PATH, 1):
        y_masks = second(s)
        assert second._last_used_event_masks
        y_plain = second(s.clone())  # a new tensor: no masks attached, mask pass runs
        assert not second._last_used_event_masks
    torch.testing.assert_close(y_masks, y_plain, rtol=0, atol=0)
    if k2 == 3 and c_mid <= 64:
        y_tc = second(s)  # default policy: the tensor-core kernel reads the spikes, masks unused
        assert not second._last_used_event_masks
        torch.testing.assert_close(y_tc, y_plain, rtol=1e-5, atol=1e-5)


def test_1x1_on_large_images_runs_from_masks_on_tensor_cores():
    """A 1x1/s1 layer (bf16 weights) on images of at least 128 pixels given the producer's event
    masks runs the tcgen05 kernel with its A operand built from the masks (x is not read): bit for
    bit the result from the spikes, within 1e-5 of the float64 reference."""
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    for c_mid, hw in ((72, 12), (256, 16), (130, 14)):
        g = torch.Generator().manual_seed(c_mid + hw)
        x = (torch.rand(4, 2, 32, hw, hw, generator=g) < 0.1).float().cuda()
        first = _fused(32, c_mid, 3, 9)
        conv2 = nn.Conv2d(c_mid, 48, 1, 1, 0)
        conv2.weight.data = (torch.randn(48, c_mid, 1, 1, generator=g) * 0.1).bfloat16().float()
        conv2 = conv2.cuda().to(torch.bfloat16)  # bf16 weights: the tensor-core kernel runs from the masks
        second = SparseConv2d.from_dense(conv2)
        s = first(x)
        assert getattr(s, "_sf_event_masks", None) is not None
        y = second(s)
        assert second._last_used_event_masks
        y_plain = second(s.clone())
        assert not second._last_used_event_masks
        ref = torch.nn.functional.conv2d(s.reshape(8, c_mid, hw, hw).double(), conv2.weight.double(),
                                         conv2.bias.double())
        y = y.double()
        y_plain = y_plain.double()
        torch.testing.assert_close(y.reshape(8, 48, hw, hw), ref, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(y, y_plain, rtol=0, atol=0)  # same kernel, same sums, same order


def test_stale_masks_are_not_used():
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    x = (torch.rand(2, 2, 32, 10, 10) < 0.2).float().cuda()
    first = _fused(32, 32, 3, 3)
    conv2 = nn.Conv2d(32, 16, 3, 1, 1).cuda()
    second = SparseConv2d.from_dense(conv2)
    s = first(x)
    s.zero_()  # in place: the attached masks no longer describe s
    y = second(s)
    assert not second._last_used_event_masks
    torch.testing.assert_close(y, conv2.bias.detach().view(1, 1, 16, 1, 1).expand_as(y), rtol=0, atol=1e-6)


def test_masks_off_by_default_and_plain_lif_unchanged():
    """Without emission the spikes carry no masks and equal the emitting kernel's spikes."""
    x = (torch.rand(3, 2, 32, 9, 11) < 0.2).float().cuda()
    a = _fused(32, 48, 3, 5)
    b = _fused(32, 48, 3, 5)
    b.emit_event_masks = False
    sa, sb = a(x), b(x)
    assert not hasattr(sb, "_sf_event_masks")
    torch.testing.assert_close(sa, sb, rtol=0, atol=0)
    torch.testing.assert_close(a.v, b.v, rtol=0, atol=0)


# Standalone LIF (the LIFNode after a BN) writing the next convolution's events.

def _lif_pair(c, h, w, dtype, seed, t=3, n=2):
    from sparseflow_b200.Ops.lif_node import LIFNode
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(t, n, c, h, w, generator=g) * 1.5 + 0.3).to(dtype).cuda()
    plain = LIFNode(tau=2.0, v_threshold=1.0, v_reset=0.0)
    ev = LIFNode(tau=2.0, v_threshold=1.0, v_reset=0.0)
    ev.emit_event_masks = True
    return x, plain, ev


@pytest.mark.parametrize("c,h,w,dtype", [(64, 14, 14, torch.float32), (32, 8, 8, torch.float32),
                                          (40, 7, 9, torch.float32), (130, 6, 6, torch.float32),
                                          (96, 12, 10, torch.float16), (64, 5, 5, torch.bfloat16)])
def test_lif_events_match_spikes_and_plain_lif(c, h, w, dtype):
    x, plain, ev = _lif_pair(c, h, w, dtype, c + h)
    s_plain = plain(x)
    s_ev = ev(x)
    assert torch.equal(s_ev, s_plain)
    assert torch.equal(ev.v, plain.v)
    masks = s_ev._sf_event_masks[0]
    t, n = x.shape[:2]
    want = _masks_from_spikes(s_ev.reshape(t * n, c, h, w))
    assert 0.05 < float(s_ev.float().mean()) < 0.95
    assert torch.equal(masks[: want.numel()].reshape(want.shape), want)
    # A second call continues from the stored membrane, like the plain node.
    assert torch.equal(ev(x), plain(x))
    assert torch.equal(ev.v, plain.v)


def test_lif_events_drive_next_conv():
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    x, _, ev = _lif_pair(64, 16, 16, torch.float32, 5, t=2, n=3)
    conv = nn.Conv2d(64, 48, 3, 1, 1)
    conv.weight.data = torch.randn(48, 64, 3, 3, generator=torch.Generator().manual_seed(1)) * 0.1
    sc = SparseConv2d.from_dense(conv.cuda())
    s = ev(x)
    from sparseflow_b200 import _lib
    with _lib.path_policy(_lib.SF_POLICY_CONV3X3_PATH, 1):  # gather kernel, from masks or spikes
        y_masks = sc(s)
        assert sc._last_used_event_masks
        y_plain = sc(s.clone())
        assert not sc._last_used_event_masks
    torch.testing.assert_close(y_masks, y_plain, rtol=0, atol=0)


@pytest.mark.parametrize("c,h,w,tau", [(64, 14, 14, 2.0), (32, 8, 8, 3.0), (128, 7, 8, 2.0)])
def test_lif_events_general_kernel(c, h, w, tau):
    """The lane-per-pixel kernel that serves shapes the bitmap path does not take, forced on shapes it would."""
    from sparseflow_b200 import _lib
    with _lib.path_policy(_lib.SF_POLICY_LIF_EVENTS_GENERAL, 1):
        _lif_events_general_body(c, h, w, tau)


def _lif_events_general_body(c, h, w, tau):
    from sparseflow_b200.Ops.lif_node import LIFNode
    g = torch.Generator().manual_seed(c)
    x = (torch.randn(3, 2, c, h, w, generator=g) * 1.5 + 0.3).cuda()
    plain = LIFNode(tau=tau, v_threshold=1.0, v_reset=0.0)
    ev = LIFNode(tau=tau, v_threshold=1.0, v_reset=0.0)
    ev.emit_event_masks = True
    s_ev, s_plain = ev(x), plain(x)
    assert torch.equal(s_ev, s_plain) and torch.equal(ev.v, plain.v)
    want = _masks_from_spikes(s_ev.reshape(6, c, h, w))
    masks = s_ev._sf_event_masks[0]
    assert torch.equal(masks[: want.numel()].reshape(want.shape), want)


@pytest.mark.parametrize("tau,v_reset", [(3.0, 0.0), (2.0, None), (0.5, -0.2)])
def test_lif_events_bitmap_path_params(tau, v_reset):
    """Bitmap path (C*H*W % 128 == 0) with non-power-of-two tau and soft / negative reset."""
    from sparseflow_b200.Ops.lif_node import LIFNode
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(4, 2, 64, 8, 8, generator=g) * 1.5 + 0.3).cuda()
    plain = LIFNode(tau=tau, v_threshold=1.0, v_reset=v_reset)
    ev = LIFNode(tau=tau, v_threshold=1.0, v_reset=v_reset)
    ev.emit_event_masks = True
    s_ev, s_plain = ev(x), plain(x)
    assert torch.equal(s_ev, s_plain) and torch.equal(ev.v, plain.v)
    want = _masks_from_spikes(s_ev.reshape(8, 64, 8, 8))
    assert torch.equal(s_ev._sf_event_masks[0].reshape(want.shape), want)


@pytest.mark.parametrize("density,expect", [(0.001, 1), (0.05, 2)])
def test_wide_3x3_masks_or_x_picks_a_route(density, expect):
    """C_in 128 3x3/s1 given x and its event masks: sparse spikes run the gather kernel from the
    masks, dense ones the tensor cores from x; the result equals that route's bit for bit and the
    oracle within fp32 rounding."""
    from sparseflow_b200 import _lib
    from sparseflow_b200.Kernels.conv2d import pack_weight
    from oracle import oracle
    g = torch.Generator().manual_seed(int(density * 1e4))
    x = (torch.rand(8, 128, 14, 14, generator=g) < density).float()
    wt = torch.randn(96, 128, 3, 3, generator=g) * 0.05
    b = torch.randn(96, generator=g) * 0.1
    xs, wp, bs = x.cuda(), pack_weight(wt.cuda()), b.cuda()
    masks = _masks_from_spikes(xs).contiguous()
    y = torch.empty(8, 96, 14, 14, device="cuda")
    _lib.sparse_conv2d_masks_or_x(xs, masks, wp, bs, y, 3, 1, 1)
    ref = torch.empty_like(y)
    with _lib.path_policy(_lib.SF_POLICY_CONV3X3_PATH, expect):
        if expect == 1:
            _lib.sparse_conv2d_from_masks(masks, tuple(xs.shape), xs.dtype, wp, bs, ref, 3, 1, 1)
        else:
            _lib.sparse_conv2d(xs, wp, bs, ref, 96, 3, 1, 1)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    o = oracle.conv2d(x.numpy(), wt.numpy(), b.numpy(), 1, 1)
    assert float((y.cpu() - torch.from_numpy(o)).abs().max()) <= 2e-5 * float(abs(o).max())
    assert _lib.conv_status(y.device) == 0


def test_fused_lif_to_wide_3x3_through_modules():
    """FusedSparseConvLIF (emitting masks) -> SparseConv2d C_in 128 at a firing rate above the
    gate: the convolution runs from x on the tensor cores and equals the plain call on the spikes."""
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    m = _fused(64, 128, 3, 11)
    g = torch.Generator().manual_seed(3)
    x = (torch.rand(3, 2, 64, 12, 12, generator=g) < 0.2).float().cuda()
    s = m(x)
    assert s._sf_event_masks is not None and float(s.mean()) > 0.01
    conv = nn.Conv2d(128, 96, 3, 1, 1, bias=True).cuda()
    sc = SparseConv2d.from_dense(conv, block_size=8)
    y = sc(s)
    plain = sc(s.clone())
    torch.cuda.synchronize()
    assert torch.equal(y, plain)
