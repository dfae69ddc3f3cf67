"""Fused conv + LIF through the tensor-core route (3x3/s1 conv into the spike buffer, then the
multi-step LIF in place) against the oracle, the fused gather kernel and the density gate."""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


def _run(x, w, b, v0, tau, vr, decay, policy, masks=False, epilogue=0):
    from sparseflow_b200 import _lib
    from sparseflow_b200.Kernels.fused_conv_lif import sparse_fused_conv_lif_forward, event_masks_of
    with _lib.path_policy(_lib.SF_POLICY_CONV3X3_PATH, policy), _lib.path_policy(_lib.SF_POLICY_LIF_TC_EPILOGUE,
                                                                                 epilogue):
        s, v, _ = sparse_fused_conv_lif_forward(x, v0, w, b, tau, 1.0, vr, decay, kernel_size=3, stride=1,
                                                padding=1, emit_event_masks=masks)
    torch.cuda.synchronize()
    assert _lib.conv_status(x.device) == 0
    return s, v, (event_masks_of(s) if masks else None)


def _masks_of_spikes(s5):
    """Event masks of [T, N, C, H, W] spikes: [T*N][H][W][ceil(C/64)] 64-bit words, bit c % 64 of
    word c // 64 set iff channel c spiked."""
    t, n, c, h, w = s5.shape
    nw = (c + 63) // 64
    bits = np.zeros((t * n, h, w, nw * 64), np.uint64)
    bits[..., :c] = (s5.reshape(t * n, c, h, w).transpose(0, 2, 3, 1) != 0)
    bits = bits.reshape(t * n, h, w, nw, 64)
    return (bits << np.arange(64, dtype=np.uint64)).sum(axis=-1, dtype=np.uint64).reshape(-1)


# t, n, c, co, h, w, density, tau, v_reset, decay
CASES = [
    (4, 2, 32, 48, 12, 12, 0.2, 2.0, 0.0, True),     # resident weights
    (3, 2, 64, 64, 9, 17, 0.05, 1.5, None, True),    # soft reset, non power-of-two tau
    (4, 1, 128, 128, 14, 14, 0.1, 2.0, 0.0, False),  # streamed weights, decay_input off
    (2, 2, 192, 40, 7, 11, 0.3, 4.0, 0.5, True),     # six-pair stages, ragged C_out
]


@pytest.mark.parametrize("t,n,c,co,h,w,density,tau,vr,decay", CASES)
def test_lif_tensor_core_route_vs_oracle_and_gather(t, n, c, co, h, w, density, tau, vr, decay):
    g = torch.Generator().manual_seed(t * 100 + c + co)
    x = (torch.rand(t, n, c, h, w, generator=g) < density).float()
    wt = torch.randn(co, c, 3, 3, generator=g) * (3.0 / (c * 9 * density)) ** 0.5
    b = torch.randn(co, generator=g) * 0.2
    v0 = torch.rand(n, co, h, w, generator=g) * 0.5
    so, near, vo = oracle.conv_lif_near(x.numpy(), wt.numpy(), b.numpy(), v0.numpy(), 1, 1, tau, 1.0, vr, decay)
    assert 0.01 < so.mean() < 0.9
    xs, ws, bs, vs = x.cuda(), wt.cuda(), b.cuda(), v0.cuda()
    s_tc, v_tc, m_tc = _run(xs, ws, bs, vs, tau, vr, decay, 2, masks=True)
    s_ga, v_ga, _ = _run(xs, ws, bs, vs, tau, vr, decay, 1)
    for s, v in ((s_tc, v_tc), (s_ga, v_ga)):
        # Spikes identical except where the membrane is within 1e-5 of v_th.
        assert oracle.spikes_match(s.cpu().numpy(), so, near)
        assert np.abs(v.cpu().numpy() - vo).max() < 1e-4
    assert s_tc.dtype == torch.float32
    np.testing.assert_array_equal(m_tc.cpu().numpy().view(np.uint64), _masks_of_spikes(s_tc.cpu().numpy()))


@pytest.mark.parametrize("c,density,masks,expect", [
    (64, 0.001, False, 1), (64, 0.05, False, 2), (64, 0.001, True, 2),
    (128, 0.002, True, 1), (128, 0.1, True, 2), (128, 0.0025, False, 1), (256, 0.003, False, 1),
    (256, 0.05, True, 2)])
def test_lif_density_gate_picks_one_route(c, density, masks, expect):
    """The sampled nonzero count picks the fused gather kernel or the tensor-core route on the
    device (C_in 64 with event masks always takes the tensor-core route); the automatic result
    (spikes, membrane, masks) equals that route's bit for bit."""
    g = torch.Generator().manual_seed(c + int(density * 1e4))
    x = (torch.rand(4, 4, c, 14, 14, generator=g) < density).float().cuda()
    wt = (torch.randn(c, c, 3, 3, generator=g) * (3.0 / (c * 9 * density)) ** 0.5).cuda()
    b = (torch.randn(c, generator=g) * 0.2).cuda()
    v0 = torch.zeros(4, c, 14, 14, device="cuda")
    auto = _run(x, wt, b, v0, 2.0, 0.0, True, 0, masks=masks)
    forced = _run(x, wt, b, v0, 2.0, 0.0, True, expect, masks=masks)
    for a, f in zip(auto, forced):
        assert (a is None and f is None) or torch.equal(a, f)


def test_lif_tensor_core_route_keeps_16bit_spikes_on_gather():
    """bf16 spikes run the fused gather kernel even when the tensor-core route is forced (the
    route would round the preactivations to bf16); results equal the gather kernel's."""
    g = torch.Generator().manual_seed(5)
    x = (torch.rand(3, 2, 64, 10, 10, generator=g) < 0.2).to(torch.bfloat16).cuda()
    wt = (torch.randn(64, 64, 3, 3, generator=g) * 0.2).cuda()
    v0 = torch.zeros(2, 64, 10, 10, device="cuda")
    a = _run(x, wt, None, v0, 2.0, 0.0, True, 2)
    f = _run(x, wt, None, v0, 2.0, 0.0, True, 1)
    assert torch.equal(a[0], f[0]) and torch.equal(a[1], f[1])


@pytest.mark.parametrize("t,n,c,co,h,w,density,tau,vr,decay", CASES + [
    (5, 3, 128, 128, 28, 28, 0.02, 2.0, 0.0, True),   # C3-like map: three-tile units, tile ring
    (3, 2, 256, 96, 14, 14, 0.05, 3.0, 0.0, False),   # non power-of-two tau (IEEE division)
])
def test_lif_in_tensor_core_epilogue_equals_two_launch_route(t, n, c, co, h, w, density, tau, vr, decay):
    """Without event masks the tensor-core route can run the LIF in the convolution's epilogue
    (one launch; the membrane stays in L2 between steps; forced here by policy). Spikes and
    membrane equal, bit for bit, the route that writes the preactivations and runs the multi-step
    LIF over them, and the spikes follow the oracle's near-threshold rule."""
    g = torch.Generator().manual_seed(t * 7 + c + co)
    x = (torch.rand(t, n, c, h, w, generator=g) < density).float()
    wt = torch.randn(co, c, 3, 3, generator=g) * (3.0 / (c * 9 * density)) ** 0.5
    b = torch.randn(co, generator=g) * 0.2
    v0 = torch.rand(n, co, h, w, generator=g) * 0.5
    xs, ws, bs, vs = x.cuda(), wt.cuda(), b.cuda(), v0.cuda()
    s_f, v_f, _ = _run(xs, ws, bs, vs, tau, vr, decay, 2, epilogue=2)
    s_m, v_m, _ = _run(xs, ws, bs, vs, tau, vr, decay, 2, epilogue=1)
    assert torch.equal(s_f, s_m) and torch.equal(v_f, v_m)
    so, near, vo = oracle.conv_lif_near(x.numpy(), wt.numpy(), b.numpy(), v0.numpy(), 1, 1, tau, 1.0, vr, decay)
    assert 0.01 < so.mean() < 0.9
    assert oracle.spikes_match(s_f.cpu().numpy(), so, near)
    assert np.abs(v_f.cpu().numpy() - vo).max() < 1e-4

