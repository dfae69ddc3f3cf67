"""Standalone multi-step LIF kernel (sf_lif_multistep) vs the PyTorch formula of the same rule."""
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


def _torch_lif(x, v0, tau, vth, v_reset, decay_input):
    from sparseflow_b200.Ops.lif_node import LIFNode
    node = LIFNode(tau=tau, v_threshold=vth, v_reset=v_reset, decay_input=decay_input)
    node.v = v0.clone()
    s = torch.stack([node._step(x[t]) for t in range(x.shape[0])], 0)
    return s, node.v


@pytest.mark.parametrize("v_reset,decay_input", [(0.0, True), (None, True), (0.0, False), (-0.2, True)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_lif_multistep_matches_torch_formula(v_reset, decay_input, dtype):
    from sparseflow_b200 import _lib
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(16, 2, 8, 7, 9, generator=g) * 1.2).to(dtype).cuda()   # numel 1008: vector path
    v0 = (torch.rand(2, 8, 7, 9, generator=g) * 0.5).cuda()
    ref_s, ref_v = _torch_lif(x, v0, 2.0, 1.0, v_reset, decay_input)
    v = v0.clone()
    s = torch.empty_like(x)
    _lib.lif_multistep(x, v, s, 2.0, 1.0, v_reset, decay_input)
    torch.testing.assert_close(s, ref_s, rtol=0, atol=0)
    torch.testing.assert_close(v, ref_v, rtol=0, atol=0)


def test_lif_multistep_odd_numel_and_oracle():
    """Scalar path (numel not a multiple of 4) against the C oracle's LIF step."""
    from sparseflow_b200 import _lib
    g = torch.Generator().manual_seed(4)
    x = torch.randn(5, 3, 5, 7, generator=g).cuda()
    v = torch.zeros(3, 5, 7, device="cuda")
    s = torch.empty_like(x)
    _lib.lif_multistep(x, v, s, 2.0, 1.0, 0.0, True)
    vo = torch.zeros(3 * 5 * 7).numpy()
    for t in range(5):
        so, vo = oracle.lif_step(x[t].cpu().reshape(-1).numpy(), vo, 2.0, 1.0, 0.0, True)
        assert (s[t].cpu().reshape(-1).numpy() == so).all()
    assert abs(v.cpu().reshape(-1).numpy() - vo).max() < 1e-6


def test_lif_node_cuda_multistep_carries_state():
    from sparseflow_b200.Ops.lif_node import LIFNode
    g = torch.Generator().manual_seed(5)
    x = torch.randn(8, 4, 16, generator=g).cuda()
    a, b = LIFNode(), LIFNode()
    y1 = torch.cat([a(x[:3]), a(x[3:])], 0)  # two calls continue from the stored v
    y2 = torch.stack([b._step(x[t]) for t in range(8)], 0)
    torch.testing.assert_close(y1, y2, rtol=0, atol=0)
    torch.testing.assert_close(a.v, b.v, rtol=0, atol=0)
