"""Dispatch end to end on the GPU: diagnostics from the prescan, decisions, dense layers put back."""
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


def _model():
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    g = torch.Generator().manual_seed(0)
    c1, c2 = nn.Conv2d(64, 64, 3, 1, 1), nn.Conv2d(64, 64, 3, 1, 1)
    for c in (c1, c2):
        c.weight.data = torch.randn(64, 64, 3, 3, generator=g) * 0.05
    m = nn.Module()
    m.sparse_in = SparseConv2d.from_dense(c1).cuda()
    m.dense_in = SparseConv2d.from_dense(c2).cuda()
    return m


class _Two(nn.Module):
    """Feeds very sparse spikes to one layer and all-ones to the other."""

    def __init__(self, m):
        super().__init__()
        self.sparse_in, self.dense_in = m.sparse_in, m.dense_in

    def forward(self, x):
        return self.sparse_in(x) + self.dense_in(torch.ones_like(x))


def test_collect_decide_apply():
    from sparseflow_b200.Utils import dispatch_model as dm
    model = _Two(_model())
    x = torch.zeros(2, 4, 64, 32, 32, device="cuda")
    x[0, 0, 3, 5, 7] = 1.0
    x[1, 2, 40, 20, 9] = 1.0
    diags = dm.collect_layer_diags(model, x)
    assert set(diags) == {"sparse_in", "dense_in"}
    assert diags["sparse_in"]["tile_zero_ratio"] > 0.9 and diags["dense_in"]["tile_zero_ratio"] == 0.0
    targets = [{"name": n, "module": getattr(model, n), "op_type": "conv", "input_shape": tuple(x.shape)}
               for n in ("sparse_in", "dense_in")]
    decs = dm.dispatch_all_layers(targets, diags)
    assert decs["sparse_in"].backend == "sparse" and decs["sparse_in"].reason_code == "R_near_one"
    assert decs["dense_in"].backend == "dense" and decs["dense_in"].reason_code == "R_guard"
    tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False  # compare the sparse path with fp32 cuDNN
    try:
        _apply_and_compare(dm, model, x, decs)
    finally:
        torch.backends.cudnn.allow_tf32 = tf32


def _apply_and_compare(dm, model, x, decs):
    with torch.no_grad():
        y_before = model(x)
        assert dm.apply_dispatch(model, decs) == 1
        assert model.dense_in.dispatch_backend == "dense"
        y_after = model(x)
        assert model.dense_in.fallback_reason == "dispatch_dense"
    torch.testing.assert_close(y_after, y_before, rtol=1e-5, atol=1e-4)
