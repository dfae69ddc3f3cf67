"""Drop-in API on the GPU: optimize() a small spiking CNN and compare with the dense model."""
import copy

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


def test_optimize_small_spiking_cnn_matches_dense():
    import sparseflow_b200 as sparseflow
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    from sparseflow_b200.snn import spiking_cnn_small
    from sparseflow_b200.Ops.lif_node import reset_net
    torch.manual_seed(0)
    model = spiking_cnn_small().cuda().eval()
    x = (torch.rand(4, 2, 3, 32, 32, device="cuda") < 0.3).float()
    dense = copy.deepcopy(model)
    sparseflow.optimize(model, sample_input=x, verbose=False, return_ms=True, collect_diag=True)
    n_sparse = sum(isinstance(m, SparseConv2d) for m in model.modules())
    assert n_sparse >= 3
    with torch.no_grad():
        reset_net(dense)
        ref = dense(x)
        reset_net(model)
        out = model(x)
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-4)
    sp = [m for m in model.modules() if isinstance(m, SparseConv2d)]
    assert all(m._last_sparse_ms > 0 for m in sp)
    assert all(m._last_diag.get("sparse_path_executed") for m in sp)


def test_sparse_conv_rejects_cpu_and_bad_rank():
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    m = SparseConv2d(8, 8, 3, 1, 1).cuda()
    with pytest.raises(ValueError):
        m(torch.zeros(8, 8, 8, device="cuda"))
    with pytest.raises(RuntimeError):
        m.cpu()(torch.zeros(1, 8, 8, 8))
