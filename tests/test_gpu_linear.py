"""SparseLinear / sparse_linear_forward (reference Ops/sparse_linear.py, Kernels/linear.py) vs F.linear."""
import numpy as np
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


def _close(y, ref, rtol=1e-5):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 1e-6)
    assert np.abs(y - ref).max() <= rtol * scale


@pytest.mark.parametrize("m,k,n,density", [(256, 2048, 10, 0.02), (37, 130, 300, 0.1), (1, 64, 16, 0.5),
                                           (1024, 512, 512, 0.01)])
def test_sparse_linear_spikes(m, k, n, density):
    from sparseflow_b200.Kernels.linear import sparse_linear_forward
    g = torch.Generator().manual_seed(m + k + n)
    x = (torch.rand(m, k, generator=g) < density).float()
    w = torch.randn(n, k, generator=g) * 0.05
    b = torch.randn(n, generator=g)
    y, _ = sparse_linear_forward(x.cuda(), w.cuda(), b.cuda())
    ref = torch.nn.functional.linear(x.double(), w.double(), b.double())
    _close(y.cpu().numpy(), ref.numpy())


def test_sparse_linear_module_5d_real_values_and_from_dense():
    """Leading [T, N] dims folded; real-valued input (an average pool of spikes) on the exact path."""
    from sparseflow_b200.Ops.sparse_linear import SparseLinear
    g = torch.Generator().manual_seed(3)
    lin = nn.Linear(96, 24)
    sl = SparseLinear.from_dense(lin).cuda()
    assert set(sl.state_dict()) == set(lin.state_dict())
    x = (torch.rand(4, 5, 96, generator=g) < 0.3).float() * torch.rand(4, 5, 96, generator=g)
    y = sl(x.cuda())
    assert y.shape == (4, 5, 24)
    ref = lin(x).detach()
    _close(y.cpu().numpy(), ref.numpy())
    with pytest.raises(ValueError):
        sl(torch.zeros(3, 95, device="cuda"))
