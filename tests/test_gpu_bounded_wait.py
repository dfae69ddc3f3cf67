"""Device-side failure detection: a wait that can never complete gives up within its limit,
reports SF_ERR_DEVICE_TIMEOUT, and leaves the context usable (no fault, trap or hang)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_context_survives():
    from sparseflow_b200 import _lib
    from sparseflow_b200.Kernels.conv2d import sparse_conv2d_forward
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.monotonic()
    st = lib.sf_selftest_bounded_wait(200_000_000, stream)  # 0.2 s limit
    elapsed = time.monotonic() - t0
    assert st == _lib.SF_ERR_DEVICE_TIMEOUT
    assert 0.15 < elapsed < 10.0
    # The context is intact: a convolution still runs and is right.
    x = (torch.rand(2, 16, 9, 9) < 0.2).float()
    w = torch.randn(8, 16, 3, 3)
    y, _ = sparse_conv2d_forward(x.cuda(), w.cuda(), None, kernel_size=3, stride=1, padding=1)
    ref = torch.nn.functional.conv2d(x.double(), w.double(), padding=1)
    assert (y.double().cpu() - ref).abs().max() < 1e-4
    assert _lib.conv_status(torch.device("cuda")) == 0
