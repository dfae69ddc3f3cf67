"""sf_prescan2d_static_ws: the prescan for callers that cannot allocate device memory.

Such callers (a host runtime that owns every device allocation, or a hot path
where cudaMalloc would synchronise the GPU) get the prescan without passing a
workspace: its look-back scratch is a static array inside the library. This
test calls the entry point directly through the C ABI and checks that two
calls in a row give exactly the metadata of the regular sf_prescan2d
(prescan metadata is compared bit-exactly everywhere in this suite). It is
collected last so that a run stopping at the first failure has run the rest.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _desc(n, c, h, w):
    from sparseflow_b200 import _lib
    return _lib.prescan_desc(n, c, h, w, h, w, 3, 1, 1, 8, 16 if h * w >= 3136 else 8, 16, 1e-6, torch.float32,
                             _lib.SF_LAYOUT_NCHW)


def _outputs(n_tiles, dev):
    return [torch.full((n_tiles,), -7, dtype=torch.int32, device=dev) for _ in range(3)] + \
        [torch.full((1,), -7, dtype=torch.int32, device=dev)]


def _regular(x, d, n_tiles):
    from sparseflow_b200 import _lib
    ag, tc, ids, cnt = _outputs(n_tiles, x.device)
    ws = torch.zeros(_lib.prescan_workspace_bytes(d), dtype=torch.uint8, device=x.device)
    _lib.prescan2d(x, d, ag, tc, ids, cnt, ws)
    return ag, tc, ids, cnt


def _static(x, d, n_tiles):
    from sparseflow_b200 import _lib
    ag, tc, ids, cnt = _outputs(n_tiles, x.device)
    lib = _lib.load()
    st = lib.sf_prescan2d_static_ws(x.data_ptr(), ctypes.byref(d), ag.data_ptr(), tc.data_ptr(), ids.data_ptr(),
                                    cnt.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.sf_status_string(st)
    return ag, tc, ids, cnt


def _same(a, b):
    ag, tc, ids, cnt = (t.cpu().numpy() for t in a)
    ag2, tc2, ids2, cnt2 = (t.cpu().numpy() for t in b)
    assert cnt[0] == cnt2[0]
    np.testing.assert_array_equal(ag, ag2)
    np.testing.assert_array_equal(tc, tc2)
    np.testing.assert_array_equal(ids[: cnt[0]], ids2[: cnt2[0]])


def test_static_workspace_prescan_matches_regular_twice():
    g = torch.Generator(device="cuda").manual_seed(99)
    # Two calls in a row with different grids, so the second call reuses the
    # array the first one left behind.
    for (n, c, h, w, p) in [(64, 64, 56, 56, 0.0003), (37, 48, 28, 28, 0.001)]:
        x = (torch.rand(n, c, h, w, device="cuda", generator=g) < p).float()
        d = _desc(n, c, h, w)
        bh, bw = d.block_h, d.block_w
        n_tiles = n * (-(-h // bh)) * (-(-w // bw))
        ref = _regular(x, d, n_tiles)
        first = _static(x, d, n_tiles)
        second = _static(x, d, n_tiles)
        torch.cuda.synchronize()
        _same(ref, first)
        _same(ref, second)
        assert 0 < int(first[3].item()) < n_tiles
    from sparseflow_b200 import _lib
    assert _lib.load().sf_prescan2d_static_ws_status(torch.cuda.current_stream().cuda_stream) == 0


def test_static_workspace_after_other_shapes_with_nan_groups():
    """A third shape after the two above (a different tile-row count), with
    NaN-poisoned channel groups: bit-exact against sf_prescan2d and the oracle,
    and the array's error word reads clear afterwards."""
    from oracle import oracle
    from sparseflow_b200 import _lib
    g = torch.Generator().manual_seed(7)
    for (n, c, h, w, p) in [(64, 64, 56, 56, 0.0003), (19, 40, 30, 30, 0.004)]:
        x = (torch.rand(n, c, h, w, generator=g) < p).float()
        if c == 40:
            x[3, 17, 5, 9] = float("nan")
            x[11, 2, 29, 0] = float("nan")
            x[18, 39, 14, 14] = float("nan")
        xd = x.cuda()
        d = _desc(n, c, h, w)
        bh, bw = d.block_h, d.block_w
        n_tiles = n * (-(-h // bh)) * (-(-w // bw))
        ref = _regular(xd, d, n_tiles)
        got = _static(xd, d, n_tiles)
        torch.cuda.synchronize()
        _same(ref, got)
        assert _lib.load().sf_prescan2d_static_ws_status(torch.cuda.current_stream().cuda_stream) == 0
    oag, otc, oids = oracle.prescan2d(x.numpy(), 0, h, w, 3, 1, 1, bh, bw, 16, 1e-6)
    ag, tc, ids, cnt = (t.cpu().numpy() for t in got)
    np.testing.assert_array_equal(ag, oag)
    np.testing.assert_array_equal(tc, otc)
    np.testing.assert_array_equal(ids[: cnt[0]], oids)


def test_static_workspace_rejects_oversize_request():
    from sparseflow_b200 import _lib
    lib = _lib.load()
    # 32769 tile rows: one more than the static array holds.
    d = _lib.prescan_desc(32769, 16, 8, 8, 8, 8, 3, 1, 1, 8, 8, 16, 1e-6, torch.float32, _lib.SF_LAYOUT_NCHW)
    x = torch.zeros(1, dtype=torch.float32, device="cuda")
    st = lib.sf_prescan2d_static_ws(x.data_ptr(), ctypes.byref(d), x.data_ptr(), x.data_ptr(), None, None, None)
    assert st == _lib.SF_ERR_WORKSPACE
