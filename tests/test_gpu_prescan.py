"""Stage-1 prescan on the GPU vs the reference's golden metadata and the CPU oracle (bit-exact)."""
import numpy as np
import pytest
import torch

from conftest import load_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

PRESCAN = load_cases("prescan")


def _run(x, layout, geom, with_ids=True):
    from sparseflow_b200.Kernels._prescan_common import prescan2d
    k, s, p, bh, bw, gs, ho, wo = geom
    n = x.shape[0]
    nt = n * (-(-ho // bh)) * (-(-wo // bw))
    ids = torch.full((nt,), -1, dtype=torch.int32, device=x.device) if with_ids else None
    cnt = torch.zeros(1, dtype=torch.int32, device=x.device) if with_ids else None
    tc, ag, ids, cnt = prescan2d(x, layout, (ho, wo), (k, k), s, p, (bh, bw), gs, 1e-6,
                                 active_ids_out=ids, active_count_out=cnt)
    torch.cuda.synchronize()
    out = (ag.cpu().numpy(), tc.cpu().numpy())
    if with_ids:
        c = int(cnt.item())
        out = out + (ids[:c].cpu().numpy(),)
    return out


@pytest.mark.parametrize("case", sorted(PRESCAN))
@pytest.mark.parametrize("dtype,layout", [(torch.float32, 0), (torch.float16, 0), (torch.float16, 1),
                                          (torch.float32, 1)])
def test_prescan_matches_reference_golden(case, dtype, layout):
    c = PRESCAN[case]
    geom = tuple(int(v) for v in c["geom"])
    x = torch.from_numpy(c["x"]).to("cuda", dtype)
    if layout == 1:
        x = x.permute(0, 2, 3, 1).contiguous()
    ag, tc, ids = _run(x, layout, geom)
    np.testing.assert_array_equal(ag, c["ag_mask"])
    np.testing.assert_array_equal(tc, c["tile_class"])
    np.testing.assert_array_equal(ids, c["active_ids"])


@pytest.mark.parametrize("case", ["c1_p02", "ragged_c40", "threshold_edges", "nan_poison", "dense_vals"])
def test_prescan_bf16_matches_oracle(case):
    c = PRESCAN[case]
    geom = tuple(int(v) for v in c["geom"])
    xb = torch.from_numpy(c["x"]).to(torch.bfloat16)
    ag, tc, ids = _run(xb.cuda(), 0, geom)
    k, s, p, bh, bw, gs, ho, wo = geom
    oag, otc, oids = oracle.prescan2d(xb.float().numpy(), 0, ho, wo, k, s, p, bh, bw, gs, 1e-6)
    np.testing.assert_array_equal(ag, oag)
    np.testing.assert_array_equal(ids, oids)


@pytest.mark.parametrize("n,c,h,w,k,s,p,density", [
    (16, 128, 56, 56, 3, 1, 1, 0.0005),
    (8, 256, 28, 28, 1, 1, 0, 0.0002),
    (6, 96, 30, 22, 3, 2, 1, 0.001),
    (5, 520, 14, 14, 3, 1, 1, 0.00002),
    (64, 64, 7, 7, 3, 1, 1, 0.002),
])
def test_prescan_random_vs_oracle(n, c, h, w, k, s, p, density):
    g = torch.Generator().manual_seed(n * 1000 + c)
    x = (torch.rand(n, c, h, w, generator=g) < density).float()
    ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    bh, bw = oracle.tile_sizes(ho, wo)
    gs = oracle.choose_group_size(c)
    ag, tc, ids = _run(x.cuda(), 0, (k, s, p, bh, bw, gs, ho, wo))
    oag, otc, oids = oracle.prescan2d(x.numpy(), 0, ho, wo, k, s, p, bh, bw, gs, 1e-6)
    np.testing.assert_array_equal(ag, oag)
    np.testing.assert_array_equal(tc, otc)
    np.testing.assert_array_equal(ids, oids)


def test_prescan_workspace_reuse_across_shapes():
    """The look-back workspace self-resets: repeated launches with changing grids stay exact."""
    from sparseflow_b200 import _lib
    from sparseflow_b200.Kernels._prescan_common import prescan_workspace
    g = torch.Generator().manual_seed(7)
    for n in (3, 17, 1, 40, 17, 2):
        x = (torch.rand(n, 64, 32, 32, generator=g) < 0.0004).float()
        ag, tc, ids = _run(x.cuda(), 0, (3, 1, 1, 8, 8, 16, 32, 32))
        oag, otc, oids = oracle.prescan2d(x.numpy(), 0, 32, 32, 3, 1, 1, 8, 8, 16, 1e-6)
        np.testing.assert_array_equal(ag, oag)
        np.testing.assert_array_equal(ids, oids)
    ws = prescan_workspace(torch.device("cuda"), 16)
    assert _lib.prescan_status(ws) == 0


def test_prescan_full_size_properties():
    """C5-cell size (T*N = 1024 images of 64x56x56): count == number of non-ZERO classes,
    ids strictly ascending, class agrees with mask popcount."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.rand(1024, 64, 56, 56, device="cuda", generator=g) < 0.0002).float()
    ag, tc, ids = _run(x, 0, (3, 1, 1, 8, 16, 16, 56, 56))
    assert len(ids) == int((tc != 0).sum())
    assert np.all(np.diff(ids) > 0)
    np.testing.assert_array_equal(tc == 0, ag == 0)
    np.testing.assert_array_equal(tc == 2, ag == 0xF)
    # spot-check two images against the oracle
    for img in (0, 777):
        oag, _, _ = oracle.prescan2d(x[img:img + 1].cpu().numpy(), 0, 56, 56, 3, 1, 1, 8, 16, 16, 1e-6)
        np.testing.assert_array_equal(ag[img * 28:(img + 1) * 28], oag)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("n,c,h,w,k,s,p,bh,bw,gs", [
    (3, 40, 30, 26, 3, 1, 1, 8, 8, 16),      # ragged channels, width not a multiple of the vector
    (2, 64, 56, 56, 3, 2, 1, 8, 16, 16),     # stride 2
    (4, 256, 14, 14, 1, 1, 0, 8, 8, 16),     # 1x1, 16 groups
])
def test_prescan_one_pass_and_two_pass_agree(dtype, n, c, h, w, k, s, p, bh, bw, gs):
    """The full workspace selects the two-pass path (streaming channel fold, then tile
    pooling); a workspace of only the look-back words selects the one-pass kernel.
    Both must give identical metadata, including at the half-precision threshold
    boundary and with NaNs."""
    import ctypes
    from sparseflow_b200 import _lib
    g = torch.Generator().manual_seed(n * 1000 + c)
    x = torch.zeros(n, c, h, w)
    m = torch.rand(n, c, h, w, generator=g)
    edge = torch.tensor([1e-6, 1.0133e-6, 1.0133e-6 * (1 + 2 ** -11), 1.02e-6, 5.96e-8, -2e-6, 0.5, 1.0])
    pick = torch.randint(0, len(edge), (n, c, h, w), generator=g)
    x = torch.where(m < 0.02, edge[pick], x)
    x[0, 0, 0, 0] = float("nan")
    x[-1, c - 1, h // 2, w // 3] = float("nan")
    xd = x.to(dtype).cuda()
    ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    d = _lib.prescan_desc(n, c, h, w, ho, wo, k, s, p, bh, bw, gs, 1e-6, dtype, 0)
    lib = _lib.load()
    nt = n * (-(-ho // bh)) * (-(-wo // bw))
    full = lib.sf_prescan2d_workspace_size(ctypes.byref(d))
    minimal = 16 + 8 * n * (-(-ho // bh))
    assert full > minimal
    outs = []
    for nbytes in (full, minimal):
        ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        ag = torch.empty(nt, dtype=torch.int32, device="cuda")
        tc = torch.empty_like(ag)
        ids = torch.full_like(ag, -1)
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.prescan2d(xd, d, ag, tc, ids, cnt, ws)
        torch.cuda.synchronize()
        assert _lib.prescan_status(ws) == 0
        cn = int(cnt.item())
        outs.append((ag.cpu().numpy(), tc.cpu().numpy(), ids[:cn].cpu().numpy()))
    for a, b in zip(outs[0], outs[1]):
        np.testing.assert_array_equal(a, b)
    oag, otc, oids = oracle.prescan2d(xd.float().cpu().numpy(), 0, ho, wo, k, s, p, bh, bw, gs, 1e-6)
    np.testing.assert_array_equal(outs[0][0], oag)
    np.testing.assert_array_equal(outs[0][2], oids)
