"""Pin the CPU oracle against golden vectors produced by the reference itself."""
import numpy as np
import pytest

from conftest import load_cases
from oracle import oracle

PRESCAN = load_cases("prescan")
CONV = load_cases("conv")
LIF = load_cases("lif")


@pytest.mark.parametrize("case", sorted(PRESCAN))
def test_prescan_oracle_matches_reference(case):
    c = PRESCAN[case]
    k, s, p, bh, bw, gs, ho, wo = (int(v) for v in c["geom"])
    ag, tc, ids = oracle.prescan2d(c["x"], 0, ho, wo, k, s, p, bh, bw, gs, 1e-6)
    np.testing.assert_array_equal(ag, c["ag_mask"])
    np.testing.assert_array_equal(tc, c["tile_class"])
    np.testing.assert_array_equal(np.sort(ids), np.sort(c["active_ids"]))
    np.testing.assert_array_equal(ids, c["active_ids"])  # ascending, like torch.nonzero


@pytest.mark.parametrize("case", sorted(PRESCAN))
def test_prescan_oracle_nhwc_equals_nchw(case):
    c = PRESCAN[case]
    k, s, p, bh, bw, gs, ho, wo = (int(v) for v in c["geom"])
    ag, tc, ids = oracle.prescan2d(np.ascontiguousarray(c["x"].transpose(0, 2, 3, 1)), 1, ho, wo, k, s, p, bh,
                                   bw, gs, 1e-6)
    np.testing.assert_array_equal(ag, c["ag_mask"])
    np.testing.assert_array_equal(ids, c["active_ids"])


def test_threshold_is_compared_in_half():
    # 17 * 2^-24 (= half(1e-6)) is not above half(1e-6); 18 * 2^-24 is.
    x = np.zeros((1, 16, 8, 8), np.float32)
    x[0, 0, 3, 3] = 17 * 2.0 ** -24
    ag, _, _ = oracle.prescan2d(x, 0, 8, 8, 3, 1, 1, 8, 8, 16, 1e-6)
    assert ag[0] == 0
    x[0, 0, 3, 3] = 18 * 2.0 ** -24
    ag, _, _ = oracle.prescan2d(x, 0, 8, 8, 3, 1, 1, 8, 8, 16, 1e-6)
    assert ag[0] == 1


@pytest.mark.parametrize("case", sorted(CONV))
def test_conv_oracle_matches_reference(case):
    c = CONV[case]
    k, s, p = (int(v) for v in c["geom"])
    x = c["x"]
    x4 = x.reshape(-1, *x.shape[-3:])
    y = oracle.conv2d(x4, c["w"], c.get("b"), s, p).reshape(c["y"].shape)
    np.testing.assert_allclose(y, c["y"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", sorted(LIF))
def test_lif_oracle_matches_reference(case):
    c = LIF[case]
    tau, vth, vr, hard, decay = (float(v) for v in c["params"])
    x = c["x"]
    t, n, ci, h, w = x.shape
    co = c["w"].shape[0]
    sp, near, v = oracle.conv_lif_near(x, c["w"], c.get("b"), np.zeros((n, co, h, w), np.float32), 1, 1, tau,
                                       vth, vr if hard else None, bool(decay))
    # Spikes may only differ where the membrane sits within 1e-5 of threshold.
    assert oracle.spikes_match(sp, c["spikes"], near)
    np.testing.assert_allclose(v, c["v"], rtol=1e-4, atol=1e-4)
