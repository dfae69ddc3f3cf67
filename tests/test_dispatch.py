"""Execution-grounded dispatch against the reference's own decisions (tests/golden/dispatch.json,
made by tests/golden/make_golden_dispatch.py from Utils/dispatch_model.py of the reference)."""
import json
import math
from pathlib import Path

import pytest
import torch
import torch.nn as nn

from sparseflow_b200.Utils import dispatch_model as dm

GOLD = json.loads((Path(__file__).parent / "golden" / "dispatch.json").read_text())


def _same(a, b):
    if b is None:  # inf in the fixture
        return isinstance(a, float) and math.isinf(a)
    if isinstance(b, float) or isinstance(a, float):
        return math.isclose(float(a), float(b), rel_tol=1e-12, abs_tol=1e-12)
    if isinstance(b, list):
        return list(a) == b
    return a == b


def _check(mine: dict, want: dict):
    for k, v in want.items():
        assert k in mine, k
        assert _same(mine[k], v), (k, mine[k], v)


@pytest.mark.parametrize("case", GOLD["decision_cases"], ids=lambda c: c["name"])
def test_decision_matches_reference(case):
    meta = dict(case["meta"])
    for k in ("kernel_size", "stride", "padding", "dilation"):
        if k in meta:
            meta[k] = tuple(meta[k])
    dec = dm.make_dispatch_decision(case["diag"], dm.ConvMeta(**meta))
    _check(dec.to_dict(), case["decision"])


def test_dispatch_all_layers_matches_reference():
    g = GOLD["dispatch_all"]
    targets = [{k: (tuple(v) if isinstance(v, list) else v) for k, v in t.items()} for t in g["targets"]]
    decs = dm.dispatch_all_layers(targets, g["diags"], set(g["zero_layers"]))
    assert sorted(decs) == sorted(g["decisions"])
    for name, want in g["decisions"].items():
        _check(decs[name].to_dict(), want)
    zs, sp = dm.decisions_to_sets(decs)
    assert sorted(zs) == g["sets"]["staticzero"] and sorted(sp) == g["sets"]["sparse"]


def test_meta_from_analyzer_target_and_apply_dispatch():
    """A ReplacementTarget-shaped record gives conv metadata; apply_dispatch routes dense layers to cuDNN."""
    from sparseflow_b200.Core.analyzer import ReplacementTarget
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    conv = nn.Conv2d(16, 32, 3, 1, 1)
    t = ReplacementTarget(conv_name="body.conv", conv_module=conv, spike_name="body.lif", op_type="conv",
                          input_h=20, input_w=20)
    meta = dm.op_meta_from_target(t)
    assert (meta.c_in, meta.c_out, meta.h_out, meta.w_out, meta.batch_size) == (16, 32, 20, 20, 1)
    assert meta.meta_source == "estimated" and meta.macs == 20 * 20 * 32 * 16 * 9

    model = nn.Sequential()
    model.add_module("body", nn.Sequential())
    model.body.add_module("conv", SparseConv2d.from_dense(conv))
    model.body.add_module("conv2", SparseConv2d.from_dense(nn.Conv2d(32, 32, 3, 1, 1)))
    decs = {"body.conv": dm.DispatchDecision(layer_name="body.conv", backend="dense"),
            "body.conv2": dm.DispatchDecision(layer_name="body.conv2", backend="sparse")}
    assert dm.apply_dispatch(model, decs) == 1
    assert model.body.conv.dispatch_backend == "dense" and model.body.conv2.dispatch_backend == "sparse"
