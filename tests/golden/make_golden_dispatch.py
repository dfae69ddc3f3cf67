"""Golden decisions of the reference's execution-grounded dispatch (Utils/dispatch_model.py).

    python tests/golden/make_golden_dispatch.py --reference /path/to/SparseFlow

Imports the reference read-only, runs its ``make_dispatch_decision`` on crafted diagnostics /
layer descriptions that reach every gate (near-one saved work, R_min and worst-case guards,
score pass / fail for 3x3 and 1x1, missing diagnostics or metadata, estimated MACs and tile
counts, low confidence, grouped and unknown operators) and its ``dispatch_all_layers`` on target
dicts (exact-zero layers, pools), and writes ``dispatch.json``. The test restates nothing: it
feeds the same inputs to ``sparseflow_b200.Utils.dispatch_model`` and compares.
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "dispatch.json"


def metas():
    m3 = dict(layer_name="l3", op_type="conv", c_in=64, c_out=64, kernel_size=(3, 3), h_in=56, w_in=56,
              h_out=56, w_out=56, batch_size=64, macs=64 * 56 * 56 * 64 * 64 * 9)
    m1 = dict(m3, layer_name="l1", kernel_size=(1, 1), padding=(0, 0), c_in=256, macs=64 * 56 * 56 * 64 * 256)
    small = dict(m3, layer_name="ls", c_in=8, c_out=8, h_in=8, w_in=8, h_out=8, w_out=8, batch_size=1,
                 macs=8 * 8 * 8 * 8 * 9)
    nometa = dict(m3, layer_name="ln", macs=0.0, meta_source="estimated")
    nobatch = dict(m3, layer_name="lb", batch_size=1, macs=56 * 56 * 64 * 64 * 9)
    grouped = dict(m3, layer_name="lg", groups=2)
    unknown = dict(m3, layer_name="lu", op_type="unknown")
    geo = dict(m3, layer_name="lq", meta_source="estimated")
    return m3, m1, small, nometa, nobatch, grouped, unknown, geo


def diag_cases():
    m3, m1, small, nometa, nobatch, grouped, unknown, geo = metas()
    full = lambda a, z, n: {"active_group_ratio": a, "tile_zero_ratio": z, "total_tile_count": n}  # noqa: E731
    return [
        ("near_one", full(0.005, 0.995, 1792), m3),
        ("score_pass_3x3", full(0.4, 0.3, 1792), m3),
        ("r_guard", full(0.9, 0.0, 1792), m3),
        ("r_guard_worst", dict(full(0.5, 0.2, 1792), active_group_ratio_p90=0.9), m3),
        ("score_fail_small", full(0.5, 0.1, 4), small),
        ("score_pass_1x1", full(0.3, 0.2, 1792), m1),
        ("score_fail_1x1_small", full(0.6, 0.0, 1792), dict(m1, c_in=8, c_out=8, macs=64 * 56 * 56 * 8 * 8)),
        ("missing_diag", {}, m3),
        ("missing_tzr_from_counts", {"active_group_ratio": 0.4, "tile_zero_count": 500, "total_tile_count": 1792}, m3),
        ("agr_from_group_counts", {"nonzero_group_count": 300, "total_group_count": 1000, "tile_zero_ratio": 0.2,
                                   "total_tile_count": 1792}, m3),
        ("tiles_from_geometry", {"active_group_ratio": 0.4, "tile_zero_ratio": 0.3}, geo),
        ("macs_estimated", dict(full(0.4, 0.3, 1792), block_m=128), nometa),
        ("batch_from_tiles", dict(full(0.4, 0.3, 1792), block_m=128), nobatch),
        ("grouped", full(0.4, 0.3, 1792), grouped),
        ("unknown_op", full(0.4, 0.3, 1792), unknown),
        ("low_confidence", {"active_group_ratio": 0.9, "tile_zero_ratio": 0.3}, geo),
        ("mix_ratios", dict(full(0.4, 0.3, 1792), denseish_tiles=100, sparse_tiles=1154), m3),
    ]


def target_cases():
    return {
        "targets": [
            {"name": "a", "op_type": "conv", "cin": 64, "cout": 64, "kernel_size": (3, 3), "input_h": 32,
             "input_w": 32, "batch_size": 8},
            {"name": "b", "op_type": "conv", "cin": 64, "cout": 128, "kernel_size": (1, 1), "padding": (0, 0),
             "input_h": 16, "input_w": 16},
            {"name": "z", "op_type": "conv", "cin": 64, "cout": 64, "input_h": 32, "input_w": 32},
            {"name": "p", "op_type": "maxpool2d"},
            {"conv_name": "c", "op_type": "conv", "cin": 32, "cout": 32, "input_h": 28, "input_w": 28,
             "input_shape": (4, 2, 32, 28, 28)},
        ],
        "diags": {"a": {"active_group_ratio": 0.2, "tile_zero_ratio": 0.5, "total_tile_count": 128},
                  "b": {"active_group_ratio": 0.8, "tile_zero_ratio": 0.1, "total_tile_count": 32},
                  "c": {"active_group_ratio": 0.3, "tile_zero_ratio": 0.4, "total_tile_count": 104}},
        "zero_layers": ["z"],
    }


def clean(d):
    return {k: (None if isinstance(v, float) and math.isinf(v) else v) for k, v in d.items()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from Utils import dispatch_model as ref
    cases = []
    for name, diag, meta in diag_cases():
        dec = ref.make_dispatch_decision(diag, ref.ConvMeta(**meta))
        cases.append({"name": name, "diag": diag, "meta": meta, "decision": clean(dec.to_dict())})
    tc = target_cases()
    decs = ref.dispatch_all_layers(tc["targets"], tc["diags"], set(tc["zero_layers"]))
    zs, sp = ref.decisions_to_sets(decs)
    tc["decisions"] = {k: clean(v.to_dict()) for k, v in decs.items()}
    tc["sets"] = {"staticzero": sorted(zs), "sparse": sorted(sp)}
    OUT.write_text(json.dumps({"decision_cases": cases, "dispatch_all": tc}, indent=1, default=list))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
