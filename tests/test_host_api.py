"""Host-side logic of the drop-in API (CPU only; no kernel is launched)."""
import re
from pathlib import Path

import pytest
import torch
import torch.nn as nn

ROOT = Path(__file__).resolve().parent.parent


def test_block_selector_rule():
    from sparseflow_b200.Utils.block_selector import select_block_size, should_replace
    assert [select_block_size(h) for h in (224, 56, 32, 31, 16, 15, 8, 7, 1)] == [16, 16, 16, 8, 8, 4, 4, None, None]
    assert should_replace(8) and not should_replace(7)


def test_group_size_and_tiles_match_reference_rule():
    from sparseflow_b200.Utils.sparse_helpers import choose_group_size, select_tile_sizes
    assert choose_group_size(64) == 16 and choose_group_size(128) == 16
    assert choose_group_size(256) == 32 and choose_group_size(1024) == 32
    assert choose_group_size(1100) == 64 and choose_group_size(2048) == 64
    assert select_tile_sizes(56, 56) == (8, 16) and select_tile_sizes(55, 57) == (8, 8)


def test_popcount_buf():
    from sparseflow_b200.Utils.sparse_helpers import popcount_buf
    m = torch.tensor([0, 1, 3, -1, 0x55555555], dtype=torch.int32)
    assert popcount_buf(m, 5).tolist() == [0, 1, 2, 32, 16]


def test_sparse_conv2d_state_dict_compatible_with_conv2d():
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    conv = nn.Conv2d(16, 32, 3, 1, 1)
    sp = SparseConv2d.from_dense(conv, block_size=8)
    assert set(sp.state_dict()) == set(conv.state_dict())
    assert torch.equal(sp.weight, conv.weight) and torch.equal(sp.bias, conv.bias)
    assert sp.block_size == 8 and "block_size=8" in sp.extra_repr()
    back = nn.Conv2d(16, 32, 3, 1, 1)
    back.load_state_dict(sp.state_dict())


def test_sparse_conv2d_errors_without_cuda():
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    sp = SparseConv2d(8, 8, 3, 1, 1)
    with pytest.raises(ValueError):
        sp(torch.zeros(8, 8, 8))
    with pytest.raises(RuntimeError):  # no silent CPU fallback
        sp(torch.zeros(1, 8, 8, 8))


def test_analyzer_finds_spike_consumers_and_replacer_swaps(capsys):
    import sparseflow_b200 as sparseflow
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    from sparseflow_b200.snn import spiking_cnn_small
    torch.manual_seed(0)
    model = spiking_cnn_small()
    x = (torch.rand(2, 2, 3, 16, 16) < 0.3).float()
    sparseflow.optimize(model, sample_input=x, verbose=True)
    kinds = [type(m).__name__ for m in model.modules()]
    # conv 0 consumes the encoded image (no spike source before it): kept dense.
    assert isinstance(model[0], nn.Conv2d) and not isinstance(model[0], SparseConv2d)
    assert isinstance(model[3], SparseConv2d) and isinstance(model[6], SparseConv2d)
    assert isinstance(model[9], SparseConv2d)
    assert model[3].sf_operator_type == "conv2d_3x3"
    assert model[6].sf_operator_type == "conv2d_3x3_s2"
    assert model[9].sf_operator_type == "conv2d_1x1"
    assert model[3].sf_backend_mode == "sparse" and model[3].block_size == 8
    # the classifier after the (transparent) average pool of the last spikes becomes SparseLinear
    assert type(model[13]).__name__ == "SparseLinear" and model[13].sf_operator_type == "linear"
    out = capsys.readouterr().out
    assert "Replacement summary: total=4, sparse=4" in out
    assert kinds.count("SparseConv2d") == 3


def test_analyzer_small_map_skip_and_block_sizes():
    from sparseflow_b200.Core.analyzer import NetworkAnalyzer
    from sparseflow_b200.Core.registry import SpikeOpRegistry
    from sparseflow_b200.snn import spiking_resnet50
    model = spiking_resnet50().eval()
    x = torch.randn(1, 1, 3, 32, 32)
    targets = NetworkAnalyzer(SpikeOpRegistry.default()).analyze(model, x)
    conv_t = [t for t in targets if t.op_type.startswith("conv2d")]
    names = {t.conv_name for t in conv_t}
    # 32x32 input -> 8x8 at layer1: layer1 and the first layer2 block's inputs only (min-side-7 rule)
    assert "layer1.0.conv1" in names and "layer1.2.conv3" in names
    assert "layer2.0.conv2" in names
    assert not any(n.startswith("layer3") or n.startswith("layer4") for n in names)
    assert all(t.block_size == 4 for t in conv_t if t.input_h == 8)


def test_replacer_static_zero_and_block_override():
    from sparseflow_b200.Core.analyzer import NetworkAnalyzer
    from sparseflow_b200.Core.registry import SpikeOpRegistry
    from sparseflow_b200.Core.replacer import ModuleReplacer, StaticZeroConv2d
    from sparseflow_b200.snn import spiking_cnn_small
    model = spiking_cnn_small()
    x = (torch.rand(2, 2, 3, 16, 16) < 0.3).float()
    targets = NetworkAnalyzer(SpikeOpRegistry.default()).analyze(model, x)
    res = ModuleReplacer(verbose=False).replace(model, targets, block_sizes={"3": 16}, static_zero_layers={"9"})
    assert res == (4, 3, 1, 0)  # the final Linear becomes SparseLinear
    assert model[3].block_size == 16
    assert isinstance(model[9], StaticZeroConv2d)
    y = model[9](torch.zeros(2, 2, 64, 8, 8))
    assert y.shape == (2, 2, 128, 8, 8)
    assert torch.allclose(y[0, 0, :, 0, 0], model[9].bias)


def test_fused_lif_module_validation():
    from sparseflow_b200.Ops.sparse_fused_conv_lif import FusedSparseConvLIF
    with pytest.raises(ValueError):
        FusedSparseConvLIF(8, 8, 5, 1, 2)
    m = FusedSparseConvLIF(8, 8, 3, 1, 1)
    with pytest.raises(ValueError):
        m(torch.zeros(8, 8, 8))


def test_bn_folding_equals_conv_bn():
    from sparseflow_b200.Kernels.fused_conv_lif import fold_bn
    torch.manual_seed(0)
    conv = nn.Conv2d(8, 16, 3, 1, 1)
    bn = nn.BatchNorm2d(16).eval()
    bn.running_mean.uniform_(-1, 1)
    bn.running_var.uniform_(0.5, 1.5)
    bn.weight.data.uniform_(0.5, 1.5)
    w, b = fold_bn(conv.weight, conv.bias, bn)
    x = torch.randn(2, 8, 10, 10)
    ref = bn(conv(x))
    got = nn.functional.conv2d(x, w, b, 1, 1)
    assert torch.allclose(ref, got, atol=1e-5)


def test_native_library_exports_every_declared_symbol():
    """The C ABI in include/*.h is exported by libsparseflow_b200.so (loaded, no kernel launched)."""
    from sparseflow_b200 import _lib
    lib = _lib.load()
    declared = set()
    for h in (ROOT / "include").glob("*.h"):
        declared |= set(re.findall(r"\b(sf_[a-z0-9_]+)\s*\(", h.read_text()))
    assert declared, "no declarations parsed"
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} not exported"
    assert set(_lib.declared_symbols()) == declared
    assert lib.sf_abi_version() == 1
    assert lib.sf_status_string(2) == b"unsupported configuration"


def test_native_argument_checks_without_gpu():
    """Validation paths that return before touching the device."""
    import ctypes
    from sparseflow_b200 import _lib
    lib = _lib.load()
    d = _lib.prescan_desc(2, 64, 32, 32, 32, 32, 3, 1, 1, 8, 8, 16, 1e-6, torch.float32, 0)
    # NCHW: look-back words, 8 bytes of group words per input pixel and one
    # count per tile row, each region rounded to 256 bytes.
    assert lib.sf_prescan2d_workspace_size(ctypes.byref(d)) == 256 + 2 * 32 * 32 * 8 + 256
    d_nhwc = _lib.prescan_desc(2, 64, 32, 32, 32, 32, 3, 1, 1, 8, 8, 16, 1e-6, torch.float32, 1)
    assert lib.sf_prescan2d_workspace_size(ctypes.byref(d_nhwc)) == 16 + 8 * 2 * 4
    bad = _lib.prescan_desc(2, 64, 32, 32, 31, 32, 3, 1, 1, 8, 8, 16, 1e-6, torch.float32, 0)
    assert lib.sf_prescan2d_workspace_size(ctypes.byref(bad)) == 0
    assert lib.sf_prescan2d(None, ctypes.byref(d), None, None, None, None, None, 0, None) == _lib.SF_ERR_INVALID_ARG
    cd = _lib.ConvDesc(1, 8, 8, 8, 8, 8, 8, 5, 1, 2, 0, 0, 0)
    assert lib.sf_sparse_conv2d(16, 16, None, 16, ctypes.byref(cd), 16, 1 << 20, None) == _lib.SF_ERR_UNSUPPORTED
    # gather layout, then (3x3, C_in <= 64) the tensor-core section at the next 256-byte boundary:
    # digit scales [3][64] fp32 and the digit image [9 taps][2 slices of 16 ch][3 * 64 rows][16 B]
    assert lib.sf_packed_weight_bytes(64, 32, 3, 0) == 32 * 9 * 64 * 4 + 3 * 64 * 4 + 9 * 2 * 192 * 16
    assert lib.sf_packed_weight_bytes(64, 256, 1, 0) == 256 * 64 * 4
    # C_in > 64: 32-channel output blocks (N = 96), digit image [4 blocks][9][8 slices][96][16]
    assert lib.sf_packed_weight_bytes(128, 128, 3, 0) == 128 * 9 * 128 * 4 + 3 * 128 * 4 + 4 * 9 * 8 * 96 * 16
    cd = _lib.ConvDesc(2, 64, 56, 56, 64, 56, 56, 3, 1, 1, 0, 0, 1)
    # masks (8 B per pixel), one flag per image (256-byte slot), one sampled-count slot
    assert lib.sf_sparse_conv2d_workspace_size(ctypes.byref(cd)) == 2 * 56 * 56 * 8 + 256 + 256


def test_optimize_turns_on_event_masks_for_sources_of_replaced_convs(monkeypatch):
    """optimize() makes the LIF nodes feeding replaced convolutions emit event masks; the switch
    SF_EMIT_EVENT_MASKS=0 leaves every node as it was."""
    import sparseflow_b200
    from sparseflow_b200.Ops.lif_node import LIFNode
    from sparseflow_b200.Ops.sparse_conv2d import SparseConv2d
    from sparseflow_b200.snn import spiking_resnet50

    def run():
        torch.manual_seed(0)
        m = spiking_resnet50().eval()
        sparseflow_b200.optimize(m, sample_input=torch.randn(2, 2, 3, 32, 32), verbose=False)
        return m

    m = run()
    emitting = {n for n, mod in m.named_modules() if isinstance(mod, LIFNode) and mod.emit_event_masks}
    replaced = {n for n, mod in m.named_modules() if isinstance(mod, SparseConv2d)}
    # sn2 feeds conv3 (1x1 on 8x8 maps: gathered from masks); sn1 feeds conv2 (3x3, C_in 64: the
    # tensor-core kernel reads the spikes themselves), so it does not emit.
    assert "layer1.0.conv2" in replaced and "layer1.0.sn2" in emitting and "layer1.0.sn1" not in emitting
    assert "layer3.0.sn1" not in emitting and "layer4.2.sn3" not in emitting  # their consumers stay dense
    monkeypatch.setenv("SF_EMIT_EVENT_MASKS", "0")
    m2 = run()
    assert not any(isinstance(mod, LIFNode) and mod.emit_event_masks for mod in m2.modules())
