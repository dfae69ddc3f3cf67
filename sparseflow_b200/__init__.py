"""sparseflow_b200: SparseFlow's spike-sparse convolution path on B200 (sm_100a).

Usage, as with the reference package (reference: __init__.py:16-74)::

    import sparseflow_b200 as sparseflow
    model = sparseflow.optimize(model, sample_input=sample_input)

``optimize`` finds every Conv2d that consumes spikes and swaps it in place
for ``SparseConv2d``, whose forward runs the native kernels in
``libsparseflow_b200.so`` (C ABI: include/sparseflow_b200.h).
"""
from __future__ import annotations

__version__ = "0.3.0"


def optimize(model, sample_input=None, block_sizes=None, verbose=True, threshold=1e-6, return_ms=False,
             collect_diag=False, profile_runtime=False):
    """Replace supported Conv2d layers of a spiking model in place; returns the same model."""
    from .Core.analyzer import NetworkAnalyzer
    from .Core.registry import SpikeOpRegistry
    from .Core.replacer import ModuleReplacer

    analyzer = NetworkAnalyzer(SpikeOpRegistry.default())
    replacer = ModuleReplacer(verbose=verbose)
    targets = analyzer.analyze(model, sample_input=sample_input)
    if verbose:
        print(f"[SparseFlow] Found {len(targets)} replaceable operators")
    replaced, sparse, static_zero, dense_keep = replacer.replace(
        model, targets, block_sizes=block_sizes,
        sparse_kwargs={"threshold": float(threshold), "return_ms": bool(return_ms),
                       "collect_diag": bool(collect_diag), "profile_runtime": bool(profile_runtime)})
    _enable_event_masks(model, targets)
    if verbose:
        print(f"[SparseFlow] Replacement summary: total={replaced}, sparse={sparse}, "
              f"static_zero={static_zero}, dense_keep={dense_keep}")
    return model


def _enable_event_masks(model, targets):
    """Spike sources (this package's LIFNode) of replaced convolutions emit the next layer's event masks,
    where that convolution runs from masks (uses_event_masks: not where a tensor-core kernel reads the
    spikes faster).

    Other spike sources (a spikingjelly neuron, say) have no such switch and are left alone; a source
    whose output is modified before the convolution sees it loses nothing, the masks are then unused.
    """
    import os
    from .Kernels.conv2d import uses_event_masks
    from .Ops.sparse_conv2d import SparseConv2d
    from .Utils.config import EMIT_EVENT_MASKS
    if not EMIT_EVENT_MASKS or os.environ.get("SF_EMIT_EVENT_MASKS", "1") == "0":
        return
    for t in targets:
        try:
            conv = model.get_submodule(t.conv_name)
            src = model.get_submodule(t.spike_name) if t.spike_name else None
        except AttributeError:
            continue
        if isinstance(conv, SparseConv2d) and src is not None and hasattr(src, "emit_event_masks") and \
                uses_event_masks(conv.in_channels, t.input_h, t.input_w, conv.kernel_size[0], conv.stride[0],
                                 conv.padding[0]):
            src.emit_event_masks = True


__all__ = ["optimize", "__version__"]
