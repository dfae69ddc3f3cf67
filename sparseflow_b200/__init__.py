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
    if verbose:
        print(f"[SparseFlow] Replacement summary: total={replaced}, sparse={sparse}, "
              f"static_zero={static_zero}, dense_keep={dense_keep}")
    return model


__all__ = ["optimize", "__version__"]
