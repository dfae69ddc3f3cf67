"""Which modules count as spike sources for the analyzer.

Public surface kept from the reference (Core/registry.py:15-109):
``SpikeOpRegistry.default()``, ``register`` and ``is_spike_op``. This build
replaces only 3x3 / 1x1 Conv2d layers fed by a spike source, so the registry
holds spike-source types and nothing else; the analyzer decides which
convolutions qualify.
"""
from __future__ import annotations

import functools
from typing import Iterable, Tuple, Type

import torch.nn as nn


@functools.lru_cache(maxsize=1)
def _known_spike_sources() -> Tuple[type, ...]:
    """This package's LIFNode, plus spikingjelly's neuron classes when that
    package is importable (it is an optional dependency)."""
    from ..Ops.lif_node import LIFNode
    found = [LIFNode]
    try:
        from spikingjelly.activation_based import neuron
    except ImportError:
        return tuple(found)
    for name in ("LIFNode", "IFNode", "ParametricLIFNode"):
        cls = getattr(neuron, name, None)
        if isinstance(cls, type):
            found.append(cls)
    return tuple(found)


class SpikeOpRegistry:
    """An ordered set of module types whose outputs are spikes."""

    def __init__(self, spike_types: Iterable[Type[nn.Module]] = ()):
        self._types: Tuple[type, ...] = ()
        for t in spike_types:
            self.register(t)

    def register(self, op_type: Type[nn.Module]) -> "SpikeOpRegistry":
        if op_type not in self._types:
            self._types = self._types + (op_type,)
        return self

    def is_spike_op(self, module) -> bool:
        return bool(self._types) and isinstance(module, self._types)

    @property
    def spike_op_types(self) -> Tuple[type, ...]:
        return self._types

    @classmethod
    def default(cls) -> "SpikeOpRegistry":
        return cls(_known_spike_sources())
