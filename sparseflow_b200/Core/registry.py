"""Spike-source and target-op registry (reference: Core/registry.py:15-109).

The default registry recognises spikingjelly's LIF/IF/ParametricLIF nodes
when spikingjelly is importable, plus this package's own ``LIFNode``.
"""
from __future__ import annotations

from typing import Tuple, Type

import torch.nn as nn

_DEFAULT_SPIKE_OPS = None


def _get_default_spike_ops() -> Tuple[type, ...]:
    global _DEFAULT_SPIKE_OPS
    if _DEFAULT_SPIKE_OPS is None:
        from ..Ops.lif_node import LIFNode
        ops = [LIFNode]
        try:
            from spikingjelly.activation_based import neuron as sj_neuron
            ops += [sj_neuron.LIFNode, sj_neuron.IFNode, sj_neuron.ParametricLIFNode]
        except ImportError:
            pass
        _DEFAULT_SPIKE_OPS = tuple(ops)
    return _DEFAULT_SPIKE_OPS


class SpikeOpRegistry:
    def __init__(self):
        self._spike_op_types: list = []
        self._target_op_types: list = [nn.Conv1d, nn.Conv2d, nn.Conv3d, nn.Linear]

    def register(self, op_type: Type[nn.Module]):
        if op_type not in self._spike_op_types:
            self._spike_op_types.append(op_type)
        return self

    def register_many(self, op_types):
        for t in op_types:
            self.register(t)
        return self

    def register_target(self, op_type: Type[nn.Module]):
        if op_type not in self._target_op_types:
            self._target_op_types.append(op_type)
        return self

    def is_spike_op(self, module: nn.Module) -> bool:
        return bool(self._spike_op_types) and isinstance(module, tuple(self._spike_op_types))

    def is_target_conv1d(self, module: nn.Module) -> bool:
        return isinstance(module, nn.Conv1d)

    def is_target_conv2d(self, module: nn.Module) -> bool:
        return isinstance(module, nn.Conv2d)

    def is_target_conv3d(self, module: nn.Module) -> bool:
        return isinstance(module, nn.Conv3d)

    def is_target_linear(self, module: nn.Module) -> bool:
        return isinstance(module, nn.Linear)

    def is_target_depthwise_conv2d(self, module: nn.Module) -> bool:
        return (isinstance(module, nn.Conv2d) and module.groups == module.in_channels
                and module.out_channels == module.in_channels)

    @property
    def spike_op_types(self) -> Tuple:
        return tuple(self._spike_op_types)

    @property
    def target_op_types(self) -> Tuple:
        return tuple(self._target_op_types)

    @classmethod
    def default(cls) -> "SpikeOpRegistry":
        return cls().register_many(_get_default_spike_ops())
