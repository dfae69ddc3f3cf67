"""Multi-step spiking layers and the synthetic spiking models the benchmarks use.

The reference builds its benchmark models with spikingjelly
(Benchmark/bench_4test.py:166-197: ``spiking_resnet*`` with ``LIFNode``,
multi-step mode, kaiming-normal fan_out re-init of convs, BN gamma=1 beta=0).
spikingjelly is not installed here, so this module defines the same topology
with thin multi-step wrappers: every layer takes [T, N, ...] tensors, convs
and BN fold T into the batch (spikingjelly's ``step_mode='m'``), and
``LIFNode`` (Ops/lif_node.py) follows every BN. The wrappers subclass the
torch layers, so ``optimize`` finds and replaces the convs as usual.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn as nn

from .Ops.lif_node import LIFNode


def _fold(x: torch.Tensor):
    return x.flatten(0, 1), x.shape[:2]


class MSConv2d(nn.Conv2d):
    def forward(self, x):
        if x.dim() == 4:
            return super().forward(x)
        y, lead = _fold(x)
        y = super().forward(y)
        return y.reshape(*lead, *y.shape[1:])


class MSBatchNorm2d(nn.BatchNorm2d):
    """BatchNorm over [T, N, C, H, W] (or [N, C, H, W]).

    In eval mode on CUDA it applies the running-statistics affine as one
    elementwise kernel, y = x * scale[c] + shift[c]: cuDNN's inference BN
    kernel is slow on this model's shapes (N*T = 2048 images of 8x8 and
    smaller maps) and took most of a Spiking-ResNet50 forward."""

    _affine_key = None
    _affine = None

    def _scale_shift(self):
        key = (self.weight._version, self.bias._version, self.running_mean._version, self.running_var._version,
               self.weight.device)
        if self._affine_key != key:
            scale = self.weight / torch.sqrt(self.running_var + self.eps)
            shift = self.bias - self.running_mean * scale
            c = scale.numel()
            self._affine = (scale.reshape(c, 1, 1).contiguous(), shift.reshape(c, 1, 1).contiguous())
            self._affine_key = key
        return self._affine

    def forward(self, x):
        if not self.training and x.is_cuda and self.affine and self.track_running_stats:
            scale, shift = self._scale_shift()
            return torch.addcmul(shift, x, scale)
        if x.dim() == 4:
            return super().forward(x)
        y, lead = _fold(x)
        y = super().forward(y)
        return y.reshape(*lead, *y.shape[1:])


class MSMaxPool2d(nn.MaxPool2d):
    def forward(self, x):
        y, lead = _fold(x)
        y = super().forward(y)
        return y.reshape(*lead, *y.shape[1:])


class MSAvgPoolFlatten(nn.Module):
    def forward(self, x):
        return x.mean(dim=(-2, -1))


class MSLinear(nn.Linear):
    pass


class Bottleneck(nn.Module):
    expansion = 4

    def __init__(self, inplanes: int, planes: int, stride: int = 1, downsample: Optional[nn.Module] = None,
                 tau: float = 2.0, v_threshold: float = 1.0):
        super().__init__()
        self.conv1 = MSConv2d(inplanes, planes, 1, bias=False)
        self.bn1 = MSBatchNorm2d(planes)
        self.sn1 = LIFNode(tau=tau, v_threshold=v_threshold)
        self.conv2 = MSConv2d(planes, planes, 3, stride, 1, bias=False)
        self.bn2 = MSBatchNorm2d(planes)
        self.sn2 = LIFNode(tau=tau, v_threshold=v_threshold)
        self.conv3 = MSConv2d(planes, planes * 4, 1, bias=False)
        self.bn3 = MSBatchNorm2d(planes * 4)
        self.downsample = downsample
        self.sn3 = LIFNode(tau=tau, v_threshold=v_threshold)

    def forward(self, x):
        identity = x if self.downsample is None else self.downsample(x)
        out = self.sn1(self.bn1(self.conv1(x)))
        out = self.sn2(self.bn2(self.conv2(out)))
        out = self.bn3(self.conv3(out))
        return self.sn3(out + identity)


class SpikingResNet(nn.Module):
    """Spiking ResNet with the torchvision ImageNet layout (7x7/2 stem + max-pool)."""

    def __init__(self, layers: List[int], num_classes: int = 10, tau: float = 2.0, v_threshold: float = 1.0):
        super().__init__()
        self.inplanes = 64
        self.conv1 = MSConv2d(3, 64, 7, 2, 3, bias=False)
        self.bn1 = MSBatchNorm2d(64)
        self.sn1 = LIFNode(tau=tau, v_threshold=v_threshold)
        self.maxpool = MSMaxPool2d(3, 2, 1)
        kw = dict(tau=tau, v_threshold=v_threshold)
        self.layer1 = self._make_layer(64, layers[0], 1, kw)
        self.layer2 = self._make_layer(128, layers[1], 2, kw)
        self.layer3 = self._make_layer(256, layers[2], 2, kw)
        self.layer4 = self._make_layer(512, layers[3], 2, kw)
        self.avgpool = MSAvgPoolFlatten()
        self.fc = MSLinear(512 * Bottleneck.expansion, num_classes)
        for m in self.modules():
            if isinstance(m, nn.Conv2d):
                nn.init.kaiming_normal_(m.weight, mode="fan_out", nonlinearity="relu")
            elif isinstance(m, nn.BatchNorm2d):
                nn.init.constant_(m.weight, 1)
                nn.init.constant_(m.bias, 0)

    def _make_layer(self, planes, blocks, stride, kw):
        down = None
        if stride != 1 or self.inplanes != planes * 4:
            down = nn.Sequential(MSConv2d(self.inplanes, planes * 4, 1, stride, bias=False),
                                 MSBatchNorm2d(planes * 4))
        layers = [Bottleneck(self.inplanes, planes, stride, down, **kw)]
        self.inplanes = planes * 4
        layers += [Bottleneck(self.inplanes, planes, **kw) for _ in range(1, blocks)]
        return nn.Sequential(*layers)

    def forward(self, x):
        x = self.maxpool(self.sn1(self.bn1(self.conv1(x))))
        x = self.layer4(self.layer3(self.layer2(self.layer1(x))))
        return self.fc(self.avgpool(x)).mean(0)


def spiking_resnet50(num_classes: int = 10, **kw) -> SpikingResNet:
    return SpikingResNet([3, 4, 6, 3], num_classes=num_classes, **kw)


def spiking_cnn_small(num_classes: int = 10) -> nn.Module:
    """A small conv-BN-LIF network used by the API tests (3x3, 3x3/s2 and 1x1 convs)."""
    return nn.Sequential(
        MSConv2d(3, 32, 3, 1, 1, bias=False), MSBatchNorm2d(32), LIFNode(),
        MSConv2d(32, 64, 3, 1, 1), MSBatchNorm2d(64), LIFNode(),
        MSConv2d(64, 64, 3, 2, 1), MSBatchNorm2d(64), LIFNode(),
        MSConv2d(64, 128, 1), MSBatchNorm2d(128), LIFNode(),
        MSAvgPoolFlatten(), MSLinear(128, num_classes),
    )
