"""Synthetic graphs for the five benchmark configurations.

Each builder returns an :class:`onnx_io.Graph` whose weights come from the
seeded generator in :mod:`synth`, so the reference loader, the numpy oracle
and the B200 engine all see identical bits.

BatchNormalization has no row in the reference (its loader rejects it,
``src/model_loader.cpp:1677-1690``); the reference only ever meets BN folded
into Conv by the exporter. The builders therefore fold BN at construction:
``W' = W * gamma / sqrt(var + eps)``, ``b' = beta - mean * gamma / sqrt(var + eps)``
with gamma=1, beta=0, mean=0, var ~ U[0.5, 1.5], eps=1e-5. The folded bias is
zero but is kept as an explicit Conv bias input.
"""

from __future__ import annotations

import math

import numpy as np

from . import synth
from .onnx_io import FLOAT, Graph


class _Builder:
    def __init__(self, config: str, opset: int = 13):
        self.config = config
        self.g = Graph(name=config, opset=opset)

    def seed(self, name: str) -> int:
        return synth.seed_of(self.config, name)

    def conv_bn(self, x: str, cin: int, cout: int, k: int, stride: int = 1, pad: int = 0,
                name: str = "conv", groups: int = 1) -> str:
        """Conv + folded BatchNorm (Kaiming-normal weights, std sqrt(2/fan_in))."""
        fan_in = (cin // groups) * k * k
        w = synth.normal((cout, cin // groups, k, k), math.sqrt(2.0 / fan_in), self.seed(name + ".w"))
        var = synth.uniform((cout,), 0.5, 1.5, self.seed(name + ".bn_var"))
        scale = (1.0 / np.sqrt(var.astype(np.float64) + 1e-5)).astype(np.float32)
        w = (w * scale[:, None, None, None]).astype(np.float32)
        b = np.zeros((cout,), np.float32)
        wn = self.g.const(name + ".weight", w)
        bn = self.g.const(name + ".bias", b)
        return self.g.op("Conv", [x, wn, bn], name=name, kernel_shape=[k, k], strides=[stride, stride],
                         pads=[pad, pad, pad, pad], dilations=[1, 1], group=groups)

    def relu(self, x: str, name: str) -> str:
        return self.g.op("Relu", [x], name=name)


def resnet18(batch: int = 1, config: str = "resnet18") -> Graph:
    """torchvision-style ResNet-18 (BasicBlock 2/2/2/2, widths 64-512)."""
    return _resnet(batch, config, bottleneck=False, blocks=(2, 2, 2, 2))


def resnet50(batch: int = 1, config: str = "resnet50", softmax: bool = True) -> Graph:
    """torchvision-style ResNet-50 (Bottleneck 3/4/6/3, widths 64-2048) + Softmax."""
    return _resnet(batch, config, bottleneck=True, blocks=(3, 4, 6, 3), softmax=softmax)


def _resnet(batch: int, config: str, bottleneck: bool, blocks, softmax: bool = False) -> Graph:
    b = _Builder(config)
    g = b.g
    x = g.add_input("input", [batch, 3, 224, 224])
    y = b.relu(b.conv_bn(x, 3, 64, 7, 2, 3, name="conv1"), "relu1")
    y = g.op("MaxPool", [y], name="maxpool", kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])
    cin = 64
    widths = (64, 128, 256, 512)
    expansion = 4 if bottleneck else 1
    for li, (nblk, width) in enumerate(zip(blocks, widths)):
        for bi in range(nblk):
            stride = 2 if (li > 0 and bi == 0) else 1
            pre = f"layer{li + 1}.{bi}"
            cout = width * expansion
            if bottleneck:
                t = b.relu(b.conv_bn(y, cin, width, 1, 1, 0, name=pre + ".conv1"), pre + ".relu1")
                t = b.relu(b.conv_bn(t, width, width, 3, stride, 1, name=pre + ".conv2"), pre + ".relu2")
                t = b.conv_bn(t, width, cout, 1, 1, 0, name=pre + ".conv3")
            else:
                t = b.relu(b.conv_bn(y, cin, width, 3, stride, 1, name=pre + ".conv1"), pre + ".relu1")
                t = b.conv_bn(t, width, cout, 3, 1, 1, name=pre + ".conv2")
            if stride != 1 or cin != cout:
                sc = b.conv_bn(y, cin, cout, 1, stride, 0, name=pre + ".downsample")
            else:
                sc = y
            y = g.op("Add", [t, sc], name=pre + ".add")
            y = b.relu(y, pre + ".relu_out")
            cin = cout
    y = g.op("GlobalAveragePool", [y], name="avgpool")
    y = g.op("Flatten", [y], name="flatten", axis=1)
    wfc = synth.normal((1000, cin), math.sqrt(2.0 / cin), b.seed("fc.w"))
    bound = 1.0 / math.sqrt(cin)
    bfc = synth.uniform((1000,), -bound, bound, b.seed("fc.b"))
    y = g.op("Gemm", [y, g.const("fc.weight", wfc), g.const("fc.bias", bfc)], name="fc", transB=1)
    if softmax:
        y = g.op("Softmax", [y], name="softmax", axis=-1)
    g.add_output(y, None, FLOAT)
    return g


def resnet_input(batch: int, config: str = "resnet18") -> np.ndarray:
    """The seeded U[-1, 1] input image batch for the ResNet configs."""
    return synth.uniform((batch, 3, 224, 224), -1.0, 1.0, synth.seed_of(config, "input"))
