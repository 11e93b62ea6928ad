"""The engine's epilogue fusion, group by group, against the oracle and
against the same graph run unfused (every node its own row)."""

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import synth
from nert_b200.onnx_io import FLOAT, Graph
from oracle import np_ref

pytestmark = pytest.mark.gpu


def _conv(g, x, cin, cout, k, s, p, name):
    w = synth.normal((cout, cin, k, k), (2.0 / (cin * k * k)) ** 0.5, synth.seed_of("fusion", name + ".w"))
    b = synth.normal((cout,), 0.1, synth.seed_of("fusion", name + ".b"))
    return g.op("Conv", [x, g.const(name + ".w", w), g.const(name + ".b", b)], name=name, kernel_shape=[k, k],
                strides=[s, s], pads=[p] * 4)


def build(kind):
    g = Graph(opset=13)
    x = g.add_input("x", [2, 64, 20, 20])
    if kind == "conv_relu":
        y = g.op("Relu", [_conv(g, x, 64, 64, 3, 1, 1, "c")], name="r")
    elif kind == "conv_add":
        r = g.add_input("r", [2, 64, 20, 20])
        y = g.op("Add", [_conv(g, x, 64, 64, 3, 1, 1, "c"), r], name="a")
    elif kind == "conv_add_relu":
        r = g.add_input("r", [2, 64, 20, 20])
        y = g.op("Relu", [g.op("Add", [r, _conv(g, x, 64, 64, 3, 1, 1, "c")], name="a")], name="rl")
    elif kind == "conv_silu":
        c = _conv(g, x, 64, 32, 1, 1, 0, "c")
        y = g.op("Mul", [c, g.op("Sigmoid", [c], name="s")], name="m")
    elif kind == "basic_block":
        t = g.op("Relu", [_conv(g, x, 64, 64, 3, 1, 1, "c1")], name="r1")
        t = _conv(g, t, 64, 64, 3, 1, 1, "c2")
        y = g.op("Relu", [g.op("Add", [t, x], name="a")], name="r2")
    elif kind == "down_block":
        t = g.op("Relu", [_conv(g, x, 64, 128, 3, 2, 1, "c1")], name="r1")
        t = _conv(g, t, 128, 128, 3, 1, 1, "c2")
        d = _conv(g, x, 64, 128, 1, 2, 0, "ds")
        y = g.op("Relu", [g.op("Add", [t, d], name="a")], name="r2")
    g.add_output(y, None, FLOAT)
    return g


@pytest.mark.parametrize("kind", ["conv_relu", "conv_add", "conv_add_relu", "conv_silu", "basic_block", "down_block"])
def test_fused_group(cuda, kind):
    from nert_b200.model import Model

    g = build(kind)
    ins = {"x": synth.normal((2, 64, 20, 20), 1.0, 1)}
    if any(n == "r" for n, _, _ in g.inputs):
        ins["r"] = synth.normal((2, 64, 20, 20), 1.0, 2)
    ref = np_ref.run(g, ins)
    name = g.outputs[0][0]
    outs = {}
    for fuse in (True, False):
        m = Model(g, {k: list(v.shape) for k, v in ins.items()}, fuse=fuse, cuda_graph=False)
        try:
            outs[fuse] = m.run(ins)[name]
            if fuse:
                assert m.stats()["fused_groups"] >= 1
        finally:
            m.close()
    assert rel_err(outs[False], ref[name]) <= TOL, "unfused"
    assert rel_err(outs[True], ref[name]) <= TOL, "fused"
