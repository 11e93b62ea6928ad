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


def _attn_graph(scale):
    """MatMul(q, k^T) / scale -> Softmax -> MatMul(., v), runtime operands."""
    g = Graph(opset=13)
    q = g.add_input("q", [2, 3, 37, 16])
    k = g.add_input("k", [2, 3, 16, 37])
    v = g.add_input("v", [2, 3, 37, 16])
    s = g.op("MatMul", [q, k], name="qk")
    s = g.op("Div", [s, g.const("scale", np.array(scale, np.float32))], name="scaled")
    a = g.op("Softmax", [s], name="sm", axis=-1)
    g.add_output(g.op("MatMul", [a, v], name="av"), None, FLOAT)
    feeds = {n: synth.normal(tuple(d), 1.0, synth.seed_of("attn", n)) for n, d, _ in g.inputs}
    return g, feeds


def _gelu_graph():
    """MatMul + bias + GELU in the ONNX export's erf form, then a second MatMul."""
    g = Graph(opset=13)
    x = g.add_input("x", [2, 50, 64])
    w1 = synth.normal((64, 256), 0.1, synth.seed_of("gelu", "w1"))
    b1 = synth.normal((256,), 0.1, synth.seed_of("gelu", "b1"))
    f = g.op("Add", [g.op("MatMul", [x, g.const("w1", w1)], name="fc1"), g.const("b1", b1)], name="fc1.bias")
    e = g.op("Erf", [g.op("Div", [f, g.const("sqrt2", np.array(np.sqrt(2.0), np.float32))], name="div")],
             name="erf")
    e = g.op("Add", [e, g.const("one", np.array(1.0, np.float32))], name="add1")
    f = g.op("Mul", [g.op("Mul", [f, e], name="mul"), g.const("half", np.array(0.5, np.float32))], name="half")
    w2 = synth.normal((256, 32), 0.1, synth.seed_of("gelu", "w2"))
    g.add_output(g.op("MatMul", [f, g.const("w2", w2)], name="fc2"), None, FLOAT)
    return g, {"x": synth.normal((2, 50, 64), 1.0, synth.seed_of("gelu", "x"))}


@pytest.mark.parametrize("kind", ["gelu", "attn_pow2", "attn_other"])
def test_fused_matmul_epilogues(cuda, kind):
    from nert_b200.model import Model, analyze

    g, ins = _gelu_graph() if kind == "gelu" else _attn_graph(8.0 if kind == "attn_pow2" else 3.0)
    plan = analyze(g, {k: list(v.shape) for k, v in ins.items()})
    groups = {e["name"]: e["group"] for e in plan["exec"]}
    if kind == "gelu":
        assert groups["fc1"] == 7  # MatMul, bias, Div, Erf, Add, Mul, Mul
    else:
        assert groups["qk"] == (2 if kind == "attn_pow2" else 1)
    ref = np_ref.run(g, ins)
    name = g.outputs[0][0]
    for fuse in (True, False):
        m = Model(g, {k: list(v.shape) for k, v in ins.items()}, fuse=fuse)
        try:
            out = m.run(ins)[name]
        finally:
            m.close()
        assert rel_err(out, ref[name]) <= TOL, fuse


def test_split_k_epilogue_matches_oracle(cuda):
    """Few output tiles, long K: the contraction splits K into slices whose
    partial sums are reduced in order before the fused bias + GELU epilogue."""
    from nert_b200.model import Model

    g = Graph(opset=13)
    x = g.add_input("x", [4, 40, 2048])
    w = synth.normal((2048, 96), 0.05, synth.seed_of("splitk", "w"))
    b = synth.normal((96,), 0.1, synth.seed_of("splitk", "b"))
    f = g.op("Add", [g.op("MatMul", [x, g.const("w", w)], name="mm"), g.const("b", b)], name="mm.bias")
    e = g.op("Erf", [g.op("Div", [f, g.const("s2", np.array(np.sqrt(2.0), np.float32))], name="d")], name="erf")
    e = g.op("Add", [e, g.const("one", np.array(1.0, np.float32))], name="a1")
    y = g.op("Mul", [g.op("Mul", [f, e], name="m1"), g.const("h", np.array(0.5, np.float32))], name="m2")
    g.add_output(y, None, FLOAT)
    ins = {"x": synth.normal((4, 40, 2048), 1.0, synth.seed_of("splitk", "x"))}
    ref = np_ref.run(g, ins)[y]
    m = Model(g, {"x": [4, 40, 2048]})
    try:
        out = m.run(ins)[y]
        again = m.run(ins)[y]
        launches = m.stats()["kernels_per_run"]
    finally:
        m.close()
    assert rel_err(out, ref) <= TOL
    np.testing.assert_array_equal(out, again)  # the reduction order is fixed
    assert launches == 2  # contraction + split-K reduce


def _heads_graph(b, t, heads, d, long_k):
    """Attention block with the head split / merge as Reshape + Transpose:
    linear -> [B, T, H, D] -> Transpose to [B, H, T, D] (and [B, H, D, T] for
    K), attention, Transpose back, Reshape, output linear. long_k makes the
    output linear's K long enough to split (its input is the merged heads)."""
    dm = heads * d
    g = Graph(opset=13)
    x = g.add_input("x", [b, t, dm])

    def w(name, shape):
        return g.const(name, synth.normal(shape, 1.0 / np.sqrt(shape[0]), synth.seed_of("heads", name)))

    split = g.const("split", np.array([b, t, heads, d], np.int64))
    merge = g.const("merge", np.array([b, t, dm], np.int64))

    def proj(name, perm):
        y = g.op("Add", [g.op("MatMul", [x, w(name + ".w", (dm, dm))], name=name), w(name + ".b", (dm,))],
                 name=name + ".bias")
        return g.op("Transpose", [g.op("Reshape", [y, split], name=name + ".r")], name=name + ".t", perm=perm)

    q = proj("q", [0, 2, 1, 3])
    k = proj("k", [0, 2, 3, 1])
    v = proj("v", [0, 2, 1, 3])
    s = g.op("Div", [g.op("MatMul", [q, k], name="qk"), g.const("scale", np.array(np.sqrt(d), np.float32))],
             name="scaled")
    a = g.op("Softmax", [s], name="sm", axis=-1)
    c = g.op("Transpose", [g.op("MatMul", [a, v], name="av")], name="ctx.t", perm=[0, 2, 1, 3])
    c = g.op("Reshape", [c, merge], name="ctx")
    g.add_output(g.op("MatMul", [c, w("o.w", (dm, 64 if long_k else dm))], name="o"), None, FLOAT)
    return g, {"x": synth.normal((b, t, dm), 1.0, synth.seed_of("heads", "x"))}


@pytest.mark.parametrize("shape", [(3, 13, 3, 32, False), (2, 197, 12, 64, False), (1, 50, 4, 128, True)],
                         ids=["t13_h3_d32", "vit_heads", "d128_long_k"])
def test_head_transposes_written_in_place(cuda, shape):
    """The projections write [B, H, T, D] / [B, H, D, T] and the attention
    output writes [B, T, H, D] directly (no Transpose rows); results match
    the oracle and the unfused graph."""
    from nert_b200.model import Model, analyze

    g, ins = _heads_graph(*shape)
    plan = analyze(g, {k: list(v.shape) for k, v in ins.items()})
    assert [e["name"] for e in plan["exec"] if e["op"] == "Transpose"] == []
    ref = np_ref.run(g, ins)
    name = g.outputs[0][0]
    for fuse in (True, False):
        m = Model(g, {k: list(v.shape) for k, v in ins.items()}, fuse=fuse)
        try:
            out = m.run(ins)[name]
        finally:
            m.close()
        assert rel_err(out, ref[name]) <= TOL, fuse
