"""Pinning the oracle (CPU only).

The numpy restatement (oracle/np_ref.py) is checked against
* the known answers of the reference's own tests (tests/golden/known_answers.py);
* the reference library itself (oracle/_ref/libnert_ref.so, compiled from the
  reference sources by oracle/Makefile) on seeded graphs;
and the reference library is checked against the same known answers, so the
two oracles and the golden values agree with one another.
"""

import numpy as np
import pytest

from conftest import rel_err
from golden.known_answers import CASES, CASES2
from helpers import case2_graph, check_outputs
from nert_b200 import configs, onnx_io, synth
from nert_b200.onnx_io import FLOAT, Graph
from oracle import np_ref, ref

needs_ref = pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built (no reference sources here)")


def single_op_graph(op, attrs, in_shapes, opset=13, n_out=1):
    g = Graph(name="single", opset=opset)
    names = [g.add_input(f"in{i}", list(s)) for i, s in enumerate(in_shapes)]
    outs = g.op(op, names, n_out=n_out, name="node", **attrs)
    for o in (outs if isinstance(outs, list) else [outs]):
        g.add_output(o, None, FLOAT)
    return g


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0].split()[1])
def test_np_ref_known_answers(case):
    cite, op, attrs, ins, exp, edims = case
    arrs = [np.array(v, np.float32).reshape(d) for v, d in ins]
    got = np_ref.run_op(op, attrs, arrs)
    assert list(got.shape) == edims, cite
    np.testing.assert_array_equal(got.ravel(), np.array(exp, np.float32), err_msg=cite)


@needs_ref
@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0].split()[1])
def test_reference_library_known_answers(case):
    cite, op, attrs, ins, exp, edims = case
    arrs = [np.array(v, np.float32).reshape(d) for v, d in ins]
    g = single_op_graph(op, attrs, [a.shape for a in arrs])
    out = ref.run_graph(g, {f"in{i}": a for i, a in enumerate(arrs)})
    got = list(out.values())[0]
    assert list(got.shape) == edims, cite
    np.testing.assert_array_equal(got.ravel(), np.array(exp, np.float32), err_msg=cite)


@pytest.mark.parametrize("case", CASES2, ids=lambda c: c[0].split()[1] + ("_" + c[1] if "(" in c[0] else ""))
def test_np_ref_known_answers_2(case):
    g, feeds, expected = case2_graph(case)
    check_outputs(np_ref.run(g, feeds), expected, case[5], case[0])


@needs_ref
@pytest.mark.parametrize("case", CASES2, ids=lambda c: c[0].split()[1] + ("_" + c[1] if "(" in c[0] else ""))
def test_reference_library_known_answers_2(case):
    g, feeds, expected = case2_graph(case)
    check_outputs(ref.run_graph(g, feeds), expected, case[5], case[0])


@needs_ref
def test_np_ref_matches_reference_resnet18():
    g = configs.resnet18(1)
    x = configs.resnet_input(1)
    a = np_ref.run(g, {"input": x})["fc_out"]
    b = ref.run_graph(g, {"input": x})["fc_out"]
    # float64 accumulation in both; only the summation order differs
    assert np.abs(a - b).max() <= 1e-6 * np.abs(b).max()


RANDOM_CASES = [
    ("Conv", {"strides": [2, 2], "pads": [1, 0, 2, 1], "dilations": [1, 2], "group": 2}, [(2, 4, 9, 11), (6, 2, 3, 3),
                                                                                      (6,)]),
    ("Conv", {"pads": [3, 3, 3, 3], "strides": [2, 2]}, [(1, 3, 20, 20), (8, 3, 7, 7)]),
    ("Gemm", {"transA": 1, "transB": 1, "alpha": 0.5, "beta": 2.0}, [(7, 5), (9, 7), (5, 9)]),
    ("MatMul", {}, [(2, 3, 5, 4), (2, 3, 4, 6)]),
    ("MaxPool", {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1], "ceil_mode": 1}, [(1, 2, 10, 9)]),
    ("MaxPool", {"kernel_shape": [5, 5], "strides": [1, 1], "pads": [2, 2, 2, 2]}, [(1, 3, 8, 8)]),
    ("GlobalAveragePool", {}, [(2, 3, 7, 7)]),
    ("Softmax", {"axis": -1}, [(3, 4, 17)]),
    ("Softmax", {"axis": 1}, [(2, 16, 5)]),
    ("Sigmoid", {}, [(4, 33)]),
    ("Add", {}, [(2, 3, 4), (3, 1)]),
    ("Div", {}, [(2, 5), (5,)]),
]


@needs_ref
@pytest.mark.parametrize("case", RANDOM_CASES, ids=lambda c: c[0] + "_" + "x".join(map(str, c[2][0])))
def test_np_ref_matches_reference_random(case):
    op, attrs, shapes = case
    arrs = [synth.normal(s, 1.0, synth.seed_of("oracle", f"{op}{i}{s}")) for i, s in enumerate(shapes)]
    if op == "Div":
        arrs[1] = arrs[1] + np.float32(3.0)
    g = single_op_graph(op, attrs, shapes)
    b = list(ref.run_graph(g, {f"in{i}": a for i, a in enumerate(arrs)}).values())[0]
    a = np_ref.run_op(op, attrs, arrs)
    assert a.shape == b.shape
    assert np.abs(a.astype(np.float64) - b).max() <= 1e-6 * max(1.0, np.abs(b).max())


def test_synth_is_pinned():
    """The generator must give the same bits on every host (GPU box included)."""
    assert synth.seed_of("resnet18", "input") == 0xC0C0D5BDA8973F9A
    u = synth.uniform((4,), -1.0, 1.0, 12345)
    n = synth.normal((3,), 1.0, 12345)
    np.testing.assert_array_equal(u, np.array([-0.7338407039642334, -0.5903668403625488, -0.7609149217605591,
                                               -0.6477644443511963], np.float32))
    np.testing.assert_allclose(n, np.array([1.1712841987609863, -1.6346750259399414, -2.0264062881469727],
                                           np.float32), rtol=2e-7)
    assert u.dtype == np.float32 and n.dtype == np.float32
    # 2**-24 lattice: every uniform value is exactly representable
    v = (synth.uniform((1000,), 0.0, 1.0, 7).astype(np.float64) * (1 << 24))
    np.testing.assert_array_equal(v, np.round(v))


def test_onnx_roundtrip():
    g = configs.resnet18(1)
    b = onnx_io.to_onnx_bytes(g)
    g2 = onnx_io.from_onnx_bytes(b)
    assert [n.op_type for n in g2.nodes] == [n.op_type for n in g.nodes]
    assert g2.nodes[0].attrs == g.nodes[0].attrs
    for k, v in g.initializers.items():
        np.testing.assert_array_equal(g2.initializers[k], v)
    assert onnx_io.to_onnx_bytes(g2) == b


@pytest.mark.parametrize("config", ["resnet18", "resnet50", "vit_b16", "yolov8n"])
def test_np_ref_matches_bench_config_fixtures(config):
    """The numpy restatement reproduces the reference library's golden
    outputs on the pinned images of each benchmarked batch."""
    import os
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_model_fixtures as mmf

    z = np.load(os.path.join(mmf.OUT, f"{config}.npz"))
    batch = int(z["batch"])
    g, name, x = mmf.graph_and_input(config, batch)
    for i in mmf.images(batch):
        got = np_ref.run(g, {name: x[i:i + 1]})
        for out_name in {k.rsplit("/", 1)[0] for k in z.files if "/" in k}:
            want = z[f"{out_name}/{i}"]
            have = mmf.subsample(config, out_name, got[out_name])
            if want.dtype == np.int64:
                np.testing.assert_array_equal(have, want, err_msg=f"{config} {out_name} {i}")
            else:
                assert rel_err(have, want) <= 1e-5, (config, out_name, i)


AVGPOOL_CASES = [
    ({"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]}, (2, 3, 17, 19)),
    ({"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1], "count_include_pad": 1}, (2, 3, 17, 19)),
    ({"kernel_shape": [2, 3], "strides": [2, 1], "pads": [0, 1, 1, 0], "ceil_mode": 1}, (1, 4, 9, 10)),
    ({"kernel_shape": [5, 5], "strides": [3, 3], "auto_pad": "SAME_UPPER"}, (1, 2, 14, 13)),
    ({"kernel_shape": [2, 2], "strides": [2, 2]}, (3, 8, 8, 8)),
]


@needs_ref
@pytest.mark.parametrize("case", AVGPOOL_CASES, ids=lambda c: "_".join(f"{k}{v}" for k, v in c[0].items()))
def test_np_ref_average_pool_bit_exact_with_reference(case):
    """AveragePool sums in float32 in the reference's order: bit-exact."""
    attrs, shape = case
    x = synth.normal(shape, 1.0, synth.seed_of("oracle_avgpool", str(case)))
    g = single_op_graph("AveragePool", attrs, [shape])
    want = list(ref.run_graph(g, {"in0": x}).values())[0]
    np.testing.assert_array_equal(np_ref.run_op("AveragePool", attrs, [x]), want)


CONVT_CASES = [
    ({"strides": [2, 2], "pads": [1, 1, 1, 1], "output_padding": [1, 1]}, (2, 8, 7, 9), (8, 6, 3, 3)),
    ({"strides": [2, 2]}, (1, 16, 10, 10), (16, 8, 2, 2)),
    ({"strides": [1, 2], "pads": [0, 1, 2, 0], "dilations": [2, 1]}, (1, 6, 5, 6), (6, 4, 3, 3)),
    ({"strides": [3, 3], "group": 2, "pads": [1, 1, 1, 1]}, (1, 8, 4, 5), (8, 3, 4, 4)),
]


@needs_ref
@pytest.mark.parametrize("case", CONVT_CASES, ids=lambda c: "_".join(f"{k}{v}" for k, v in c[0].items()))
def test_np_ref_conv_transpose_matches_reference(case):
    attrs, xs, ws = case
    x = synth.normal(xs, 1.0, synth.seed_of("oracle_convt", str(case) + "x"))
    w = synth.normal(ws, 0.3, synth.seed_of("oracle_convt", str(case) + "w"))
    b = synth.normal((ws[1] * attrs.get("group", 1),), 1.0, synth.seed_of("oracle_convt", str(case) + "b"))
    g = Graph(opset=13)
    g.add_input("x", list(xs))
    y = g.op("ConvTranspose", ["x", g.const("w", w), g.const("b", b)], name="ct", **attrs)
    g.add_output(y, None, FLOAT)
    want = list(ref.run_graph(g, {"x": x}).values())[0]
    got = np_ref.run(g, {"x": x})[y]
    assert got.shape == want.shape
    assert np.abs(got.astype(np.float64) - want).max() <= 1e-5 * np.abs(want).max()


def _movement_graph(kind):
    """Seeded single-node graphs for the rows the random cases above leave
    out: normalisation, the data-movement rows (with their constant
    operands) and the int64-producing TopK. Returns (graph, feed)."""
    from nert_b200.onnx_io import INT64

    seed = synth.seed_of("oracle_moves", kind)
    g = Graph(name=kind, opset=17 if kind == "layernorm" else 13)
    x4 = (2, 6, 5, 7)
    feed = {"x": synth.normal(x4, 1.0, seed)}
    x = g.add_input("x", list(x4))
    outs = []
    if kind == "layernorm":
        feed = {"x": synth.normal((3, 7, 48), 2.0, seed)}
        x = g.inputs[0][0]
        g.inputs[0] = (x, [3, 7, 48], FLOAT)
        outs = [g.op("LayerNormalization", [x, g.const("s", synth.normal((48,), 1.0, seed ^ 1)),
                                             g.const("b", synth.normal((48,), 1.0, seed ^ 2))],
                     name="ln", axis=-1, epsilon=1e-6)]
    elif kind == "erf_gelu":
        t = g.op("Div", [x, g.const("r2", np.array(1.4142135, np.float32))], name="d")
        t = g.op("Add", [g.op("Erf", [t], name="e"), g.const("one", np.array(1.0, np.float32))], name="a")
        outs = [g.op("Mul", [g.op("Mul", [x, t], name="m"), g.const("h", np.array(0.5, np.float32))], name="m2")]
    elif kind == "transpose":
        outs = [g.op("Transpose", [x], name="t", perm=[0, 2, 3, 1])]
    elif kind == "concat_split":
        a, b, c = g.op("Split", [x, g.const("sz", np.array([1, 3, 2], np.int64))], n_out=3, name="sp", axis=1)
        outs = [g.op("Concat", [c, a, b], name="cat", axis=1)]
    elif kind == "resize_nearest":
        outs = [g.op("Resize", [x, g.const("roi", np.zeros((0,), np.float32)),
                                g.const("sc", np.array([1, 1, 2, 2], np.float32))], name="r", mode="nearest")]
    elif kind == "resize_linear_sizes":
        outs = [g.op("Resize", [x, g.const("roi", np.zeros((0,), np.float32)), g.const("sc", np.zeros((0,), np.float32)),
                                g.const("sizes", np.array([2, 6, 9, 4], np.int64))], name="r", mode="linear")]
    elif kind == "gather_negative":
        outs = [g.op("Gather", [x, g.const("idx", np.array([[4, -1], [0, -5]], np.int64))], name="ga", axis=3)]
    elif kind == "slice_negative_step":
        outs = [g.op("Slice", [x, g.const("st", np.array([-1, 1], np.int64)), g.const("en", np.array([-100, 6], np.int64)),
                               g.const("ax", np.array([3, 1], np.int64)), g.const("sp", np.array([-2, 2], np.int64))],
                     name="sl")]
    elif kind == "reduce_mean":
        outs = [g.op("ReduceMean", [x], name="rm", axes=[2, 3], keepdims=1)]
    elif kind == "topk":
        feed = {"x": synth.normal((3, 50), 1.0, seed)}
        g.inputs[0] = ("x", [3, 50], FLOAT)
        v, i = g.op("TopK", ["x", g.const("k", np.array([7], np.int64))], n_out=2, name="tk", axis=-1)
        g.add_output(v, None, FLOAT)
        g.add_output(i, None, INT64)
        return g, feed
    elif kind == "elementwise":
        y = g.add_input("y", list(x4))
        feed["y"] = np.abs(synth.normal(x4, 1.0, seed ^ 3)) + np.float32(0.5)
        t = g.op("Sub", [g.op("Relu", [x], name="re"), g.op("Sqrt", [y], name="sq")], name="su")
        outs = [g.op("Pow", [y, g.const("p", np.array(1.5, np.float32))], name="pw"), t]
    for o in outs:
        g.add_output(o, None, FLOAT)
    return g, feed


MOVEMENT_KINDS = ["layernorm", "erf_gelu", "transpose", "concat_split", "resize_nearest", "resize_linear_sizes",
                  "gather_negative", "slice_negative_step", "reduce_mean", "topk", "elementwise"]


@needs_ref
@pytest.mark.parametrize("kind", MOVEMENT_KINDS)
def test_np_ref_matches_reference_movement_rows(kind):
    """Float outputs within 1e-6 x max|ref| (the reference accumulates
    LayerNormalization and ReduceMean in double as np_ref does); int64 outputs
    (TopK indices) equal."""
    g, feed = _movement_graph(kind)
    want = ref.run_graph(g, feed)
    got = np_ref.run(g, feed)
    assert set(got) >= set(want)
    for name, b in want.items():
        a = got[name]
        assert a.shape == b.shape, name
        if b.dtype == np.int64:
            np.testing.assert_array_equal(a, b, err_msg=name)
        else:
            assert np.abs(a.astype(np.float64) - b).max() <= 1e-6 * max(1.0, np.abs(b).max()), name
