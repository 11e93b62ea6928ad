"""Parity of every remaining row on the B200 (engine single-op graphs and the
nert::Device plug-in) against the oracle: the reference's known answers
(CASES2) and seeded config-sized cases. Float rows within
max|err| <= 1e-4 * max|ref|; int64 rows and TopK/Gather indices bit-exact."""

import numpy as np
import pytest

from conftest import TOL, rel_err
from golden.known_answers import CASES2
from helpers import case2_graph, check_outputs
from nert_b200 import synth
from nert_b200.onnx_io import FLOAT, INT64, Graph
from oracle import np_ref

pytestmark = pytest.mark.gpu


def run_engine(g, feeds, **kw):
    from nert_b200.model import Model

    m = Model(g, {k: list(v.shape) for k, v in feeds.items()}, **kw)
    try:
        return m.run(feeds)
    finally:
        m.close()


@pytest.mark.parametrize("case", CASES2, ids=lambda c: c[0].split()[1] + ("_" + c[1] if "(" in c[0] else ""))
def test_known_answers_engine(cuda, case):
    g, feeds, expected = case2_graph(case)
    if not feeds:
        pytest.skip("no runtime input")
    check_outputs(run_engine(g, feeds), expected, max(case[5], 1e-6), case[0])


def one(op, in_shapes, attrs=None, consts=None, n_out=1, opset=13, dtypes=None):
    g = Graph(opset=opset)
    names, feeds = [], {}
    consts = consts or {}
    for i, s in enumerate(in_shapes):
        if i in consts:
            names.append(g.const(f"c{i}", consts[i]))
            continue
        dt = (dtypes or {}).get(i, "f32")
        if dt == "i64":
            feeds[f"in{i}"] = np.asarray(synth.uniform(s, 0, 1, 100 + i) * 1000, np.int64)
            names.append(g.add_input(f"in{i}", list(s), INT64))
        else:
            feeds[f"in{i}"] = synth.normal(s, 1.0, synth.seed_of("rows", f"{op}{i}{s}"))
            names.append(g.add_input(f"in{i}", list(s)))
    outs = g.op(op, names, n_out=n_out, name="node", **(attrs or {}))
    for o in (outs if isinstance(outs, list) else [outs]):
        g.add_output(o, None, FLOAT)
    return g, feeds


def compare(g, feeds):
    ref = np_ref.run(g, feeds)
    got = run_engine(g, feeds)
    for k, want in ref.items():
        have = got[k]
        assert have.shape == want.shape, (k, have.shape, want.shape)
        if want.dtype == np.int64:
            np.testing.assert_array_equal(have, want)
        else:
            assert rel_err(have, want) <= TOL, (k, rel_err(have, want))


ROW_CASES = [
    ("softmax_vit", "Softmax", [(4, 12, 197, 197)], {"axis": -1}, {}),
    ("softmax_long", "Softmax", [(8, 5000)], {"axis": -1}, {}),
    ("softmax_dfl", "Softmax", [(2, 16, 4, 8400)], {"axis": 1}, {}),
    ("layernorm_vit", "LayerNormalization", [(8, 197, 768), (768,), (768,)], {"axis": -1, "epsilon": 1e-6},
     {1: synth.normal((768,), 1.0, 7), 2: synth.normal((768,), 1.0, 8)}),
    ("layernorm_wide", "LayerNormalization", [(16, 2048), (2048,)], {"axis": -1}, {1: synth.normal((2048,), 1.0, 9)}),
    ("erf", "Erf", [(3, 197, 3072)], {}, {}),
    ("sigmoid", "Sigmoid", [(2, 80, 8400)], {}, {}),
    ("sqrt_abs", "Abs", [(1000,)], {}, {}),
    ("transpose_tokens", "Transpose", [(8, 768, 196)], {"perm": [0, 2, 1]}, {}),
    ("transpose_heads", "Transpose", [(8, 197, 12, 64)], {"perm": [0, 2, 1, 3]}, {}),
    ("transpose_k", "Transpose", [(8, 197, 12, 64)], {"perm": [0, 2, 3, 1]}, {}),
    ("concat_c", "Concat", [(2, 16, 80, 80), (2, 16, 80, 80), (2, 32, 80, 80)], {"axis": 1}, {}),
    ("concat_last", "Concat", [(2, 144, 6400), (2, 144, 1600), (2, 144, 400)], {"axis": 2}, {}),
    ("maxpool_sppf", "MaxPool", [(2, 128, 20, 20)], {"kernel_shape": [5, 5], "strides": [1, 1], "pads": [2] * 4}, {}),
    ("maxpool_2x2", "MaxPool", [(3, 5, 17, 21)], {"kernel_shape": [2, 2], "strides": [2, 2]}, {}),
    ("maxpool_dil", "MaxPool", [(2, 4, 13, 14)],
     {"kernel_shape": [3, 3], "strides": [1, 1], "pads": [2, 2, 2, 2], "dilations": [2, 2]}, {}),
    ("maxpool_ceil", "MaxPool", [(2, 8, 15, 15)],
     {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [0, 0, 1, 1], "ceil_mode": 1}, {}),
    ("gap_r50", "GlobalAveragePool", [(4, 2048, 7, 7)], {}, {}),
    ("resize_up", "Resize", [(2, 256, 20, 20), (0,), (4,)], {"mode": "nearest"},
     {1: np.zeros((0,), np.float32), 2: np.array([1, 1, 2, 2], np.float32)}),
    # nearest on the last two axes (two-axis gather path): fractional scales,
    # odd sizes, rank 3; a resized leading axis takes the general kernel
    ("resize_near_frac", "Resize", [(2, 5, 17, 23), (0,), (4,)], {"mode": "nearest"},
     {1: np.zeros((0,), np.float32), 2: np.array([1, 1, 1.5, 0.75], np.float32)}),
    ("resize_near_rank3", "Resize", [(6, 9, 11), (0,), (3,)], {"mode": "nearest"},
     {1: np.zeros((0,), np.float32), 2: np.array([1, 3, 2], np.float32)}),
    ("resize_near_lead", "Resize", [(2, 3, 8, 8), (0,), (4,)], {"mode": "nearest"},
     {1: np.zeros((0,), np.float32), 2: np.array([1, 2, 2, 2], np.float32)}),
    ("resize_linear", "Resize", [(1, 3, 17, 23), (0,), (4,)], {"mode": "linear"},
     {1: np.zeros((0,), np.float32), 2: np.array([1, 1, 1.5, 2.25], np.float32)}),
    ("slice_step", "Slice", [(4, 30, 40), (2,), (2,), (2,), (2,)], {},
     {1: np.array([1, 35], np.int64), 2: np.array([28, 2], np.int64), 3: np.array([1, 2], np.int64),
      4: np.array([3, -2], np.int64)}),
    ("reducemean_tail", "ReduceMean", [(4, 64, 7, 7)], {"axes": [2, 3], "keepdims": 1}, {}),
    ("pow", "Pow", [(64, 64), (64, 64)], {}, {}),
    # broadcast binaries: scalar, row, per-row value, mirrored, unaligned and rank-3 forms
    ("div_scalar", "Div", [(3, 197, 3072), ()], {}, {1: np.array(1.4142135, np.float32)}),
    ("sub_scalar_first", "Sub", [(), (4, 197, 768)], {}, {0: np.array(1.0, np.float32)}),
    ("add_row", "Add", [(8, 197, 768), (1, 197, 768)], {}, {}),
    ("mul_col", "Mul", [(96, 400), (96, 1)], {}, {}),
    ("div_row_first", "Div", [(768,), (16, 768)], {}, {}),
    ("add_row_unaligned", "Add", [(6, 7, 13), (7, 13)], {}, {}),
    ("mul_channel", "Mul", [(2, 64, 20, 20), (1, 64, 1, 1)], {}, {}),
    ("sub_outer", "Sub", [(5, 1, 12), (1, 9, 1)], {}, {}),
    # permutes: rows kept (vector and scalar widths), tiled, unit axes, rank 5
    ("transpose_ctx", "Transpose", [(8, 12, 197, 64)], {"perm": [0, 2, 1, 3]}, {}),
    ("transpose_rows_odd", "Transpose", [(3, 5, 7, 9)], {"perm": [1, 0, 2, 3]}, {}),
    ("transpose_unit", "Transpose", [(1, 197, 1, 768)], {"perm": [2, 3, 0, 1]}, {}),
    ("transpose_r5", "Transpose", [(2, 3, 4, 5, 6)], {"perm": [4, 2, 0, 3, 1]}, {}),
    ("transpose_nchw_nhwc", "Transpose", [(2, 80, 33, 35)], {"perm": [0, 2, 3, 1]}, {}),
]


@pytest.mark.parametrize("case", ROW_CASES, ids=lambda c: c[0])
def test_row_parity(cuda, case):
    name, op, shapes, attrs, consts = case
    g, feeds = one(op, shapes, attrs, consts, opset=17 if op == "LayerNormalization" else 13)
    if op == "Pow":
        feeds["in0"] = np.abs(feeds["in0"]) + np.float32(0.5)
    compare(g, feeds)


def test_split_unequal(cuda):
    g, feeds = one("Split", [(2, 96, 40, 40), (3,)], {"axis": 1}, {1: np.array([16, 48, 32], np.int64)}, n_out=3)
    compare(g, feeds)


def test_gather_rows_and_scalar(cuda):
    g = Graph(opset=13)
    g.add_input("x", [4, 197, 768])
    y = g.op("Gather", ["x", g.const("i", np.array(0, np.int64))], name="cls", axis=1)
    g.add_output(y, None, FLOAT)
    compare(g, {"x": synth.normal((4, 197, 768), 1.0, 3)})
    g = Graph(opset=13)
    g.add_input("x", [8400, 4])
    g.add_input("idx", [300], INT64)
    y = g.op("Gather", ["x", "idx"], name="rows", axis=0)
    g.add_output(y, None, FLOAT)
    idx = (synth.uniform((300,), 0, 1, 4) * 8400).astype(np.int64)
    idx[::7] -= 8400  # negative indices wrap
    compare(g, {"x": synth.normal((8400, 4), 1.0, 5), "idx": idx})


@pytest.mark.parametrize("rows,length,k", [(1, 672000, 300), (16, 672000, 300), (64, 1000, 5), (3, 50, 50)])
def test_topk_bit_exact(cuda, rows, length, k):
    """Tie-free inputs (a seeded permutation of distinct values): values and
    int64 indices must match the reference order exactly."""
    base = np.arange(rows * length, dtype=np.float64)
    perm = np.argsort(synth.uniform((rows * length,), 0, 1, 11), kind="stable")
    x = ((base[perm] / (rows * length)) * 2 - 1).astype(np.float32).reshape(rows, length)
    g, _ = one("TopK", [(rows, length), (1,)], {"axis": -1}, {1: np.array([k], np.int64)}, n_out=2)
    feeds = {"in0": x}
    ref = np_ref.run(g, feeds)
    got = run_engine(g, feeds)
    for name in ref:
        np.testing.assert_array_equal(got[name], ref[name])


@pytest.mark.parametrize("length", [4096, 300001], ids=["row_kernel", "split_passes"])
def test_topk_ties_take_smallest_index(cuda, length):
    x = np.zeros((2, length), np.float32)
    x[:, ::3] = 1.0  # many exact ties
    g, _ = one("TopK", [(2, length), (1,)], {"axis": -1}, {1: np.array([100], np.int64)}, n_out=2)
    ref = np_ref.run(g, {"in0": x})
    got = run_engine(g, {"in0": x})
    for name in ref:
        np.testing.assert_array_equal(got[name], ref[name])


def test_int64_index_arithmetic(cuda):
    g = Graph(opset=13)
    g.add_input("i", [2, 300], INT64)
    a = g.op("Div", ["i", g.const("n", np.array(80, np.int64))], name="div")
    c = g.op("Sub", ["i", g.op("Mul", [a, g.const("n2", np.array(80, np.int64))], name="mul")], name="sub")
    g.add_output(a, None, INT64)
    g.add_output(c, None, INT64)
    i = (synth.uniform((2, 300), 0, 1, 6) * 672000).astype(np.int64)
    compare(g, {"i": i})


def test_gather_out_of_range_reports_device_error(cuda):
    from nert_b200 import _lib

    g = Graph(opset=13)
    g.add_input("x", [10, 4])
    g.add_input("idx", [3], INT64)
    y = g.op("Gather", ["x", "idx"], name="rows", axis=0)
    g.add_output(y, None, FLOAT)
    with pytest.raises(_lib.NB2Error) as e:
        run_engine(g, {"x": np.ones((10, 4), np.float32), "idx": np.array([1, 10, 2], np.int64)})
    assert e.value.status == _lib.ERR_DEVICE
    # the context stays usable after the reported error
    out = run_engine(g, {"x": np.ones((10, 4), np.float32), "idx": np.array([1, 9, -10], np.int64)})
    assert np.all(list(out.values())[0] == 1.0)


def test_topk_long_rows_mixed_ties(cuda):
    """Long rows take a sampled threshold, one filtering read and an exact sort
    of the survivors; a row whose survivors overflow (here 200,000 exact ties
    at the top) is redone by the radix passes while the other rows keep the
    fast result. Row 0: distinct values; row 1: 500 exact ties of the largest
    value among distinct ones (resolved by index); row 2: the overflow row."""
    L = 672000
    base = np.argsort(synth.uniform((3 * L,), 0, 1, 21), kind="stable").astype(np.float64)
    x = ((base / (3 * L)) * 2 - 1).astype(np.float32).reshape(3, L)
    pos = (synth.uniform((500,), 0, 1, 22) * L).astype(np.int64)
    x[1, pos] = 2.0
    x[2, ::3] = 3.0
    g, _ = one("TopK", [(3, L), (1,)], {"axis": -1}, {1: np.array([300], np.int64)}, n_out=2)
    ref = np_ref.run(g, {"in0": x})
    got = run_engine(g, {"in0": x})
    for name in ref:
        np.testing.assert_array_equal(got[name], ref[name])


AVGPOOL_GPU_CASES = [
    ({"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]}, (2, 16, 57, 57)),
    ({"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1], "count_include_pad": 1}, (2, 16, 57, 57)),
    ({"kernel_shape": [2, 3], "strides": [2, 1], "pads": [0, 1, 1, 0], "ceil_mode": 1}, (1, 4, 9, 10)),
    ({"kernel_shape": [7, 7], "strides": [1, 1]}, (4, 512, 7, 7)),
]


@pytest.mark.parametrize("case", AVGPOOL_GPU_CASES, ids=lambda c: "_".join(f"{k}{v}" for k, v in c[0].items()))
def test_average_pool_bit_exact(cuda, case):
    """AveragePool (engine row) sums in the reference's order: bit-exact with
    the oracle, which is bit-exact with the reference library."""
    attrs, shape = case
    g, feeds = one("AveragePool", [shape], attrs)
    ref = np_ref.run(g, feeds)
    got = run_engine(g, feeds)
    for name in ref:
        np.testing.assert_array_equal(got[name], ref[name])


@pytest.mark.parametrize("length,k", [(5000, 2000), (300000, 1500), (20000, 20000)], ids=["short", "long", "whole_row"])
def test_topk_large_k(cuda, length, k):
    """K above 1024 (the reference accepts any constant K,
    src/kernels/top_k.cpp:53-142): radix passes then a rank-by-count
    placement, bit-exact; half the values repeat, so ties resolve by index."""
    x = synth.normal((3, length), 1.0, 31)
    x[:, ::2] = np.round(x[:, ::2] * 4) / 4  # many exact ties
    g, _ = one("TopK", [(3, length), (1,)], {"axis": -1}, {1: np.array([k], np.int64)}, n_out=2)
    ref = np_ref.run(g, {"in0": x})
    got = run_engine(g, {"in0": x})
    for name in ref:
        np.testing.assert_array_equal(got[name], ref[name])


CONVT_GPU_CASES = [
    ({"strides": [2, 2], "pads": [1, 1, 1, 1], "output_padding": [1, 1]}, (2, 64, 20, 20), (64, 32, 3, 3)),
    ({"strides": [2, 2]}, (2, 128, 20, 20), (128, 64, 2, 2)),
    ({"strides": [1, 2], "pads": [0, 1, 2, 0], "dilations": [2, 1]}, (1, 6, 15, 16), (6, 4, 3, 3)),
    ({"strides": [3, 3], "group": 2, "pads": [1, 1, 1, 1]}, (1, 8, 14, 15), (8, 3, 4, 4)),
]


@pytest.mark.parametrize("case", CONVT_GPU_CASES, ids=lambda c: "_".join(f"{k}{v}" for k, v in c[0].items()))
def test_conv_transpose_engine(cuda, case):
    """ConvTranspose as a stride-1 tensor-core Conv over the zero-inserted
    input, against the restatement of src/kernels/conv_transpose.cpp."""
    attrs, xs, ws = case
    x = synth.normal(xs, 1.0, 61)
    w = synth.normal(ws, 1.0 / np.sqrt(ws[0] * ws[2] * ws[3]), 62)
    b = synth.normal((ws[1] * attrs.get("group", 1),), 1.0, 63)
    g = Graph(opset=13)
    g.add_input("x", list(xs))
    y = g.op("ConvTranspose", ["x", g.const("w", w), g.const("b", b)], name="ct", **attrs)
    g.add_output(y, None, FLOAT)
    ref = np_ref.run(g, {"x": x})[y]
    got = run_engine(g, {"x": x})[y]
    assert got.shape == ref.shape
    assert rel_err(got, ref) <= TOL


@pytest.mark.parametrize("shape,k,chain", [((16, 128, 20, 20), 5, 3), ((2, 7, 13, 9), 3, 2), ((1, 3, 1, 1), 5, 1),
                                          ((3, 5, 40, 41), 5, 3)], ids=["yolo_b16", "ragged", "one_pixel", "p4"])
def test_sppf_fused_bit_exact(cuda, shape, k, chain):
    """The SPPF step (one pass per plane, ops_pool.cu) against the reference
    MaxPool cascade and Concat, bit-exact; the plan must have fused it."""
    from nert_b200 import model as nbm

    g = Graph(opset=13)
    x = g.add_input("x", list(shape))
    ins, cur = [x], x
    for l in range(chain):
        cur = g.op("MaxPool", [cur], name=f"m{l + 1}", kernel_shape=[k, k], strides=[1, 1], pads=[k // 2] * 4)
        ins.append(cur)
    g.add_output(g.op("Concat", ins, name="cat", axis=1), None, FLOAT)
    assert [e["op"] for e in nbm.analyze(g, {"x": list(shape)})["exec"]] == ["SPPF"]
    xv = synth.normal(shape, 1.0, 123)
    xv.ravel()[::17] = -np.inf  # in-range -inf taps stay -inf only where the whole window is
    ref = np_ref.run(g, {"x": xv})
    got = run_engine(g, {"x": xv})
    np.testing.assert_array_equal(list(got.values())[0], list(ref.values())[0])


def test_sppf_c_abi_matches_rows(cuda):
    """nb2_sppf through the C ABI against the unfused MaxPool rows."""
    import torch

    from nert_b200 import _lib
    from nert_b200._lib import i64s

    L, dev = _lib.lib(), _lib.device(0)
    x = torch.randn(4, 32, 20, 20, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    y = torch.empty(4, 128, 20, 20, device="cuda")
    _lib.check(L.nb2_sppf(dev, x.data_ptr(), i64s(x.shape), y.data_ptr(), 5, 3))
    _lib.check(L.nb2_device_synchronize(dev))
    cur, want = x, [x]
    for _ in range(3):
        cur = torch.nn.functional.max_pool2d(cur, 5, 1, 2)
        want.append(cur)
    assert torch.equal(y, torch.cat(want, 1))
    # invalid arguments are refused before any launch
    assert L.nb2_sppf(dev, x.data_ptr(), i64s(x.shape), y.data_ptr(), 4, 3) != 0


@pytest.mark.parametrize("fill", ["flood_of_ties", "best_at_row_end", "duplicates", "mostly_neg_inf"])
def test_topk_long_rows_exact(cuda, fill):
    """Long rows (the sampled-threshold path, with the radix passes for rows
    it cannot make exact): exact values and indices in (value desc, index
    asc) order on inputs that stress it, against the oracle."""
    L, rows, k = 2 * 32768 + 100, 3, 300
    rng = np.random.default_rng(synth.seed_of("topk_long", fill))
    if fill == "flood_of_ties":
        x = np.zeros((rows, L), np.float32)
        x[:, ::997] = 1.0  # fewer ones than k: the rest are the smallest-index zeros
    elif fill == "best_at_row_end":
        x = rng.standard_normal((rows, L)).astype(np.float32)
        x[:, -100:] += 10.0  # the best values all in the row's last 100
    elif fill == "duplicates":
        x = rng.integers(0, 50, (rows, L)).astype(np.float32)
    else:
        x = np.full((rows, L), -np.inf, np.float32)
        x[:, rng.integers(0, L, 200)] = rng.standard_normal(200).astype(np.float32)
    g, _ = one("TopK", [(rows, L), (1,)], {"axis": -1}, {1: np.array([k], np.int64)}, n_out=2)
    ref = np_ref.run(g, {"in0": x})
    got = run_engine(g, {"in0": x})
    for name in ref:
        np.testing.assert_array_equal(got[name], ref[name])
