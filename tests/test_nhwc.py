"""Channels-last (NHWC) trunk of the B200 engine.

The engine keeps a Conv trunk NHWC inside its arena (the Conv A operand then
arrives by TMA im2col); graph inputs and outputs stay NCHW, so results must
equal the all-NCHW path and the oracle. CPU tests check the layout assignment
through the host-only planner; GPU tests run both layouts against the numpy
restatement of the reference kernels (max|err| <= 1e-4 * max|ref|).
"""

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import configs, model
from oracle import np_ref

# (id, batch, cin, h, w, c, m, kernel, strides, pads, dilations, residual, pool, gap)
# (c >= 64: a Conv with at most 32 output channels runs the direct CUDA-core
# kernel, which reads and writes NCHW)
CHAINS = [
    ("3x3s1_res", 2, 3, 20, 20, 64, 64, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), True, False, False),
    ("3x3s2_m40", 2, 8, 16, 15, 64, 40, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), False, False, False),
    ("1x1s2_res", 2, 16, 14, 14, 64, 128, (1, 1), (2, 2), (0, 0, 0, 0), (1, 1), True, False, False),
    ("7x7s2p3", 1, 3, 23, 29, 64, 64, (7, 7), (2, 2), (3, 3, 3, 3), (1, 1), False, False, False),
    ("asym_pads", 2, 4, 17, 13, 64, 48, (3, 3), (2, 2), (0, 0, 1, 1), (1, 1), False, False, False),
    ("dil2", 1, 5, 19, 21, 96, 64, (3, 3), (1, 1), (2, 2, 2, 2), (2, 2), False, False, False),
    ("5x3_s3x1_m42", 2, 3, 25, 11, 64, 42, (5, 3), (3, 1), (2, 1, 2, 1), (1, 1), False, False, False),
    ("pool_gap", 2, 3, 33, 31, 64, 64, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), True, True, True),
    ("b4_56x56", 4, 16, 56, 56, 64, 64, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), True, False, False),
    # C % 32 != 0: the last 32-channel block of each tap reads past C as zeros
    ("c80_3x3_m80", 2, 3, 20, 20, 80, 80, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), False, False, False),
    ("c48_1x1s2_res", 2, 5, 17, 19, 48, 64, (1, 1), (2, 2), (0, 0, 0, 0), (1, 1), True, False, False),
    ("c36_3x3_pool", 1, 3, 21, 23, 36, 64, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), False, True, False),
    ("c100_5x5s2_dil", 2, 3, 23, 21, 100, 40, (5, 5), (2, 2), (4, 4, 3, 3), (2, 2), False, False, False),
]


def _chain(case):
    _, n, cin, h, w, c, m, k, s, p, d, res, pool, gap = case
    return configs.conv_chain(n, cin, h, w, c, m, kernel=k, strides=s, pads=p, dilations=d, residual=res,
                              pool=pool, gap=gap, tag="nhwc_" + case[0])


def _layout(g, flags=0):
    a = model.analyze(g, {n: d for n, d, _ in g.inputs}, flags)
    return {k: v["nhwc"] for k, v in a["tensors"].items()}


@pytest.mark.parametrize("case", CHAINS, ids=[c[0] for c in CHAINS])
def test_chain_layout_assignment(case):
    g, _ = _chain(case)
    lay = _layout(g)
    io = {n for n, _, _ in g.inputs} | {o[0] for o in g.outputs}
    assert not any(lay[t] for t in io), "graph inputs and outputs stay NCHW"
    mid_in = [n for n in g.nodes if n.name == "mid"][0].inputs[0]
    assert lay[mid_in], "the middle Conv reads channels-last"
    assert not any(_layout(g, model.NCHW_ONLY).values())


def test_resnet_trunk_is_channels_last_and_vit_is_not():
    lay = _layout(configs.resnet18(1))
    assert lay["maxpool_out"] and lay["layer4.1.relu_out_out"]
    assert not lay["input"] and not lay["avgpool_out"] and not lay["fc_out"]
    assert not any(_layout(configs.vit_b16(1, layers=1)).values())


def test_a_reshaped_split_half_keeps_the_block_nchw():
    """A Split output that also feeds a reshape (no channels-last form)
    makes the Split's input, both halves and the Concat NCHW."""
    from nert_b200.onnx_io import FLOAT, Graph

    h = Graph(opset=13)
    x = h.add_input("x", [1, 32, 8, 8])
    t = h.op("Conv", [x, h.const("w0", np.ones((64, 32, 3, 3), np.float32))], name="c0", kernel_shape=[3, 3],
             pads=[1, 1, 1, 1])
    p, q = h.op("Split", [t, h.const("sz", np.array([32, 32], np.int64))], n_out=2, name="sp", axis=1)
    c = h.op("Concat", [p, q], name="cc", axis=1)
    h.add_output(h.op("Conv", [c, h.const("w1", np.ones((64, 64, 3, 3), np.float32))], name="c1",
                      kernel_shape=[3, 3], pads=[1, 1, 1, 1]), None, FLOAT)
    h.add_output(h.op("Reshape", [q, h.const("shape", np.array([1, -1], np.int64))], name="flat"), None, FLOAT)
    lay = _layout(h)
    assert not any(lay[v] for v in (t, p, q, c))


def test_yolo_c2f_blocks_and_neck_are_channels_last():
    lay = _layout(configs.yolov8n(1))
    for t in ("b4.split_out1", "b4.cat_out", "b8.cat_out", "up1_out", "cat1_out", "up2_out", "n21.cat_out"):
        assert lay[t], t
    # 16-channel halves feed the direct CUDA-core Conv; the head reshapes
    assert not lay["b2.cat_out"] and not lay["b2.split_out1"] and not lay["h0.cat_out"]


def test_channels_need_16_byte_pixels_for_channels_last():
    lay = _layout(_chain(("c42", 1, 3, 12, 12, 42, 64, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), False, False,
                          False))[0])
    assert not lay["head_relu_out"]  # 42 channels: 168-byte pixels
    lay = _layout(_chain(("c44", 1, 3, 12, 12, 44, 64, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), False, False,
                          False))[0])
    assert lay["head_relu_out"]


def test_grouped_and_narrow_convs_keep_their_input_nchw():
    from nert_b200.onnx_io import FLOAT, Graph

    g = Graph(name="grp", opset=13)
    x = g.add_input("x", [1, 8, 10, 10])
    w0 = np.ones((32, 8, 1, 1), np.float32)
    w1 = np.ones((32, 8, 3, 3), np.float32)
    w2 = np.ones((48, 32, 1, 1), np.float32)  # more than 32 outputs: a tensor-core Conv
    w3 = np.ones((8, 48, 1, 1), np.float32)
    t0 = g.op("Conv", [x, g.const("w0", w0)], name="c0", kernel_shape=[1, 1])
    t1 = g.op("Conv", [t0, g.const("w1", w1)], name="grouped", kernel_shape=[3, 3], pads=[1] * 4, group=4)
    t2 = g.op("Conv", [t1, g.const("w2", w2)], name="c2", kernel_shape=[1, 1])
    t3 = g.op("Conv", [t2, g.const("w3", w3)], name="narrow_in", kernel_shape=[1, 1])
    y = g.op("Conv", [t3, g.const("w4", np.ones((8, 8, 1, 1), np.float32))], name="out", kernel_shape=[1, 1])
    g.add_output(y, None, FLOAT)
    lay = _layout(g)
    assert not lay[t0]   # read by a grouped Conv
    assert lay[t1]       # produced by a Conv, read by a C % 32 == 0 Conv
    assert not lay[t2]   # read by the direct CUDA-core Conv (8 outputs)
    assert not lay[t3]


def _c2f_neck_graph(n, h, w, mode="nearest"):
    """A detector's C2f block and PAN step in miniature: stem -> stride-2
    Conv -> 1x1 Conv -> Split(32, 32) -> bottleneck (3x3 + residual Add) ->
    Concat(3 parts) -> 1x1 Conv -> Resize x2 -> Concat with the stem's
    output -> 1x1 Conv (graph output)."""
    from nert_b200 import synth
    from nert_b200.onnx_io import FLOAT, Graph

    g = Graph(name="c2f_neck", opset=13)
    x = g.add_input("x", [n, 3, 2 * h, 2 * w])
    k = [0]

    def conv(t, cin, cout, ks, stride=1, relu=True):
        k[0] += 1
        wt = synth.normal((cout, cin, ks, ks), (2.0 / (cin * ks * ks)) ** 0.5, synth.seed_of("c2f", f"w{k[0]}"))
        bi = synth.normal((cout,), 0.1, synth.seed_of("c2f", f"b{k[0]}"))
        y = g.op("Conv", [t, g.const(f"w{k[0]}", wt), g.const(f"b{k[0]}", bi)], name=f"conv{k[0]}",
                 kernel_shape=[ks, ks], strides=[stride, stride], pads=[ks // 2] * 4)
        return g.op("Relu", [y], name=f"relu{k[0]}") if relu else y

    s = conv(x, 3, 64, 3)
    d = conv(s, 64, 64, 3, 2)
    t1 = conv(d, 64, 64, 1)
    a, b = g.op("Split", [t1, g.const("halves", np.array([32, 32], np.int64))], n_out=2, name="split", axis=1)
    r = g.op("Add", [b, conv(conv(b, 32, 32, 3), 32, 32, 3)], name="res")
    t2 = conv(g.op("Concat", [a, b, r], name="cat", axis=1), 96, 64, 1)
    up = g.const("scales", np.array([1, 1, 2, 2], np.float32))
    u = g.op("Resize", [t2, g.const("roi", np.zeros((0,), np.float32)), up], name="up", mode=mode)
    y = conv(g.op("Concat", [u, s], name="cat2", axis=1), 128, 64, 1, relu=False)
    g.add_output(y, None, FLOAT)
    feed = {"x": synth.uniform((n, 3, 2 * h, 2 * w), -1.0, 1.0, synth.seed_of("c2f", f"x{n}{h}{w}"))}
    return g, feed


def test_split_concat_resize_join_the_channels_last_trunk():
    g, _ = _c2f_neck_graph(2, 12, 10)
    lay = _layout(g)
    for t in ("split_out0", "split_out1", "res_out", "cat_out", "up_out", "cat2_out", "relu1_out", "relu4_out"):
        assert lay[t], t
    assert not lay["x"] and not lay[g.outputs[0][0]]
    assert not any(_layout(g, model.NCHW_ONLY).values())
    # a Conv reading a 22-channel half (88-byte pixels) cannot take TMA
    # im2col: the Split's and Concat's tensors then all stay NCHW
    from nert_b200.onnx_io import FLOAT, Graph

    for read_half in (False, True):
        h = Graph(opset=13)
        x = h.add_input("x", [1, 32, 8, 8])
        t = h.op("Conv", [x, h.const("w0", np.ones((64, 32, 1, 1), np.float32))], name="c0", kernel_shape=[1, 1])
        p, q = h.op("Split", [t, h.const("sz", np.array([42, 22], np.int64))], n_out=2, name="sp", axis=1)
        c = h.op("Concat", [q, p], name="cc", axis=1)
        h.add_output(h.op("Conv", [c, h.const("w1", np.ones((64, 64, 1, 1), np.float32))], name="c1",
                          kernel_shape=[1, 1]), None, FLOAT)
        if read_half:
            h.add_output(h.op("Conv", [q, h.const("w2", np.ones((64, 22, 1, 1), np.float32))], name="c2",
                              kernel_shape=[1, 1]), None, FLOAT)
        lay = _layout(h)
        assert [lay[v] for v in (t, p, q, c)] == [not read_half] * 4, read_half


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["nearest", "linear"])
def test_split_concat_resize_channels_last_match_oracle(cuda, mode):
    g, feed = _c2f_neck_graph(2, 12, 10, mode)
    out = g.outputs[0][0]
    ref = np_ref.run(g, feed)[out]
    res = {}
    for cl in (True, False):
        m = model.Model(g, {"x": list(feed["x"].shape)}, channels_last=cl)
        try:
            res[cl] = m.run(feed)[out]
            labels = [lab for lab, _ in m.profile()]
        finally:
            m.close()
        for op in ("Split:", "Concat:", "Resize:"):
            assert any(lab.startswith(op) and lab.endswith("[nhwc]") for lab in labels) == cl, (op, labels)
        assert rel_err(res[cl], ref) <= TOL, cl
    assert rel_err(res[True], res[False]) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("case", CHAINS, ids=[c[0] for c in CHAINS])
def test_chain_channels_last_matches_nchw_and_oracle(cuda, case):
    g, feed = _chain(case)
    ref = np_ref.run(g, feed)
    out_name = g.outputs[0][0]
    outs = {}
    for cl in (True, False):
        m = model.Model(g, {k: list(v.shape) for k, v in feed.items()}, channels_last=cl)
        try:
            outs[cl] = m.run(feed)[out_name]
            labels = [lab for lab, _ in m.profile()]
        finally:
            m.close()
        assert any("nhwc" in lab for lab in labels) == cl, labels
        assert rel_err(outs[cl], ref[out_name]) <= TOL, cl
    assert rel_err(outs[True], outs[False]) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("builder,batch,out", [(configs.resnet18, 2, "fc_out"), (configs.resnet50, 1, None)])
def test_resnet_channels_last_equals_nchw(cuda, builder, batch, out):
    g = builder(batch)
    x = configs.resnet_input(batch)
    out = out or g.outputs[0][0]
    res = {}
    for cl in (True, False):
        m = model.Model(g, {"input": list(x.shape)}, channels_last=cl)
        try:
            res[cl] = m.run({"input": x})[out]
        finally:
            m.close()
    ref = np_ref.run(g, {"input": x})[out]
    assert rel_err(res[True], ref) <= TOL
    assert rel_err(res[False], ref) <= TOL


# (id, N, C, H, W, M, kernel, strides, pads, dilations): narrow-channel convs on an NCHW graph input
C4_CASES = [
    ("stem7x7", 2, 3, 224, 224, 64, (7, 7), (2, 2), (3, 3, 3, 3), (1, 1)),
    ("yolo3x3s2", 2, 3, 64, 80, 16, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1)),
    ("patch16", 2, 3, 224, 224, 96, (16, 16), (16, 16), (0, 0, 0, 0), (1, 1)),
    ("c1_dil", 1, 1, 37, 41, 40, (3, 5), (1, 2), (2, 1, 0, 3), (2, 1)),
    ("c4_odd", 3, 4, 19, 23, 130, (5, 5), (3, 3), (2, 2, 2, 2), (1, 1)),
    ("c6_3x3", 2, 6, 33, 35, 24, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1)),
    ("c8_3x3s2", 2, 8, 40, 48, 32, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1)),
    ("c12_5x5", 1, 12, 29, 31, 70, (5, 5), (1, 1), (2, 2, 2, 2), (1, 1)),
    ("c16_3x3s2", 2, 16, 64, 80, 32, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1)),
    ("c16_1x1", 2, 16, 20, 20, 48, (1, 1), (1, 1), (0, 0, 0, 0), (1, 1)),
]


def _cvec_label(c):
    return "[c4]" if c <= 4 else ("[c8]" if c <= 8 else "[c16]")


def _c4_graph(case):
    name, n, c, h, w, m, k, s, p, d = case
    from nert_b200 import synth
    from nert_b200.onnx_io import FLOAT, Graph

    g = Graph(opset=13)
    x = g.add_input("x", [n, c, h, w])
    wt = synth.normal((m, c, k[0], k[1]), (2.0 / (c * k[0] * k[1])) ** 0.5, synth.seed_of("c4", name + "w"))
    bi = synth.normal((m,), 0.1, synth.seed_of("c4", name + "b"))
    y = g.op("Relu", [g.op("Conv", [x, g.const("w", wt), g.const("b", bi)], name="conv", kernel_shape=list(k),
                           strides=list(s), pads=list(p), dilations=list(d))], name="relu")
    g.add_output(y, None, FLOAT)
    return g, {"x": synth.uniform((n, c, h, w), -1.0, 1.0, synth.seed_of("c4", name + "x"))}


@pytest.mark.gpu
@pytest.mark.parametrize("case", C4_CASES, ids=[c[0] for c in C4_CASES])
def test_narrow_channel_conv_c4_path(cuda, case):
    """NCHW inputs with up to 16 channels run on an NHWC copy padded to 4, 8
    or 16 channels (one to four 16-byte loads per tap); off with
    channels_last=False. Layers with at most 32 outputs and few
    multiply-adds per pixel take the direct CUDA-core kernel instead."""
    g, feed = _c4_graph(case)
    _, _, c, _, _, m_out, k = case[:7]
    direct = m_out <= 32 and c * k[0] * k[1] * m_out <= 2560
    tag = "[direct]" if direct else _cvec_label(case[2])
    ref = np_ref.run(g, feed)
    out_name = g.outputs[0][0]
    for cl in (True, False):
        m = model.Model(g, {"x": list(feed["x"].shape)}, channels_last=cl)
        try:
            out = m.run(feed)[out_name]
            labels = [lab for lab, _ in m.profile()]
        finally:
            m.close()
        assert any(tag in lab for lab in labels) == (cl or direct), labels
        assert rel_err(out, ref[out_name]) <= TOL, cl


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(2, 64, 30, 26, 48, 3, 1, 1), (1, 96, 17, 17, 130, 5, 2, 2),
                                   (2, 48, 21, 27, 40, 3, 1, 1), (1, 80, 18, 22, 64, 3, 2, 1),
                                   (1, 17, 15, 16, 33, 5, 1, 2)],
                         ids=["3x3", "5x5s2", "c48_3x3", "c80_3x3s2", "c17_5x5"])
def test_nchw_graph_input_takes_transposed_tma_path(cuda, shape):
    """A spatial Conv on an NCHW tensor with more than 16 channels (a
    single-op graph) runs on an NHWC copy, channels zero padded to a multiple
    of 32, through TMA im2col; results match the oracle."""
    from nert_b200 import synth
    from nert_b200.onnx_io import FLOAT, Graph

    n, c, h, w, m, k, s, p = shape
    g = Graph(opset=13)
    x = g.add_input("x", [n, c, h, w])
    wt = synth.normal((m, c, k, k), (1.0 / (c * k * k)) ** 0.5, synth.seed_of("tnhwc", "w"))
    y = g.op("Conv", [x, g.const("w", wt)], name="conv", kernel_shape=[k, k], strides=[s, s], pads=[p] * 4)
    g.add_output(y, None, FLOAT)
    feed = {"x": synth.normal((n, c, h, w), 1.0, synth.seed_of("tnhwc", "x"))}
    ref = np_ref.run(g, feed)[y]
    m_ = model.Model(g, {"x": [n, c, h, w]})
    try:
        out = m_.run(feed)[y]
        labels = [lab for lab, _ in m_.profile()]
    finally:
        m_.close()
    assert any("[t>nhwc]" in lab for lab in labels), labels
    assert rel_err(out, ref) <= TOL
