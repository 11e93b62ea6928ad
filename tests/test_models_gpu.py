"""Whole-graph parity of the B200 engine against the oracle.

Every graph runs through the engine's public API (nert_b200.model.Model:
ONNX bytes -> C++ loader/shapes/fusion/planner -> sm_100a rows) and is
compared with the numpy restatement of the reference kernels on the same
seeded inputs and weights (max|err| <= 1e-4 * max|ref|).
"""

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import configs
from oracle import np_ref

pytestmark = pytest.mark.gpu


def _run(graph, inputs, **kw):
    from nert_b200.model import Model

    m = Model(graph, {k: list(v.shape) for k, v in inputs.items()}, **kw)
    try:
        return m.run(inputs), m.stats()
    finally:
        m.close()


@pytest.mark.parametrize("fuse,cuda_graph", [(True, True), (False, False), (True, False)],
                         ids=["fused_graph", "unfused_eager", "fused_eager"])
def test_resnet18_b2(cuda, fuse, cuda_graph):
    g = configs.resnet18(2)
    x = configs.resnet_input(2)
    ref = np_ref.run(g, {"input": x})["fc_out"]
    out, stats = _run(g, {"input": x}, fuse=fuse, cuda_graph=cuda_graph)
    assert rel_err(out["fc_out"], ref) <= TOL
    if fuse:
        assert stats["fused_groups"] == 17


def test_resnet18_repeat_runs_are_identical(cuda):
    from nert_b200.model import Model

    g = configs.resnet18(1)
    x = configs.resnet_input(1)
    m = Model(g, {"input": [1, 3, 224, 224]})
    try:
        a = m.run({"input": x})["fc_out"]
        b = m.run({"input": x})["fc_out"]
        x2 = configs.resnet_input(1, "other")
        c = m.run({"input": x2})["fc_out"]
    finally:
        m.close()
    np.testing.assert_array_equal(a, b)
    assert rel_err(c, np_ref.run(g, {"input": x2})["fc_out"]) <= TOL


def _prefix(g, k):
    from nert_b200 import onnx_io

    h = onnx_io.Graph(name="prefix", opset=g.opset)
    h.nodes = g.nodes[:k]
    used = {i for n in h.nodes for i in n.inputs}
    h.initializers = {n: v for n, v in g.initializers.items() if n in used}
    h.inputs = list(g.inputs)
    h.outputs = [(h.nodes[-1].outputs[0], None, 1)]
    return h


def test_many_models_in_one_process(cuda):
    """Models built, run and freed back to back reuse device memory; every
    upload must be ordered before the rows that read it (a pageable
    cudaMemcpy can return before its DMA lands)."""
    from nert_b200.model import Model

    g = configs.resnet18(1)
    x = configs.resnet_input(1)
    for k in (6, 7, 8, 11, 13, 19, 30, 41, 49):
        h = _prefix(g, k)
        name = h.outputs[0][0]
        ref = np_ref.run(h, {"input": x})[name]
        for fuse in (True, False):
            m = Model(h, {"input": [1, 3, 224, 224]}, fuse=fuse, cuda_graph=fuse)
            try:
                got = m.run({"input": x})[name]
            finally:
                m.close()
            assert rel_err(got, ref) <= TOL, (k, fuse)


def test_vit_b16_b2(cuda):
    """Config 4 (full 12-layer ViT-B/16) at batch 2."""
    g = configs.vit_b16(2)
    x = configs.vit_input(2)
    ref = np_ref.run(g, {"input": x})["head_out"]
    out, stats = _run(g, {"input": x})
    assert rel_err(out["head_out"], ref) <= TOL
    assert stats["fused_groups"] >= 12 * 6  # Q, K, V, proj(+res), fc1, fc2(+res) per layer


def _topk_order(v, k):
    """Indices of the k largest values, ties by the smaller index first
    (src/kernels/top_k.cpp:129-134)."""
    return np.lexsort((np.arange(v.size), -v.astype(np.float64)))[:k]


def _yolo_check(out, ref, tol=TOL):
    """TopK bit-exact on the scores the GPU computed (values and int64
    indices, reference order); class ids and the box Gather exact given those
    indices; scores, boxes and TopK values within tolerance of the oracle; a
    pick that differs from the oracle's is a near tie in value."""
    scores, boxes = out["scores.flat_out"], out["boxes_out"]
    vals, idx, cls, det = out["topk_out0"], out["topk_out1"], out["class_idx_out"], out["det_boxes_out"]
    assert idx.dtype == np.int64 and cls.dtype == np.int64
    assert rel_err(scores, ref["scores.flat_out"]) <= tol
    assert rel_err(boxes, ref["boxes_out"]) <= tol
    assert rel_err(vals, ref["topk_out0"]) <= tol
    scale = float(np.abs(ref["topk_out0"]).max())
    for b in range(vals.shape[0]):
        want = _topk_order(scores[b], vals.shape[1])
        np.testing.assert_array_equal(idx[b], want)
        np.testing.assert_array_equal(vals[b], scores[b][want])
        np.testing.assert_array_equal(cls[b], want % 80)
        np.testing.assert_array_equal(det[b], boxes[b][:, want // 80].T)
        same = idx[b] == ref["topk_out1"][b]
        assert np.all(np.abs(vals[b][~same] - ref["topk_out0"][b][~same]) <= tol * scale)
        np.testing.assert_array_equal(cls[b][same], ref["class_idx_out"][b][same])


@pytest.mark.parametrize("batch", [1, 2])
def test_yolov8n(cuda, batch):
    """Config 3 (YOLOv8n-style detector, 640x640)."""
    g = configs.yolov8n(batch, expose_scores=True)
    x = configs.yolo_input(batch)
    ref = np_ref.run(g, {"images": x})
    out, stats = _run(g, {"images": x})
    _yolo_check(out, ref)
    assert stats["fused_groups"] >= 50


def test_resnet50_b1_softmax(cuda):
    g = configs.resnet50(1, expose_logits=True)
    x = configs.resnet_input(1, "resnet50")
    ref = np_ref.run(g, {"input": x})
    out, stats = _run(g, {"input": x})
    for name, _, _ in g.outputs:
        assert rel_err(out[name], ref[name]) <= TOL, name
    assert stats["fused_groups"] >= 49


def test_captured_graph_survives_split_k_workspace_growth(cuda):
    """A model whose captured CUDA graph splits K (ResNet-18 b1, layer 4)
    keeps working after a later call on the same GPU needs a larger split-K
    buffer: the outgrown buffer is retired, never freed, so the graph's
    replays keep writing into memory they own."""
    import torch

    from nert_b200 import ops
    from nert_b200.model import Model

    g = configs.resnet18(1)
    x = configs.resnet_input(1)
    ref = np_ref.run(g, {"input": x})["fc_out"]
    m = Model(g, {"input": [1, 3, 224, 224]})
    try:
        first = m.run({"input": x})["fc_out"]
        # 72 output tiles, 128 K blocks: split into equal K spans per CTA,
        # whose partial tiles (148 x 2 x 64 KB) outgrow the model's buffer
        a = torch.randn(1152, 4096, device="cuda")
        b = torch.randn(4096, 1024, device="cuda") / 64
        y = ops.gemm(a, b)
        from nert_b200 import _lib

        assert _lib.last_contraction(0)["k_slices"] == 0
        want = (a.double() @ b.double()).float()
        assert rel_err(y.cpu().numpy(), want.cpu().numpy()) <= TOL
        again = m.run({"input": x})["fc_out"]
    finally:
        m.close()
    np.testing.assert_array_equal(first, again)
    assert rel_err(again, ref) <= TOL


def test_pipelined_host_runs_keep_each_input(cuda):
    """run_async copies each run's inputs on a copy stream into one of two
    staging buffers while the previous run computes: four runs queued back to
    back on four different pinned inputs must each return their own result."""
    from nert_b200.model import HostBuffer, Model

    g = configs.resnet18(1)
    xs = [configs.resnet_input(1, f"pipe{i}") for i in range(4)]
    m = Model(g, {"input": [1, 3, 224, 224]})
    try:
        hin = [HostBuffer((1, 3, 224, 224)) for _ in xs]
        hout = [HostBuffer((1, 1000)) for _ in xs]
        for hb, x in zip(hin, xs):
            hb.array[...] = x
        m.run_into([hin[0].ptr], [hout[0].ptr])  # captures the graph
        for hb, ho in zip(hin, hout):
            m.run_async([hb.ptr], [ho.ptr])
        m.synchronize()
        for x, ho in zip(xs, hout):
            ref = np_ref.run(g, {"input": x})["fc_out"]
            assert rel_err(ho.array, ref) <= TOL
    finally:
        m.close()


def test_resnet18_with_batchnorm_nodes(cuda):
    """The unfolded export (Conv then BatchNormalization, folded at load)
    matches the oracle on the folded graph."""
    x = configs.resnet_input(2)
    ref = np_ref.run(configs.resnet18(2), {"input": x})["fc_out"]
    out, _ = _run(configs.resnet18(2, bn_nodes=True), {"input": x})
    assert rel_err(out["fc_out"], ref) <= TOL


def test_standalone_batchnorm_row(cuda):
    """A BatchNormalization that follows no Conv runs as the per-channel
    affine y = x * gamma / sqrt(var + eps) + (beta - mean * gamma / sqrt(var + eps))."""
    from nert_b200 import synth
    from nert_b200.onnx_io import FLOAT, Graph

    g = Graph(opset=13)
    g.add_input("x", [2, 6, 5, 7])
    r = g.op("Relu", ["x"], name="r")
    gamma, beta = synth.normal((6,), 1.0, 1), synth.normal((6,), 1.0, 2)
    mean, var = synth.normal((6,), 1.0, 3), synth.uniform((6,), 0.5, 2.0, 4)
    stats = [g.const(n, v) for n, v in (("g", gamma), ("b", beta), ("m", mean), ("v", var))]
    y = g.op("BatchNormalization", [r] + stats, name="bn", epsilon=1e-3)
    g.add_output(y, None, FLOAT)
    x = synth.normal((2, 6, 5, 7), 1.0, 5)
    out, _ = _run(g, {"x": x})
    a = gamma.astype(np.float64) / np.sqrt(var.astype(np.float64) + np.float32(1e-3))
    want = np.maximum(x, 0).astype(np.float64) * a[None, :, None, None] + (beta - mean * a)[None, :, None, None]
    assert rel_err(out[y], want) <= TOL
