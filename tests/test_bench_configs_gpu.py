"""Parity at the benchmarked batch sizes: ResNet-18 bs64, ResNet-50 b32,
ViT-B/16 b32 and the YOLOv8n-style detector at b16, through the engine's
public API (CUDA-graph replay, fusion and the channels-last trunk on).

At these batches the contraction kernel takes schedules that small batches
never reach (128-wide tiles with several tiles per CTA, two tiles in flight,
no split K), so the outputs are compared, image by image, with the golden
outputs of the reference's own CPU library on the same images
(tests/golden/models/*.npz, written by tests/golden/make_model_fixtures.py).
Float outputs: max|err| <= 1e-4 * max|ref| per image and output; int64
outputs and TopK indices bit-exact where stated.
"""

import os

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import configs

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "models")
SCORE_STRIDE, BOX_STRIDE = 127, 11  # as make_model_fixtures.py stores them


def _golden(config):
    z = np.load(os.path.join(GOLDEN, f"{config}.npz"))
    per_image = {}
    for key in z.files:
        if "/" in key:
            name, i = key.rsplit("/", 1)
            per_image.setdefault(int(i), {})[name] = z[key]
    return int(z["batch"]), per_image


def _run(graph, feeds):
    from nert_b200.model import Model

    m = Model(graph, {k: list(v.shape) for k, v in feeds.items()})
    try:
        out = m.run(feeds)
        again = m.run(feeds)  # the second run replays the captured graph
        return out, again
    finally:
        m.close()


@pytest.mark.parametrize("config", ["resnet18", "resnet50", "vit_b16"])
def test_classifier_at_bench_batch(cuda, config):
    batch, gold = _golden(config)
    build = {"resnet18": (configs.resnet18, lambda b: configs.resnet_input(b)),
             "resnet50": (lambda b: configs.resnet50(b, expose_logits=True),
                          lambda b: configs.resnet_input(b, "resnet50")),
             "vit_b16": (configs.vit_b16, configs.vit_input)}[config]
    g = build[0](batch)
    out, again = _run(g, {"input": build[1](batch)})
    for name, _, _ in g.outputs:  # ResNet-50: the softmax and its logits
        np.testing.assert_array_equal(out[name], again[name])
        assert out[name].shape[0] == batch
        for i, want in gold.items():
            err = rel_err(out[name][i], want[name])
            assert err <= TOL, (config, name, i, err)


def _topk_order(v: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values, ties by the smaller index first
    (src/kernels/top_k.cpp:129-134)."""
    order = np.lexsort((np.arange(v.size), -v.astype(np.float64)))
    return order[:k]


def test_yolov8n_at_bench_batch(cuda):
    batch, gold = _golden("yolov8n")
    g = configs.yolov8n(batch, expose_scores=True)
    out, again = _run(g, {"images": configs.yolo_input(batch)})
    for k in out:
        np.testing.assert_array_equal(out[k], again[k])
    scores, boxes = out["scores.flat_out"], out["boxes_out"]
    vals, cls, det = out["topk_out0"], out["class_idx_out"], out["det_boxes_out"]
    assert cls.dtype == np.int64
    k = vals.shape[1]
    for b in range(batch):
        # TopK is bit-exact on the scores this run computed: same values,
        # same int64 indices, in the reference order
        idx = _topk_order(scores[b], k)
        np.testing.assert_array_equal(out["topk_out1"][b], idx)
        np.testing.assert_array_equal(vals[b], scores[b][idx])
        anchor = idx // 80
        np.testing.assert_array_equal(cls[b], idx - 80 * anchor)
        # the box Gather copies the decoded boxes of the chosen anchors
        np.testing.assert_array_equal(det[b], boxes[b][:, anchor].T)
    for i, want in gold.items():
        assert rel_err(scores[i][::SCORE_STRIDE], want["scores.flat_out"]) <= TOL, i
        assert rel_err(boxes[i][:, ::BOX_STRIDE], want["boxes_out"]) <= TOL, i
        assert rel_err(vals[i], want["topk_out0"]) <= TOL, i
        # a pick that differs from the reference's must be a near tie in value
        scale = float(np.abs(want["topk_out0"]).max())
        same = out["topk_out1"][i] == want["topk_out1"]
        assert np.all(np.abs(vals[i][~same] - want["topk_out0"][~same]) <= TOL * scale), i
        np.testing.assert_array_equal(cls[i][same], want["class_idx_out"][same])
        assert rel_err(det[i][same], want["det_boxes_out"][same]) <= TOL, i
