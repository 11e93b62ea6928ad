"""Generate the golden outputs of the benchmarked model configurations.

TEST INFRASTRUCTURE: runs the reference's own CPU library (oracle/_ref,
compiled from the reference sources by oracle/Makefile) through its loader
and executor (``oracle.ref.run_graph``) on single images of each benchmarked
batch, and stores the outputs in ``tests/golden/models/<config>.npz``.

Images are independent in every config (BatchNorm is folded, no op couples
the batch), and every weight is seeded by tensor name only, so image ``i`` of
the batch-B run must reproduce the batch-1 graph's output on that image. The
inputs are the first ``B`` images of the seeded batch, so the GPU test
regenerates them with ``configs.*_input(B)``.

Stored per image ``i`` (keys ``<output>/<i>``): every graph output, except
that the YOLO pre-TopK scores [672000] are subsampled every SCORE_STRIDE-th
element and its boxes [4, 8400] every BOX_STRIDE-th anchor, to keep the files
small.

    python tests/golden/make_model_fixtures.py [config ...]
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "models")

# config -> (benchmarked batch, images of that batch that are pinned)
CONFIGS = {
    "resnet18": 64,
    "resnet50": 32,
    "vit_b16": 32,
    "yolov8n": 16,
}
SCORE_STRIDE = 127
BOX_STRIDE = 11


def images(batch: int) -> list[int]:
    return [0, batch // 2, batch - 1]


def graph_and_input(config: str, batch: int):
    """(batch-1 graph, input name, seeded batch-B input) of one config."""
    sys.path.insert(0, ROOT)
    from nert_b200 import configs

    if config == "resnet18":
        return configs.resnet18(1), "input", configs.resnet_input(batch)
    if config == "resnet50":
        return configs.resnet50(1, expose_logits=True), "input", configs.resnet_input(batch, "resnet50")
    if config == "vit_b16":
        return configs.vit_b16(1), "input", configs.vit_input(batch)
    if config == "yolov8n":
        return configs.yolov8n(1, expose_scores=True), "images", configs.yolo_input(batch)
    raise KeyError(config)


def subsample(config: str, name: str, arr: np.ndarray) -> np.ndarray:
    """The stored form of output ``name`` of one image (batch axis dropped)."""
    a = arr[0]
    if config == "yolov8n" and name == "scores.flat_out":
        return a[::SCORE_STRIDE].copy()
    if config == "yolov8n" and name == "boxes_out":
        return a[:, ::BOX_STRIDE].copy()
    return a


def one(job):
    config, batch, i = job
    sys.path.insert(0, ROOT)
    from oracle import ref

    g, name, x = graph_and_input(config, batch)
    out = ref.run_graph(g, {name: np.ascontiguousarray(x[i:i + 1])})
    return config, i, {k: subsample(config, k, v) for k, v in out.items()}


def main(argv):
    sys.path.insert(0, ROOT)
    from oracle import ref

    if not ref.available():
        ref.build()
    wanted = argv or list(CONFIGS)
    jobs = [(c, CONFIGS[c], i) for c in wanted for i in images(CONFIGS[c])]
    results: dict[str, dict[str, np.ndarray]] = {c: {} for c in wanted}
    import multiprocessing as mp

    with cf.ProcessPoolExecutor(max_workers=min(8, os.cpu_count() or 1), mp_context=mp.get_context("spawn")) as ex:
        for config, i, outs in ex.map(one, jobs):
            for k, v in outs.items():
                results[config][f"{k}/{i}"] = v
            print(f"{config} image {i}: {', '.join(outs)}", flush=True)
    os.makedirs(OUT, exist_ok=True)
    for config, arrs in results.items():
        arrs["batch"] = np.array(CONFIGS[config], np.int64)
        np.savez_compressed(os.path.join(OUT, f"{config}.npz"), **arrs)


if __name__ == "__main__":
    main(sys.argv[1:])
