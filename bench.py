#!/usr/bin/env python
"""ResNet-18 fp32 inference throughput on the B200 layer (images/s, bs64 per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload resnet18|resnet50|vit_b16|yolov8n|sweep] [--batch B]

A step is one full forward pass (default: ResNet-18, batch 64 per GPU,
3x224x224, seeded synthetic input and Kaiming weights, BatchNorm folded)
through the engine's public API. Multi-GPU runs are batch-sharded replicas
(one process per GPU under torchrun, no collective on the data path); rank
timings are combined as the max over ranks.

* value:  device-resident input, one CUDA-graph replay per step, timed with
          CUDA events on the engine's stream; L2 is flushed (256 MB write)
          between steps, outside the timed events.
* e2e:    the same through Model.run_async (pinned host input -> H2D -> run ->
          D2H of every output) per step, timed as one region over all steps
          (the input copy of a step overlaps the previous step's forward).
* roofline: the tensor-core Conv/Gemm/MatMul kernel's algorithmic FLOP/s
          over its time inside the timed replay (ms_per_step x its share of
          an eager pass with an event between rows) against the pool's
          measured bf16 GEMM peak / 2 (tf32) / 3 (3xTF32-effective).
* bandwidth_rows: every HBM-bound row at its largest config geometry,
          algorithmic bytes / CUDA-event time, against the measured HBM copy
          bandwidth (1 GPU only).
* --gpus N under torchrun: rank r runs its slice of one seeded global batch
          (weak scaling: --batch per GPU; strong: --global-batch fixed).
* cpu_baseline: the reference NERT CpuDevice (oracle/_ref, compiled from the
          reference sources) on the host cores, one image per process.

Other workloads (the remaining benchmark configs) print the same line with
their own metric; `sweep` prints the single-op sweep (config 1).
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ResNet-18 fp32 images/s bs64 at 1/2/4/8 B200; Conv/GEMM % of TF32 tensor peak"
UNIT = "images/s"
DEFAULT_BATCH = {"resnet18": 64, "resnet50": 32, "vit_b16": 32, "yolov8n": 16, "sweep": 32, "conv": 64, "rows": 0,
                 "attention": 32}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--workload", default="resnet18", choices=list(DEFAULT_BATCH))
    p.add_argument("--batch", type=int, default=None,
                   help="images per GPU (weak scaling: the global batch grows with the GPU count)")
    p.add_argument("--global-batch", type=int, default=None,
                   help="fixed global batch split over the GPUs by the library's shard plan (strong scaling)")
    p.add_argument("--no-rows", action="store_true", help="skip the bandwidth-row table")
    p.add_argument("--ref-device", default="cpu", choices=["cpu", "cuda"],
                   help="--impl reference: the reference CpuDevice (the driver's arm) or its own CudaDevice "
                        "(cuDNN Conv, cuBLAS Gemm/MatMul; the GPU baseline)")
    p.add_argument("--api", default="engine", choices=["engine", "seam"],
                   help="seam: the reference's own loader and executor (oracle/_ref) on nert::b200::Device")
    p.add_argument("--conv", default="3,224,224,64,7,2,3",
                   help="--workload conv: C,H,W,M,K,S,P of one Conv+Relu on an NCHW input of --batch images")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--precision", default="3xtf32", choices=["3xtf32", "1xtf32"])
    a = p.parse_args()
    if a.batch is None:
        a.batch = DEFAULT_BATCH[a.workload]
    return a


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def metric_for(workload: str, batch: int) -> str:
    if workload == "resnet18":
        return METRIC
    return {"resnet50": f"ResNet-50 fp32 images/s bs{batch} per B200",
            "vit_b16": f"ViT-B/16 fp32 images/s bs{batch} per B200",
            "yolov8n": f"YOLOv8n-style fp32 images/s bs{batch} per B200 (640x640, TopK 300)",
            "sweep": "single-op sweep fp32 TFLOP/s per op (config 1)",
            "conv": "one Conv+Relu through the engine, fp32 TFLOP/s"}[workload]


def build_workload(workload: str, batch: int, rows: slice | None = None):
    """(graph, feeds) of one benchmark config; with ``rows`` the graph is
    built for that slice of a seeded batch of ``batch`` images and fed it."""
    from nert_b200 import configs

    n = batch if rows is None else rows.stop - rows.start
    sl = rows if rows is not None else slice(0, batch)
    if workload == "resnet18":
        return configs.resnet18(n), {"input": configs.resnet_input(batch)[sl]}
    if workload == "resnet50":
        return configs.resnet50(n), {"input": configs.resnet_input(batch, "resnet50")[sl]}
    if workload == "vit_b16":
        return configs.vit_b16(n), {"input": configs.vit_input(batch)[sl]}
    if workload == "yolov8n":
        return configs.yolov8n(n), {"images": configs.yolo_input(batch)[sl]}
    raise ValueError(workload)


# ---- reference CPU leg (oracle/_ref, the reference's own CpuDevice) ----------

_REF = None
_REF_FEED = None


def _ref_worker_init(onnx_path, input_name, shape):
    global _REF, _REF_FEED
    from oracle import ref

    _REF = ref.RefModel(onnx_path, {input_name: list(shape)})
    _REF_FEED = (input_name, shape)


def _ref_worker_run(seed):
    import numpy as np

    from nert_b200 import synth

    name, shape = _REF_FEED
    x = synth.uniform(tuple(shape), -1.0, 1.0, seed)
    t0 = time.perf_counter()
    _REF.run({name: x.astype(np.float32)})
    return time.perf_counter() - t0


class RefPool:
    """One spawned process per core, each holding the reference Model at batch 1."""

    def __init__(self, cores: int, workload: str = "resnet18"):
        import multiprocessing as mp

        from nert_b200 import onnx_io

        self.tmp = tempfile.TemporaryDirectory()
        g, feeds = build_workload(workload, 1)
        name, x = next(iter(feeds.items()))
        path = onnx_io.save(g, os.path.join(self.tmp.name, f"{workload}_b1.onnx"))
        self.cores = cores
        self.pool = mp.get_context("spawn").Pool(cores, initializer=_ref_worker_init,
                                                 initargs=(path, name, list(x.shape)))

    def step(self) -> float:
        """`cores` images in parallel; returns wall seconds."""
        t0 = time.perf_counter()
        self.pool.map(_ref_worker_run, list(range(self.cores)), chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()
        self.tmp.cleanup()


def ref_cores() -> int:
    return max(1, min(os.cpu_count() or 1, 8))


def run_reference_cuda(args):
    """The reference's unmodified loader and executor on its own CudaDevice
    (src/cuda_device.cpp: cuDNN Conv src/cuda/conv.cu:230-530, cuBLAS
    Gemm/MatMul src/cuda/gemm.cu:84-166, mat_mul.cu:94-198, a synchronise after
    every row), built by oracle/Makefile: the GPU baseline. Times
    nert::Model::RunTyped (host input -> output) per step."""
    from oracle import ref

    from nert_b200 import onnx_io

    if not ref.available(cuda=True):
        print(json.dumps({"impl": "reference", "device": "cuda",
                          "unavailable": "oracle/_ref/libnert_ref_cuda.so was not built (needs nvcc and cuDNN)"}))
        return 0
    cases = []
    if args.workload == "sweep":
        from nert_b200 import configs

        cases = [(n, *configs.sweep_conv(n, args.batch)) for n, *_ in configs.SWEEP_CONVS]
        cases += [(f"gemm_{m}x{n}x{k}", *configs.sweep_gemm(m, n, k)) for m, n, k in configs.SWEEP_GEMMS]
    else:
        g, feeds = build_workload(args.workload, args.batch)
        cases = [(args.workload, g, feeds)]
    rows = []
    with tempfile.TemporaryDirectory() as d:
        for name, g, feeds in cases:
            path = onnx_io.save(g, os.path.join(d, f"{name}.onnx"))
            m = ref.RefModel(path, {k: list(v.shape) for k, v in feeds.items()}, cuda=True)
            try:
                for _ in range(max(1, args.warmup)):
                    m.run(feeds)
                ms = []
                for _ in range(args.steps):
                    m.run(feeds)
                    ms.append(m.last_ms)
            finally:
                m.close()
            from nert_b200 import model as nbm

            flops = sum(contraction_flops(g, nbm.analyze(g, {k: list(v.shape) for k, v in feeds.items()})).values())
            t = sum(ms) / len(ms)
            rows.append({"case": name, "ms": t, "tflops": flops / (t * 1e-3) / 1e12})
    if args.workload == "sweep":
        total_ms = sum(r["ms"] for r in rows)
        line = {"impl": "reference", "device": "reference CudaDevice (cuDNN, cuBLAS) on B200",
                "metric": metric_for("sweep", args.batch), "value": sum(r["tflops"] * r["ms"] for r in rows) / total_ms,
                "unit": "TFLOP/s", "ms_per_step": total_ms, "ops": rows}
    else:
        t = rows[0]["ms"]
        line = {"impl": "reference", "device": "reference CudaDevice (cuDNN, cuBLAS) on B200",
                "metric": metric_for(args.workload, args.batch), "value": args.batch / (t * 1e-3), "unit": UNIT,
                "ms_per_step": t, "contraction_tflops": rows[0]["tflops"]}
    line.update({"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                 "scaling": "weak", "vs_baseline": None, "dtype": "f32 (cuDNN / cuBLAS FP32)",
                 "data": "synthetic (seeded inputs and weights, BN folded)",
                 "config": {"workload": args.workload, "per_gpu_batch": args.batch},
                 "timing": "nert::Model::RunTyped wall time (host input to host output, a device synchronise "
                           "after every row, as the reference does)"})
    print(json.dumps(line), flush=True)
    return 0


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    if args.ref_device == "cuda":
        return run_reference_cuda(args)
    from oracle import ref

    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libnert_ref.so was not built"}))
        return 0
    if args.workload in ("sweep", "conv", "rows", "attention"):
        print(json.dumps({"impl": "reference", "unavailable": "the single-op workloads have no reference CPU arm"}))
        return 0
    cores = ref_cores()
    pool = RefPool(cores, args.workload)
    try:
        for _ in range(max(0, args.warmup)):
            pool.step()
        walls = [pool.step() for _ in range(args.steps)]
    finally:
        pool.close()
    total = sum(walls)
    value = cores * args.steps / total
    sample = (f"{cores} {args.workload} images per step (batch 1 each, one process per core) of the "
              f"bs{args.batch} workload")
    line = {
        "impl": "reference", "metric": metric_for(args.workload, args.batch), "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (f64 accumulation)",
        "data": "synthetic (seeded inputs and weights, BN folded)",
        "config": {"workload": args.workload, "model": args.workload, "per_gpu_batch": args.batch,
                   "global_batch": args.batch * args.gpus, "device": "host CPU"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- clocks --------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        self.out.flush()
        self.out.seek(0)
        rows = [r.split(", ") for r in self.out.read().strip().splitlines() if r.strip()]
        os.unlink(self.out.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
                for nm, v in zip(names, r[4:8]):
                    if v.strip() == "Active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- roofline helpers ------------------------------------------------------------

def measure_tf32_peak() -> float:
    """Dense TF32 TFLOP/s of a library GEMM (torch/cuBLAS, 8192^3, best of 10)."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        for _ in range(3):
            torch.matmul(a, b)
        torch.cuda.synchronize()
        best = 1e9
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b)
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


# dram__bytes_read.sum + dram__bytes_write.sum over the contraction launches of
# one forward, from the ncu capture summarised in profiles/ (per workload, batch)
TRAFFIC_BYTES = {("resnet18", 64): int((788.3 + 196.2) * 1e6)}


def tensor_peak(precision: str) -> tuple[float, str]:
    """Roofline denominator for the tf32 contraction kernel.

    The measured dense bf16 GEMM rate of this GPU pool (MEASURED_PEAKS.json,
    burst figure; 1590 TFLOP/s fallback when the file is absent) halved for
    tf32 (the tensor pipe's tf32 rate is half its bf16 rate), and divided by
    three more in 3xTF32 mode (three MMAs per product).
    """
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            bf16, src = float(json.load(f)["bf16_tflops"]), "of measured"
    except (OSError, KeyError, ValueError):
        bf16, src = 1590.0, "of fallback"
    div = 6.0 if precision == "3xtf32" else 2.0
    return bf16 / div, f"{src} bf16 {bf16:.1f} TFLOP/s / {div:g} ({precision}: tf32 = bf16/2" + \
        (", three MMAs per product)" if div == 6.0 else ")")


def row_name(label: str) -> str:
    """Node name of a profile label 'Op[+fused]:name[layout]'."""
    name = label.split(":", 1)[1]
    return re.sub(r"(\[[^\]]*\])+$", "", name)


def contraction_flops(graph, analysis) -> dict:
    """Algorithmic FLOPs (2*M*N*K) of every Conv / Gemm / MatMul row, by node name."""
    import numpy as np

    t = analysis["tensors"]
    nodes = {n.name: n for n in graph.nodes}
    shape = lambda name: graph.initializers[name].shape if name in graph.initializers else tuple(t[name]["dims"])
    out = {}
    for e in analysis["exec"]:
        n = nodes[e["name"]]
        y = t[e["outs"][0]]["dims"]
        if e["op"] == "Conv":
            k = int(np.prod(shape(n.inputs[1])[1:]))
        elif e["op"] == "Gemm":
            a = shape(n.inputs[0])
            k = a[0] if n.attrs.get("transA", 0) else a[1]
        elif e["op"] == "MatMul":
            k = shape(n.inputs[0])[-1]
        else:
            continue
        out[e["name"]] = 2.0 * float(np.prod(y)) * k
    return out


def contraction_bytes(graph, analysis) -> dict:
    """Algorithmic bytes of every Conv / Gemm / MatMul row: its operands read
    once (activation, weight, a fused residual) and its output written once."""
    import numpy as np

    t = analysis["tensors"]
    nodes = {n.name: n for n in graph.nodes}
    numel = lambda name: (int(np.prod(graph.initializers[name].shape)) if name in graph.initializers
                          else int(np.prod(t[name]["dims"])))
    out = {}
    for e in analysis["exec"]:
        if e["op"] not in ("Conv", "Gemm", "MatMul"):
            continue
        n = nodes[e["name"]]
        b = numel(n.inputs[0]) + numel(n.inputs[1]) + int(np.prod(t[e["outs"][0]]["dims"]))
        if e.get("residual"):
            b += numel(e["residual"])
        out[e["name"]] = 4.0 * b
    return out


def layer_roofline(sums: dict, flops: dict, nbytes: dict, tensor_peak_tflops: float, hbm_gbs: float) -> dict:
    """Each contraction row against its own roofline: the slower of its FLOPs
    at the tensor peak and its bytes at the HBM peak (short-K 1x1 convs are
    HBM-bound). `frac` = the rows' roofline time / their measured time."""
    rows, bound_ms, meas_ms, t_ms, h_ms = [], 0.0, 0.0, 0.0, 0.0
    for lab, ms in sums.items():
        name = row_name(lab)
        if name not in flops or ms <= 0:
            continue
        tt = flops[name] / (tensor_peak_tflops * 1e12) * 1e3
        th = nbytes.get(name, 0.0) / (hbm_gbs * 1e9) * 1e3
        b = max(tt, th)
        bound_ms += b
        meas_ms += ms
        t_ms += tt if tt >= th else 0.0
        h_ms += th if th > tt else 0.0
        rows.append([lab, round(ms, 4), round(flops[name] / (ms * 1e-3) / 1e12, 1),
                     round(nbytes.get(name, 0.0) / (ms * 1e-3) / 1e9, 0), "tensor" if tt >= th else "hbm",
                     round(b / ms, 3)])
    rows.sort(key=lambda r: -r[1])
    return {"frac": bound_ms / meas_ms if meas_ms else None, "rows_ms": meas_ms,
            "tensor_bound_roofline_ms": t_ms, "hbm_bound_roofline_ms": h_ms,
            "columns": ["row", "ms", "TFLOP/s", "GB/s", "bound", "frac of its roofline"], "rows": rows[:12]}


def hbm_peak() -> tuple[float, str]:
    """Measured HBM copy bandwidth of this pool (MEASURED_PEAKS.json), else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "of measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "of fallback"


def bandwidth_rows(local: int, reps: int = 10, warm: int = 3) -> list[dict]:
    """Every HBM-bound row at the largest config geometry that uses it,
    launched through the C ABI on the layer's stream and timed with CUDA
    events around each launch (L2 flushed before each by a 256 MB write and a
    read of the same buffer).
    bytes = the row's algorithmic bytes (read once + write once)."""
    import ctypes

    import torch

    from nert_b200 import _lib
    from nert_b200._lib import i64s

    L = _lib.lib()
    dev = _lib.device(local)
    stream = torch.cuda.ExternalStream(L.nb2_device_stream(dev), device=torch.device("cuda", local))
    cuda = torch.device("cuda", local)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=cuda)
    flush_sum = torch.empty((), dtype=torch.float32, device=cuda)
    g = torch.Generator(device=cuda)
    g.manual_seed(7)

    def rnd(*shape):
        return torch.rand(shape, device=cuda, generator=g) * 2 - 1

    rows = []

    def add(name, shape, nbytes, fn):
        rows.append((name, shape, nbytes, fn))

    p = lambda t: t.data_ptr()
    # MaxPool: ResNet bs64 stem pool and YOLO b16 SPPF
    x = rnd(64, 64, 112, 112)
    y = torch.empty(64, 64, 56, 56, device=cuda)
    add("MaxPool 3x3/s2 ResNet bs64", [64, 64, 112, 112], 4 * (x.numel() + y.numel()),
        lambda x=x, y=y: L.nb2_maxpool2d(dev, p(x), i64s(x.shape), p(y), i64s(y.shape), i64s([3, 3]), i64s([2, 2]),
                                         i64s([1, 1, 1, 1]), i64s([1, 1])))
    x2 = rnd(16, 128, 20, 20)
    y2 = torch.empty_like(x2)
    add("MaxPool 5x5/s1 SPPF YOLO b16", [16, 128, 20, 20], 8 * x2.numel(),
        lambda x=x2, y=y2: L.nb2_maxpool2d(dev, p(x), i64s(x.shape), p(y), i64s(y.shape), i64s([5, 5]),
                                           i64s([1, 1]), i64s([2, 2, 2, 2]), i64s([1, 1])))
    # GlobalAveragePool: ResNet-50 b32
    x3 = rnd(32, 2048, 7, 7)
    y3 = torch.empty(32 * 2048, device=cuda)
    add("GlobalAveragePool ResNet-50 b32", [32, 2048, 7, 7], 4 * (x3.numel() + y3.numel()),
        lambda x=x3, y=y3: L.nb2_row_mean(dev, p(x), 32 * 2048, 49, p(y)))
    # Softmax: ViT attention rows, YOLO DFL bins (axis 1 of [16, 16, 33600])
    x4 = rnd(32, 12, 197, 197)
    y4 = torch.empty_like(x4)
    add("Softmax ViT b32 [32,12,197,197]", list(x4.shape), 8 * x4.numel(),
        lambda x=x4, y=y4: L.nb2_softmax(dev, p(x), p(y), 32 * 12 * 197, 197, 1))
    x5 = rnd(16, 16, 33600)
    y5 = torch.empty_like(x5)
    add("Softmax DFL YOLO b16 (axis of 16)", list(x5.shape), 8 * x5.numel(),
        lambda x=x5, y=y5: L.nb2_softmax(dev, p(x), p(y), 16, 16, 33600))
    # LayerNormalization: ViT b32
    x6 = rnd(32 * 197, 768)
    y6 = torch.empty_like(x6)
    sc, bi = rnd(768), rnd(768)
    add("LayerNormalization ViT b32", [32, 197, 768], 8 * x6.numel() + 8 * 768,
        lambda x=x6, y=y6, s=sc, b=bi: L.nb2_layernorm(dev, p(x), p(s), p(b), p(y), None, None, 32 * 197, 768,
                                                         ctypes.c_float(1e-6)))
    # TopK and the box Gather: YOLO b16
    x7 = torch.rand(16, 672000, device=cuda, generator=g)
    v7 = torch.empty(16, 300, device=cuda)
    i7 = torch.empty(16, 300, dtype=torch.int64, device=cuda)
    add("TopK k=300 YOLO b16 [16,672000]", [16, 672000], 4 * x7.numel() + 12 * 16 * 300,
        lambda x=x7, v=v7, i=i7: L.nb2_topk(dev, p(x), p(v), p(i), 16, 672000, 300))
    x8 = rnd(16 * 8400, 4)
    idx8 = torch.randint(0, 16 * 8400, (16 * 300,), device=cuda, generator=g)
    y8 = torch.empty(16 * 300, 4, device=cuda)
    add("Gather boxes YOLO b16", [16 * 8400, 4], 8 * y8.numel() + 8 * idx8.numel(),
        lambda x=x8, i=idx8, y=y8: L.nb2_gather(dev, p(x), p(i), p(y), 1, 16 * 8400, 4, 16 * 300, 4))
    # Resize nearest x2: YOLO b16 PAN up-sampling
    x9 = rnd(16, 256, 20, 20)
    y9 = torch.empty(16, 256, 40, 40, device=cuda)
    sc9 = (ctypes.c_double * 4)(1.0, 1.0, 2.0, 2.0)
    add("Resize nearest x2 YOLO b16", [16, 256, 20, 20], 4 * (x9.numel() + y9.numel()),
        lambda x=x9, y=y9: L.nb2_resize(dev, p(x), p(y), i64s(x.shape), i64s(y.shape), sc9, 4, 0, 0, 0, 0))
    # Transpose ViT patch tokens, Concat of the YOLO head levels
    x10 = rnd(32, 768, 196)
    y10 = torch.empty(32, 196, 768, device=cuda)
    add("Transpose ViT b32 [32,768,196]->[32,196,768]", [32, 768, 196], 8 * x10.numel(),
        lambda x=x10, y=y10: L.nb2_transpose(dev, p(x), p(y), i64s(x.shape), i64s([0, 2, 1]), 3, 4))
    parts = [rnd(16, 144, n) for n in (6400, 1600, 400)]
    whole = torch.empty(16, 144, 8400, device=cuda)
    c_parts = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in parts])
    add("Concat YOLO head b16 [16,144,8400]", [16, 144, 8400], 8 * whole.numel(),
        lambda w=whole: L.nb2_concat_split(dev, 1, p(w), c_parts, i64s([6400, 1600, 400]), 3, 16 * 144, 1, 4))
    # elementwise: residual Add, score Sigmoid
    a11, b11 = rnd(64, 128, 28, 28), rnd(64, 128, 28, 28)
    y11 = torch.empty_like(a11)
    add("Add ResNet bs64 [64,128,28,28]", list(a11.shape), 12 * a11.numel(),
        lambda a=a11, b=b11, y=y11: L.nb2_binary(dev, 0, 0, p(a), i64s(a.shape), 4, p(b), i64s(b.shape), 4, p(y),
                                                 i64s(y.shape), 4))
    x12 = rnd(16, 80, 8400)
    y12 = torch.empty_like(x12)
    add("Sigmoid YOLO b16 scores", list(x12.shape), 8 * x12.numel(),
        lambda x=x12, y=y12: L.nb2_unary(dev, 1, p(x), p(y), x.numel()))

    peak, src = hbm_peak()
    out = []
    torch.cuda.synchronize()
    for name, shape, nbytes, fn in rows:
        with torch.cuda.stream(stream):
            for _ in range(warm):
                _lib.check(fn())
            evs = []
            for _ in range(reps):
                # flush L2: write 256 MB, then read it back so the lines the
                # row's reads evict are clean (no write-back inside its time)
                flush.zero_()
                flush_sum.copy_(flush.sum())
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                _lib.check(fn())
                e.record(stream)
                evs.append((s, e))
        _lib.check(L.nb2_device_synchronize(dev))
        torch.cuda.synchronize()
        us = 1000.0 * sum(s.elapsed_time(e) for s, e in evs) / reps
        gbs = nbytes / (us * 1e-6) / 1e9
        out.append({"row": name, "shape": shape, "bytes": int(nbytes), "us": round(us, 2), "gbs": round(gbs, 1),
                    "frac": round(gbs / peak, 3), "peak_gbs": peak, "peak_note": src})
    del flush
    return out


# ---- B200 leg ------------------------------------------------------------------------

def run_conv(args, local):
    """One Conv(+Relu) of the given geometry as an engine graph, timed like
    the sweep: CUDA-graph replays, L2 flushed between them (also the target
    for the committed ncu captures of single contraction launches)."""
    import math

    import torch

    from nert_b200 import model as nbm
    from nert_b200 import synth
    from nert_b200.onnx_io import FLOAT, Graph

    c, h, w, m, k, st, pd = (int(v) for v in args.conv.split(","))
    n = args.batch
    g = Graph(opset=13)
    x = g.add_input("x", [n, c, h, w])
    wt = synth.normal((m, c, k, k), math.sqrt(2.0 / (c * k * k)), synth.seed_of("bench_conv", "w"))
    bi = synth.normal((m,), 0.1, synth.seed_of("bench_conv", "b"))
    y = g.op("Relu", [g.op("Conv", [x, g.const("w", wt), g.const("b", bi)], name="conv", kernel_shape=[k, k],
                           strides=[st, st], pads=[pd] * 4)], name="relu")
    g.add_output(y, None, FLOAT)
    feed = {"x": synth.uniform((n, c, h, w), -1.0, 1.0, synth.seed_of("bench_conv", "x"))}
    mdl = nbm.Model(g, {"x": [n, c, h, w]}, device=local)
    mdl.run(feed)
    flops = sum(contraction_flops(g, nbm.analyze(g, {"x": [n, c, h, w]})).values())
    stream = torch.cuda.ExternalStream(mdl.stream(), device=torch.device("cuda", local))
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    evs = []
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            mdl.launch()
        for _ in range(args.steps):
            flush.zero_()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            mdl.launch()
            e0.record(stream)
            evs.append((s0, e0))
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
    rows = {lab: t for lab, t in mdl.profile()}
    kpr = mdl.stats()["kernels_per_run"]
    mdl.close()
    peak, note = tensor_peak(args.precision)
    print(json.dumps({"metric": metric_for("conv", n), "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (3xTF32)",
                      "data": "synthetic", "config": {"workload": "conv", "batch": n, "conv": args.conv,
                                                      "l2": "flushed between timed steps"},
                      "rows_ms": rows, "roofline": {"bound": "tensor", "peak": peak, "peak_note": note,
                                                    "frac": flops / (ms * 1e-3) / 1e12 / peak},
                      "gpu_launches": kpr * args.steps}), flush=True)
    return 0


def run_attention(args, local):
    """The ViT-B/16 attention chain (QK^T, / 8, Softmax, AV, head merge) of
    `--batch` images x 12 heads x 197 tokens as an engine graph, which the
    engine fuses into one attention step; timed like the conv workload (also
    the target of the committed ncu capture of that kernel)."""
    import numpy as np
    import torch

    from nert_b200 import model as nbm
    from nert_b200 import synth
    from nert_b200.onnx_io import FLOAT, Graph

    B, H, T, D = args.batch, 12, 197, 64
    g = Graph(opset=13)
    q = g.add_input("q", [B, H, T, D])
    k = g.add_input("k", [B, H, D, T])
    v = g.add_input("v", [B, H, T, D])
    sc = g.op("Div", [g.op("MatMul", [q, k], name="qk"), g.const("c", np.array(8.0, np.float32))], name="sc")
    o = g.op("MatMul", [g.op("Softmax", [sc], name="sm", axis=-1), v], name="av")
    o = g.op("Reshape", [g.op("Transpose", [o], name="t", perm=[0, 2, 1, 3]),
                         g.const("m", np.array([B, T, H * D], np.int64))], name="merge")
    g.add_output(o, None, FLOAT)
    feed = {"q": synth.normal((B, H, T, D), 1.0, synth.seed_of("bench_attn", "q")),
            "k": synth.normal((B, H, D, T), 1.0, synth.seed_of("bench_attn", "k")),
            "v": synth.normal((B, H, T, D), 1.0, synth.seed_of("bench_attn", "v"))}
    mdl = nbm.Model(g, {n: list(a.shape) for n, a in feed.items()}, device=local)
    mdl.run(feed)
    stream = torch.cuda.ExternalStream(mdl.stream(), device=torch.device("cuda", local))
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    evs = []
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            mdl.launch()
        for _ in range(args.steps):
            flush.zero_()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            mdl.launch()
            e0.record(stream)
            evs.append((s0, e0))
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
    rows = {lab: t for lab, t in mdl.profile()}
    kpr = mdl.stats()["kernels_per_run"]
    mdl.close()
    flops = 4.0 * B * H * T * T * D
    peak, note = tensor_peak(args.precision)
    print(json.dumps({"metric": "fused attention TFLOP/s (ViT-B/16 heads, T=197, d=64)",
                      "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32 (3xTF32)", "data": "synthetic",
                      "config": {"workload": "attention", "batch": B, "heads": H, "tokens": T, "head_dim": D,
                                 "l2": "flushed between timed steps"},
                      "rows_ms": rows, "roofline": {"bound": "tensor", "peak": peak, "peak_note": note,
                                                    "frac": flops / (ms * 1e-3) / 1e12 / peak},
                      "gpu_launches": kpr * args.steps}), flush=True)
    return 0


def run_seam(args, local):
    """The workload through the drop-in boundary: the reference's unmodified
    LoadGraphFromFile -> nert::Model -> Run (compiled from its sources into
    oracle/_ref) on nert::b200::Device(local). Every Run stages the input from
    host memory, runs node by node through the seam rows and copies the output
    back; timed with CUDA events on the device's stream around each Run."""
    import ctypes

    import torch

    from nert_b200 import _lib, onnx_io
    from oracle import ref

    if not ref.available() or not os.path.exists(_lib.DEVICE_LIB_PATH):
        print(json.dumps({"metric": metric_for(args.workload, args.batch), "unavailable":
                          "the reference library or the device plug-in was not built"}))
        return 0
    ref.lib()
    L = _lib.lib()
    dl = ctypes.CDLL(_lib.DEVICE_LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    dl.nb2_nert_device.restype = ctypes.c_void_p
    dl.nb2_nert_device.argtypes = [ctypes.c_int]
    handle = dl.nb2_nert_device(local)
    graph, feeds = build_workload(args.workload, args.batch)
    tmp = tempfile.TemporaryDirectory()
    path = onnx_io.save(graph, os.path.join(tmp.name, "model.onnx"))
    m = ref.RefModel(path, {k: list(v.shape) for k, v in feeds.items()}, handle)
    stream = torch.cuda.ExternalStream(L.nb2_device_stream(_lib.device(local)), device=torch.device("cuda", local))
    for _ in range(max(3, args.warmup)):
        m.run(feeds)
    evs, walls, runs = [], [], []
    for _ in range(args.steps):
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        t0 = time.perf_counter()
        out = m.run(feeds)
        walls.append(time.perf_counter() - t0)
        runs.append(m.last_ms)  # nert::Model::RunTyped alone (inputs already in its HostTensorMap)
        e0.record(stream)
        evs.append((s0, e0))
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
    wall_ms = 1000.0 * sum(walls) / len(walls)
    run_ms = sum(runs) / len(runs)
    m.close()
    tmp.cleanup()
    v = args.batch / (run_ms * 1e-3)
    print(json.dumps({
        "metric": metric_for(args.workload, args.batch), "value": v, "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": run_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (3xTF32 tensor-core contractions)",
        "timing": "value = batch / the wall time of nert::Model::RunTyped (host input -> staged upload -> rows -> "
                  "host output); event_ms_per_step brackets the whole call including the C shim's copy of the "
                  "input into the reference's HostTensorMap",
        "event_ms_per_step": ms,
        "data": "synthetic (seeded inputs, Kaiming / N(0,0.02) weights, BN folded)",
        "config": {"workload": args.workload, "per_gpu_batch": args.batch, "api": "seam",
                   "path": "reference LoadGraphFromFile -> nert::Model -> Run on nert::b200::Device (one row per "
                           "node, no fusion, no graph replay)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": int(sum(a.nbytes for a in feeds.values())),
                "d2h_bytes_per_step": int(sum(a.nbytes for a in out.values())), "ms_per_step": run_ms,
                "wall_ms_per_step": wall_ms},
        "gpu_launches": None}), flush=True)
    return 0


def run_sweep(args, local):
    """Config 1: every Conv shape at batch 32 and every Gemm shape, one row each."""
    import torch

    from nert_b200 import configs
    from nert_b200 import model as nbm

    stream_ops = []
    rows = []
    cases = [(n, *configs.sweep_conv(n, args.batch)) for n, *_ in configs.SWEEP_CONVS]
    cases += [(f"gemm_{m}x{n}x{k}", *configs.sweep_gemm(m, n, k)) for m, n, k in configs.SWEEP_GEMMS]
    for name, g, feeds in cases:
        m = nbm.Model(g, {k: list(v.shape) for k, v in feeds.items()}, device=local)
        m.run(feeds)
        flops = sum(contraction_flops(g, nbm.analyze(g, {k: list(v.shape) for k, v in feeds.items()})).values())
        stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))
        flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
        evs = []
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                m.launch()
            for _ in range(args.steps):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                m.launch()
                e.record(stream)
                evs.append((s, e))
        torch.cuda.synchronize()
        ms = sum(s.elapsed_time(e) for s, e in evs) / len(evs)
        rows.append({"op": name, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "gflop": flops / 1e9,
                     "kernels_per_run": m.stats()["kernels_per_run"]})
        stream_ops.append(m.stats()["kernels_per_run"] * args.steps)
        del flush
        m.close()
    tf32 = measure_tf32_peak()
    total_ms = sum(r["ms"] for r in rows)
    total_flop = sum(r["gflop"] for r in rows) * 1e9
    line = {
        "metric": metric_for("sweep", args.batch), "value": total_flop / (total_ms * 1e-3) / 1e12,
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (3xTF32 tensor-core contractions, fp32 accumulate)" if args.precision == "3xtf32"
        else "f32 (1xTF32 contractions, opt-in)",
        "data": "synthetic (seeded N(0,1) data, N(0,1)/sqrt(fan_in) weights)",
        "config": {"workload": "sweep", "conv_batch": args.batch, "precision": args.precision,
                   "l2": "flushed between timed steps"},
        "ops": rows,
        "roofline": {"bound": "tensor", "peak": tensor_peak(args.precision)[0], "unit": "TFLOP/s",
                     "peak_note": tensor_peak(args.precision)[1], "tf32_dense_live": tf32,
                     "achieved": total_flop / (total_ms * 1e-3) / 1e12,
                     "frac": total_flop / (total_ms * 1e-3) / 1e12 / tensor_peak(args.precision)[0]},
        "gpu_launches": int(sum(stream_ops)),
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    rank, world, local = dist_env()

    cpu = None
    if (rank == 0 and world == 1 and not args.no_cpu_baseline
            and args.workload not in ("sweep", "conv", "rows", "attention")
            and args.api == "engine"):
        from oracle import ref

        if ref.available():
            cpu = {"pool": RefPool(ref_cores(), args.workload)}  # spawned before the first GPU call

    import numpy as np
    import torch

    if args.precision == "1xtf32":
        os.environ["NERT_B200_PRECISION"] = "1xtf32"
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local)

    if args.workload == "sweep":
        return run_sweep(args, local)
    if args.workload == "conv":
        return run_conv(args, local)
    if args.workload == "attention":
        return run_attention(args, local)
    if args.workload == "rows":
        # the HBM-bound rows alone (also the target of their committed ncu
        # captures): --steps timed launches per row after --warmup untimed
        rows = bandwidth_rows(local, reps=args.steps, warm=args.warmup)
        print(json.dumps({"metric": "HBM-bound rows: algorithmic GB/s", "unit": "GB/s", "n_gpus": 1,
                          "steps": args.steps, "warmup": args.warmup, "data": "synthetic",
                          "config": {"workload": "rows", "l2": "flushed before each launch"},
                          "bandwidth_rows": rows}), flush=True)
        return 0
    if args.api == "seam":
        return run_seam(args, local)

    from nert_b200 import model as nbm

    # this rank's slice of one seeded global batch, by the library's shard
    # plan (weak scaling: batch per GPU fixed; strong: the global batch fixed)
    from nert_b200.sharding import rank_slice

    strong = args.global_batch is not None
    global_batch = args.global_batch if strong else args.batch * world
    my_rows = rank_slice(global_batch, rank, world)
    batch = my_rows.stop - my_rows.start
    graph, feeds = build_workload(args.workload, global_batch, my_rows)
    dims = {k: list(v.shape) for k, v in feeds.items()}
    m = nbm.Model(graph, dims, device=local)
    stats = m.stats()
    h_in = []
    for io in m.inputs:
        hb = nbm.HostBuffer(io["shape"], io["dtype"])
        hb.array[...] = feeds[io["name"]]
        h_in.append(hb)
    h_out = [nbm.HostBuffer(io["shape"], io["dtype"]) for io in m.outputs]
    in_ptrs, out_ptrs = [b.ptr for b in h_in], [b.ptr for b in h_out]
    m.run_into(in_ptrs, out_ptrs)  # stages the inputs, captures the CUDA graph

    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MB > 126 MB L2

    def barrier():
        if dist is not None:
            dist.barrier()

    def timed(fn, steps):
        evs = []
        with torch.cuda.stream(stream):
            for _ in range(steps):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                fn()
                e.record(stream)
                evs.append((s, e))
        torch.cuda.synchronize()
        stream.synchronize()
        return [s.elapsed_time(e) for s, e in evs]

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            m.launch()
            m.run_async(in_ptrs, out_ptrs)
    m.synchronize()
    torch.cuda.synchronize()

    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    dev_ms = timed(m.launch, args.steps)
    m.synchronize()
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    # end to end: one timed region over all steps (each step's host->device
    # copy runs on the engine's copy stream and overlaps the previous step's
    # forward, so per-step events would not bracket it); L2 is flushed inside
    # the region before every step
    torch.cuda.synchronize()
    m.synchronize()
    with torch.cuda.stream(stream):
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        for _ in range(args.steps):
            flush.zero_()
            m.run_async(in_ptrs, out_ptrs)
        r1.record(stream)
    m.synchronize()
    torch.cuda.synchronize()
    barrier()

    # the opt-in 1xTF32 mode on the same model, reported apart (one GPU):
    # the graph is recaptured for the other precision, then timed the same way
    tf32_1x = None
    if world == 1 and args.precision == "3xtf32":
        from nert_b200 import _lib

        hdev = _lib.device(local)
        _lib.check(_lib.lib().nb2_device_set_precision(hdev, 1))  # NB2_PREC_1XTF32
        try:
            with torch.cuda.stream(stream):
                for _ in range(max(3, args.warmup)):
                    m.launch()
            m.synchronize()
            ms1 = timed(m.launch, args.steps)
            m.synchronize()
        finally:
            _lib.check(_lib.lib().nb2_device_set_precision(hdev, 0))  # NB2_PREC_3XTF32
        t1 = sum(ms1) / len(ms1)
        tf32_1x = {"value": global_batch / (t1 * 1e-3), "unit": UNIT, "ms_per_step": t1,
                   "note": "opt-in 1xTF32 (one tf32 product per multiply-add, not fp32-accurate), same model and "
                           "timing as `value`, reported apart from the fp32 (3xTF32) headline"}

    mean_dev = sum(dev_ms) / len(dev_ms)
    mean_e2e = r0.elapsed_time(r1) / args.steps
    if dist is not None:
        t = torch.tensor([mean_dev, mean_e2e], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mean_dev, mean_e2e = float(t[0]), float(t[1])

    # roofline of the tensor-core contraction kernel (eager passes, event per row)
    analysis = nbm.analyze(graph, dims)
    flops = contraction_flops(graph, analysis)
    cbytes = contraction_bytes(graph, analysis)
    sums = {}
    reps = 3
    for _ in range(reps):
        for label, ms in m.profile():
            sums[label] = sums.get(label, 0.0) + ms / reps
    tc_eager = sum(ms for lab, ms in sums.items() if row_name(lab) in flops)
    tc_flop = sum(flops.values())
    total_prof = sum(sums.values())
    # the contraction rows' share of the eager pass applied to the timed
    # CUDA-graph replay: the kernel's time inside the step that `value` times
    share = tc_eager / total_prof if total_prof else 0.0
    tc_time = mean_dev * share
    achieved = tc_flop / (tc_time * 1e-3) / 1e12 if tc_time > 0 else None
    top_rows = sorted(sums.items(), key=lambda kv: -kv[1])[:5]
    by_op = {}
    for lab, ms in sums.items():
        op = lab.split(":", 1)[0]
        if "MatMul" in op:  # attention products apart from the linear layers
            nm = row_name(lab)
            op += " (attention)" if (".qk" in nm or ".av" in nm or "attn" in nm) else ""
        by_op[op] = round(by_op.get(op, 0.0) + ms, 4)
    # the fused attention step (its two contractions, 4*B*H*T^2*D FLOP, plus
    # the softmax), reported apart from the contraction kernel's roofline
    attn = None
    attn_flop = 0.0
    for e in analysis["exec"]:
        if e["op"] == "Attention":
            b_, h_, t_, d_ = analysis["tensors"][e["ins"][0]]["dims"]
            attn_flop += 4.0 * b_ * h_ * t_ * t_ * d_
    if attn_flop:
        a_eager = sum(ms for lab, ms in sums.items() if lab.startswith("Attention:"))
        a_time = mean_dev * (a_eager / total_prof if total_prof else 0.0)
        a_tf = attn_flop / (a_time * 1e-3) / 1e12 if a_time > 0 else None
        attn = {"kernel": "attention_kernel (fused QK^T, scale, softmax, PV on tcgen05, 3xTF32)",
                "flops_per_step": attn_flop, "kernel_ms_per_step": a_time, "achieved": a_tf,
                "unit": "TFLOP/s", "frac": (a_tf / tensor_peak(args.precision)[0]) if a_tf else None,
                "note": "FLOPs of the two contractions only; the softmax between them runs on the CUDA cores"}
    rows_table = bandwidth_rows(local) if (rank == 0 and world == 1 and not args.no_rows) else None

    line = None
    if rank == 0:
        tf32 = measure_tf32_peak()
        peak, peak_note = tensor_peak(args.precision)
        line = {
            "metric": metric_for(args.workload, batch),
            "value": global_batch / (mean_dev * 1e-3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": mean_dev,
            "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "f32 (3xTF32 tensor-core contractions, fp32 accumulate)" if args.precision == "3xtf32"
            else "f32 (1xTF32 contractions, opt-in)",
            "data": "synthetic (seeded inputs, Kaiming / N(0,0.02) weights, BN folded)",
            "config": {"workload": args.workload, "model": args.workload, "per_gpu_batch": batch,
                       "global_batch": global_batch, "parallelism": f"batch-sharded x{world} (no collective)",
                       "shard": "rank r runs its slice of one seeded global batch (library shard plan)",
                       "l2": "flushed (256 MB write) between timed steps, outside the step events",
                       "precision": args.precision, "cuda_graph": True,
                       "fused_groups": stats["fused_groups"], "rows_per_run": stats["exec_nodes"]},
            "e2e": {"value": global_batch / (mean_e2e * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": int(sum(b.nbytes for b in h_in)),
                    "d2h_bytes_per_step": int(sum(b.nbytes for b in h_out)), "ms_per_step": mean_e2e,
                    "timing": "one CUDA-event region over all steps of Model.run_async from pinned host buffers: "
                              "each step's input copy (on the engine's copy stream, overlapping the previous "
                              "step's forward), the forward and the output copy; L2 flushed inside the region "
                              "before every step"},
            "roofline": {"bound": "tensor", "kernel": "igemm_kernel (tcgen05 implicit-GEMM Conv/Gemm/MatMul)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved / peak) if achieved else None,
                         "peak_note": peak_note,
                         "tf32_dense_live": tf32,
                         "frac_of_tf32_dense_live": (achieved / tf32) if achieved else None,
                         "flops_per_step": tc_flop, "kernel_ms_per_step": tc_time,
                         "share_of_step": share,
                         "kernel_ms_note": "ms_per_step (timed CUDA-graph replay) x the contraction rows' share "
                                           "of an eager pass with an event between rows",
                         "kernel_ms_eager": tc_eager,
                         "per_layer": layer_roofline(sums, flops, cbytes, tensor_peak(args.precision)[0],
                                                     hbm_peak()[0]),
                         "traffic": TRAFFIC_BYTES.get((args.workload, batch)),
                         "traffic_note": "DRAM bytes read+written by the contraction launches of one step, "
                                         "from one ncu capture (profiles/resnet18_b64_igemm_dram.md)"
                         if (args.workload, batch) in TRAFFIC_BYTES else None},
            "attention": attn,
            "tf32_1x": tf32_1x,
            "top_rows_ms": [[lab, round(ms, 4)] for lab, ms in top_rows],
            "profile_ms_by_op": by_op,
            "bandwidth_rows": rows_table,
            "clocks": clk,
            "gpu_launches": int(stats["kernels_per_run"]) * args.steps * world,
        }
    del flush
    m.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()

    if rank == 0 and cpu is not None:
        pool = cpu["pool"]
        try:
            pool.step()  # warm
            walls = [pool.step() for _ in range(1 if args.workload != "resnet18" else 2)]
        finally:
            pool.close()
        v = pool.cores * len(walls) / sum(walls)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": pool.cores, "kind": "reference",
                                "sample": f"{len(walls)} x {pool.cores} {args.workload} images (batch 1, one "
                                          "process per core)"}
    elif rank == 0:
        line["cpu_baseline"] = None
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
