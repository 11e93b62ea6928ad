"""The drop-in boundary: the reference's own, unmodified host path
(nert::LoadGraphFromFile -> nert::Model -> Run, compiled from the reference
sources into oracle/_ref/libnert_ref.so) running on nert::b200::Device(0)
from libnert_b200_device.so, compared with the same graph on
nert::CpuDevice(). Mirrors the reference's CUDA parity tests
(test/cuda_kernels_test.cpp:142-178, test/cuda_conv_test.cpp:182-213), with
the north-star bound max|err| <= 1e-4 * max|ref|.
"""

import ctypes
import os

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import _lib, configs, synth
from nert_b200.onnx_io import FLOAT, Graph
from oracle import ref

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built")]


@pytest.fixture(scope="module")
def b200_device(cuda):
    ref.lib()  # the reference library first: the plug-in binds to its nert::Model
    _lib.lib()
    if not os.path.exists(_lib.DEVICE_LIB_PATH):
        pytest.fail("libnert_b200_device.so was not built (needs the NERT headers at build time)")
    dl = ctypes.CDLL(_lib.DEVICE_LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    dl.nb2_nert_device.restype = ctypes.c_void_p
    dl.nb2_nert_device.argtypes = [ctypes.c_int]
    h = dl.nb2_nert_device(0)
    assert h, _lib.lib().nb2_last_error().decode()
    return h


def both(graph, inputs, dev):
    cpu = ref.run_graph(graph, inputs)
    gpu = ref.run_graph(graph, inputs, device=dev)
    return cpu, gpu


def test_model_conv_golden(b200_device):
    """cuda_conv_test.cpp:182 ModelConvMatchesCpu: weights and bias as graph inputs."""
    g = Graph(opset=13)
    for n, d in (("x", [1, 1, 3, 3]), ("w", [1, 1, 3, 3]), ("b", [1])):
        g.add_input(n, d)
    y = g.op("Conv", ["x", "w", "b"], name="cv", pads=[1, 1, 1, 1])
    g.add_output(y, None, FLOAT)
    ins = {"x": np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3), "w": np.ones((1, 1, 3, 3), np.float32),
           "b": np.array([10.0], np.float32)}
    cpu, gpu = both(g, ins, b200_device)
    np.testing.assert_array_equal(list(cpu.values())[0].ravel(), [22, 31, 26, 37, 55, 43, 34, 49, 38])
    np.testing.assert_allclose(list(gpu.values())[0], list(cpu.values())[0], rtol=1e-6)


def test_micro_graph_gemm_relu_add(b200_device):
    """cuda_kernels_test.cpp:142 MicroGraphMatchesCpuWithinTolerance shape: Gemm -> Relu -> Add."""
    g = Graph(opset=13)
    g.add_input("a", [8, 16])
    w = g.const("w", synth.normal((16, 12), 0.3, 5))
    c = g.const("c", synth.normal((12,), 1.0, 6))
    t = g.op("Relu", [g.op("Gemm", ["a", w, c], name="gemm")], name="relu")
    y = g.op("Add", [t, g.const("bias", synth.normal((12,), 1.0, 7))], name="add")
    g.add_output(y, None, FLOAT)
    ins = {"a": synth.normal((8, 16), 1.0, 8)}
    cpu, gpu = both(g, ins, b200_device)
    assert rel_err(list(gpu.values())[0], list(cpu.values())[0]) <= TOL


def test_resnet18_through_reference_executor(b200_device):
    g = configs.resnet18(2)
    x = configs.resnet_input(2)
    cpu, gpu = both(g, {"input": x}, b200_device)
    assert rel_err(gpu["fc_out"], cpu["fc_out"]) <= TOL


def test_unknown_op_names_node_and_op(b200_device):
    """The executor rejects an op with no row, naming node and op
    (src/executor.cpp:485-488); there is no CPU fallback."""
    g = Graph(opset=13)
    g.add_input("x", [4])
    y = g.op("Cos", ["x"], name="trig")
    g.add_output(y, None, FLOAT)
    with pytest.raises(RuntimeError) as e:
        ref.run_graph(g, {"x": np.ones(4, np.float32)}, device=b200_device)
    assert "Cos" in str(e.value) and "trig" in str(e.value)


@pytest.mark.parametrize("config", ["resnet50", "vit_b16", "yolov8n"])
def test_config_through_reference_executor(b200_device, config):
    """Configs 2-4 at batch 1 through the reference loader and executor on the
    new handle (ViT-B/16 at opset 17 for LayerNormalization), against the
    numpy restatement of the reference CPU kernels (pinned to the reference
    library on these graphs by tests/test_oracle.py; the reference CpuDevice
    itself takes minutes on ViT-B/16)."""
    from oracle import np_ref

    g, name, x = {
        "resnet50": lambda: (configs.resnet50(1, expose_logits=True), "input", configs.resnet_input(1, "resnet50")),
        "vit_b16": lambda: (configs.vit_b16(1), "input", configs.vit_input(1)),
        "yolov8n": lambda: (configs.yolov8n(1, expose_scores=True), "images", configs.yolo_input(1)),
    }[config]()
    want = np_ref.run(g, {name: x})
    gpu = ref.run_graph(g, {name: x}, device=b200_device)
    if config != "yolov8n":
        for out in want:
            assert rel_err(gpu[out], want[out]) <= TOL, (config, out)
        return
    for out in ("scores.flat_out", "boxes_out", "topk_out0"):
        assert rel_err(gpu[out], want[out]) <= TOL, out
    # TopK bit-exact on the scores this run computed; the Gather and the
    # class ids exact given those indices; picks that differ from the
    # oracle's are near ties in value
    scores, boxes, idx = gpu["scores.flat_out"][0], gpu["boxes_out"][0], gpu["topk_out1"][0]
    order = np.lexsort((np.arange(scores.size), -scores.astype(np.float64)))[:300]
    np.testing.assert_array_equal(idx, order)
    np.testing.assert_array_equal(gpu["class_idx_out"][0], order % 80)
    np.testing.assert_array_equal(gpu["det_boxes_out"][0], boxes[:, order // 80].T)
    same = idx == want["topk_out1"][0]
    scale = float(np.abs(want["topk_out0"]).max())
    assert np.all(np.abs(gpu["topk_out0"][0][~same] - want["topk_out0"][0][~same]) <= TOL * scale)


def test_resident_weights_are_packed_once_and_dropped_on_release(b200_device):
    """Conv/Gemm weights are packed for the tensor cores on first use and
    reused on later Runs; a second model loaded into the released memory gets
    its own packing (its weights differ), so results never go stale."""
    from nert_b200 import onnx_io

    x = configs.resnet_input(1)
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        outs = {}
        for tag in ("resnet18", "other"):
            g = configs.resnet18(1, config=tag)
            path = onnx_io.save(g, os.path.join(d, f"{tag}.onnx"))
            m = ref.RefModel(path, {"input": [1, 3, 224, 224]}, b200_device)
            try:
                first = m.run({"input": x})["fc_out"]
                again = m.run({"input": x})["fc_out"]
            finally:
                m.close()
            np.testing.assert_array_equal(first, again)
            cpu = ref.run_graph(g, {"input": x})["fc_out"]
            assert rel_err(first, cpu) <= TOL, tag
            outs[tag] = first
    assert np.abs(outs["resnet18"] - outs["other"]).max() > 1e-3


@pytest.mark.skipif(not ref.available(cuda=True), reason="reference CUDA library not built")
def test_reference_cuda_baseline_matches_oracle(cuda):
    """The GPU baseline (the reference's own CudaDevice: cuDNN Conv, cuBLAS
    Gemm) agrees with the oracle on ResNet-18, so its timings are of a correct
    run."""
    from oracle import np_ref

    g = configs.resnet18(1)
    x = configs.resnet_input(1)
    got = ref.run_graph(g, {"input": x}, cuda=True)["fc_out"]
    assert rel_err(got, np_ref.run(g, {"input": x})["fc_out"]) <= TOL


def test_average_pool_row_through_reference_executor(b200_device):
    """The AveragePool row on the new handle, SAME_UPPER padding resolved as
    the reference does, bit-exact with the reference CpuDevice."""
    g = Graph(opset=13)
    g.add_input("x", [2, 8, 14, 13])
    y = g.op("AveragePool", ["x"], name="pool", kernel_shape=[5, 5], strides=[3, 3], auto_pad="SAME_UPPER",
             count_include_pad=1)
    g.add_output(y, None, FLOAT)
    cpu, gpu = both(g, {"x": synth.normal((2, 8, 14, 13), 1.0, 77)}, b200_device)
    np.testing.assert_array_equal(list(gpu.values())[0], list(cpu.values())[0])


def test_conv_transpose_row_through_reference_executor(b200_device):
    """The ConvTranspose row on the new handle against the reference CpuDevice."""
    g = Graph(opset=13)
    g.add_input("x", [2, 16, 9, 11])
    w = g.const("w", synth.normal((16, 8, 3, 3), 0.25, 81))
    y = g.op("ConvTranspose", ["x", w], name="ct", strides=[2, 2], pads=[1, 0, 1, 0], output_padding=[1, 1])
    g.add_output(y, None, FLOAT)
    cpu, gpu = both(g, {"x": synth.normal((2, 16, 9, 11), 1.0, 82)}, b200_device)
    assert rel_err(list(gpu.values())[0], list(cpu.values())[0]) <= TOL


def test_reference_constant_folding_with_b200_rows(b200_device):
    """nert::FoldConstants (src/constant_folding.cpp:32-95) runs each
    all-constant node with the given device's rows on the initializers' HOST
    bytes. With the B200 handle the rows stage those views through HBM, so
    folding with it gives the graph the CPU fold gives, within the north-star
    bound (the folded MatMul runs on the tensor cores)."""
    g = Graph(opset=13)
    g.add_input("x", [2, 8, 6, 6])
    a = g.const("a", synth.normal((8,), 1.0, 91))
    b = g.const("b", synth.normal((8,), 1.0, 92))
    s = g.op("Add", [a, b], name="fold_add")
    s = g.op("Mul", [s, b], name="fold_mul")
    s = g.op("Relu", [s], name="fold_relu")
    p = g.const("p", synth.normal((8, 64), 0.3, 93))
    q = g.const("q", synth.normal((64, 8), 0.3, 94))
    m = g.op("MatMul", [p, q], name="fold_matmul")
    w = g.const("w", synth.normal((8, 8, 3, 3), 0.2, 95))
    y = g.op("Conv", ["x", w, s], name="cv", pads=[1, 1, 1, 1])
    y = g.op("Add", [y, g.const("shape4", np.ones((1, 8, 1, 1), np.float32))], name="y_add")
    y = g.op("Reshape", [y, g.const("rs", np.array([2, 8, 36], np.int64))], name="rs")
    y = g.op("MatMul", [m, y], name="mix")
    g.add_output(y, None, FLOAT)
    x = synth.normal((2, 8, 6, 6), 1.0, 96)
    import tempfile

    from nert_b200 import onnx_io

    with tempfile.TemporaryDirectory() as d:
        path = onnx_io.save(g, os.path.join(d, "model.onnx"))
        plain = ref.RefModel(path, {"x": [2, 8, 6, 6]})
        cpu_fold = ref.RefModel(path, {"x": [2, 8, 6, 6]}, fold=True)
        b200_fold = ref.RefModel(path, {"x": [2, 8, 6, 6]}, fold=True, fold_device=b200_device)
        try:
            assert cpu_fold.folded == b200_fold.folded == 4
            want = list(plain.run({"x": x}).values())[0]
            via_cpu = list(cpu_fold.run({"x": x}).values())[0]
            via_b200 = list(b200_fold.run({"x": x}).values())[0]
        finally:
            for mdl in (plain, cpu_fold, b200_fold):
                mdl.close()
    np.testing.assert_array_equal(via_cpu, want)
    assert rel_err(via_b200, want) <= TOL


def test_reference_runtime_bench_harness_on_b200(cuda):
    """The reference's own runtime bench harness (bench/runtime/main.cpp,
    compiled unchanged by `make -C oracle bench_runtime`, its CUDA slot given
    the B200 handle): every op case it runs on the device matches its
    CpuDevice result within the harness's own tolerance, and it exits 0."""
    import subprocess

    exe = os.path.join(os.path.dirname(ref.__file__), "_ref", "nert_bench_runtime_b200")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/nert_bench_runtime_b200 was not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    rows = [ln for ln in out.splitlines() if " CUDA " in ln]
    assert rows and not any("FAIL" in ln for ln in rows), out[-3000:]
    assert any(ln.startswith("PASSED") for ln in out.splitlines()), out[-3000:]
