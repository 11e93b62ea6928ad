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
