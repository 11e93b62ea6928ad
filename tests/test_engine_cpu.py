"""Host-side checks of the B200 engine that need no GPU.

* libnert_b200.so loads and exports every entry point include/nert_b200.h
  declares (no compute call is made without a GPU);
* the C++ ONNX reader + shape inference agree with the reference's output
  shapes, and the fusion peephole groups exactly the expected epilogues;
* the arena plan never lets two simultaneously-live tensors overlap and
  never places a row's output over one of its inputs (the reference
  planner's guarantee, src/memory_planner.cpp:5-16, test
  memory_planner_test.cpp:415 OutputNeverAliasesItsInput);
* malformed graphs are rejected with the node named.
"""

import ctypes
import os
import re

import numpy as np
import pytest

from nert_b200 import _lib, configs, onnx_io
from nert_b200 import model as nbm
from nert_b200 import sharding  # noqa: F401  (binds the nb2_shard* entry points)
from nert_b200.onnx_io import FLOAT, Graph

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "nert_b200.h")).read()
    return sorted(set(re.findall(r"\b(nb2_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    bound = set(_lib._SIGS)
    assert set(header_symbols()) <= bound


def test_error_reporting_without_gpu():
    lib = _lib.lib()
    h = ctypes.c_void_p()
    # no CUDA device in this container: a clean error status, not a crash
    st = lib.nb2_device_open(0, ctypes.byref(h))
    if st != 0:
        assert lib.nb2_last_error().decode()


def _intervals(a):
    t = a["tensors"]
    defs = {}
    for i, e in enumerate(a["exec"]):
        if e["alias"]:
            continue
        for o in e["outs"]:
            defs.setdefault(t[o]["root"], i)
    iv = {}
    for name, info in t.items():
        r = info["root"]
        if info["offset"] < 0 or r in iv or r not in defs:
            continue
        start = defs[r]
        end = max(start, info["last_use"]) if info["last_use"] >= 0 else start
        size = (t[r]["bytes"] + 255) // 256 * 256 or 256
        iv[r] = (start, end, t[r]["offset"], size)
    return iv


@pytest.mark.parametrize("builder,batch,fused", [(configs.resnet18, 64, 17), (configs.resnet50, 32, 49)],
                         ids=["resnet18_b64", "resnet50_b32"])
def test_plan_has_no_live_overlap(builder, batch, fused):
    g = builder(batch)
    a = nbm.analyze(g, {"input": [batch, 3, 224, 224]})
    assert a["fused_groups"] == fused
    iv = _intervals(a)
    roots = list(iv)
    for i in range(len(roots)):
        s1, e1, o1, b1 = iv[roots[i]]
        for j in range(i + 1, len(roots)):
            s2, e2, o2, b2 = iv[roots[j]]
            if s1 <= e2 and s2 <= e1:  # live at the same time
                assert o1 + b1 <= o2 or o2 + b2 <= o1, (roots[i], roots[j])
    assert a["arena"] <= nbm.analyze(g, {"input": [batch, 3, 224, 224]}, flags=nbm.NO_FUSION)["arena"]


def test_output_shape_matches_reference_and_order():
    g = configs.resnet18(8)
    a = nbm.analyze(g, {"input": [8, 3, 224, 224]})
    assert a["tensors"]["fc_out"]["dims"] == [8, 1000]
    names = [e["name"] for e in a["exec"]]
    # a downsample conv must run before the conv that fuses the residual it feeds
    assert names.index("layer2.0.downsample") < names.index("layer2.0.conv2")
    fused = {e["name"]: e for e in a["exec"]}
    assert fused["layer2.0.conv2"]["residual"] == "layer2.0.downsample_out"
    assert fused["layer2.0.conv2"]["act"] == 1
    assert fused["conv1"]["act"] == 1 and fused["conv1"]["group"] == 2


def test_silu_and_matmul_bias_fusion():
    g = Graph(opset=13)
    x = g.add_input("x", [2, 8, 6, 6])
    w = g.const("w", np.ones((4, 8, 1, 1), np.float32))
    c = g.op("Conv", [x, w], name="c")
    s = g.op("Sigmoid", [c], name="s")
    m = g.op("Mul", [c, s], name="m")
    f = g.op("Reshape", [m, g.const("shape", np.array([2, -1], np.int64))], name="r")
    mm = g.op("MatMul", [f, g.const("wm", np.ones((144, 5), np.float32))], name="mm")
    y = g.op("Add", [mm, g.const("b", np.ones((5,), np.float32))], name="add")
    g.add_output(y, None, FLOAT)
    a = nbm.analyze(g, {"x": [2, 8, 6, 6]})
    ops = {e["name"]: e for e in a["exec"]}
    assert ops["c"]["act"] == 2 and ops["c"]["group"] == 3
    assert ops["mm"]["bias"] == "b"
    assert a["fused_groups"] == 2
    assert ops["r"]["alias"]


def test_unknown_op_is_rejected_naming_the_node():
    g = Graph(opset=13)
    x = g.add_input("x", [2, 3])
    y = g.op("HardSwish", [x], name="mystery")
    g.add_output(y, None, FLOAT)
    with pytest.raises(_lib.NB2Error) as e:
        nbm.analyze(g, {"x": [2, 3]})
    assert "mystery" in str(e.value) and "HardSwish" in str(e.value)
    assert e.value.status == _lib.ERR_INVALID


def test_malformed_onnx_is_rejected():
    with pytest.raises(_lib.NB2Error):
        nbm.analyze(b"\x0a\x05garbage-not-protobuf", {"x": [1]})


def test_missing_input_shape_is_rejected():
    g = configs.resnet18(1)
    with pytest.raises(_lib.NB2Error) as e:
        nbm.analyze(g, {})
    assert "input" in str(e.value)


def test_onnx_file_roundtrip_through_engine_reader(tmp_path):
    g = configs.resnet18(2)
    p = onnx_io.save(g, str(tmp_path / "r18.onnx"))
    a = nbm.analyze(p, {"input": [2, 3, 224, 224]})
    assert a["opset"] == 13 and a["tensors"]["fc_out"]["dims"] == [2, 1000]


def test_vit_gelu_and_scale_fusion_plan():
    from nert_b200 import configs

    g = configs.vit_b16(2, layers=1)
    a = nbm.analyze(g, {"input": [2, 3, 224, 224]})
    rows = {e["name"]: e for e in a["exec"]}
    assert rows["blk0.fc1"]["group"] == 7 and rows["blk0.fc1"]["act"] == 4  # bias + erf-form GELU
    # QK^T, / sqrt(64), Softmax, AV and the head merge: one fused attention step
    assert rows["blk0.ctx"]["op"] == "Attention" and rows["blk0.ctx"]["group"] == 6
    assert not any(e["op"] in ("Erf", "Div", "Softmax", "MatMul") and e["name"].startswith("blk0.")
                   and e["name"] not in ("blk0.q", "blk0.k", "blk0.v", "blk0.proj", "blk0.fc1", "blk0.fc2")
                   for e in a["exec"])
    # without the fused step the scale is the QK^T contraction's epilogue alpha
    b = nbm.analyze(g, {"input": [2, 3, 224, 224]}, flags=nbm.NO_ATTENTION)
    rows = {e["name"]: e for e in b["exec"]}
    assert rows["blk0.qk"]["group"] == 2
    assert not any(e["op"] in ("Erf", "Div", "Attention") for e in b["exec"])


def test_vit_head_transposes_written_in_place_plan():
    """The head split (linear -> Reshape -> Transpose) and merge (MatMul ->
    Transpose) are absorbed: the contraction writes the transposed layout
    directly, so no Transpose row is left but the patch-embedding one."""
    from nert_b200 import configs

    g = configs.vit_b16(2, layers=2)
    a = nbm.analyze(g, {"input": [2, 3, 224, 224]}, flags=nbm.NO_ATTENTION)
    rows = {e["name"]: e for e in a["exec"]}
    for b in ("blk0", "blk1"):
        assert rows[f"{b}.q"]["group"] == 4 and rows[f"{b}.q"]["perm"] == [0, 2, 1, 3]
        assert rows[f"{b}.k"]["group"] == 4 and rows[f"{b}.k"]["perm"] == [0, 2, 3, 1]
        assert rows[f"{b}.v"]["group"] == 4 and rows[f"{b}.v"]["perm"] == [0, 2, 1, 3]
        assert rows[f"{b}.av"]["group"] == 2 and rows[f"{b}.av"]["perm"] == [0, 2, 1, 3]
    assert [e["name"] for e in a["exec"] if e["op"] == "Transpose"] == ["patch.tokens"]


def test_transpose_after_matmul_kept_when_not_a_head_split():
    """A Transpose whose permutation mixes a row axis into the columns in a
    way the output map cannot express stays a separate row."""
    from nert_b200 import synth
    from nert_b200.onnx_io import FLOAT, Graph

    g = Graph(opset=13)
    x = g.add_input("x", [6, 10, 24])
    y = g.op("MatMul", [x, g.const("w", synth.normal((24, 20), 0.1, 5))], name="mm")
    t = g.op("Transpose", [g.op("Reshape", [y, g.const("s", np.array([60, 4, 5], np.int64))], name="rs")],
             name="tr", perm=[2, 0, 1])
    g.add_output(t, None, FLOAT)
    a = nbm.analyze(g, {"x": [6, 10, 24]})
    # columns 20 = 4 x 5: inner block 5 is not a multiple of 16, so no map
    assert any(e["op"] == "Transpose" for e in a["exec"])


def test_batchnorm_folded_into_conv_at_load():
    """An export that keeps BatchNormalization after every Conv plans to the
    same rows as the folded graph (the reference loader rejects the op,
    src/model_loader.cpp:1677-1690; the engine folds it at load)."""
    dims = {"input": [2, 3, 224, 224]}
    a = nbm.analyze(configs.resnet18(2, bn_nodes=True), dims)
    b = nbm.analyze(configs.resnet18(2), dims)
    assert [e["op"] for e in a["exec"]] == [e["op"] for e in b["exec"]]
    assert "BatchNormalization" not in {e["op"] for e in a["exec"]}


def test_batchnorm_without_conv_stays_a_row():
    g = Graph(opset=13)
    g.add_input("x", [2, 5, 3, 4])
    r = g.op("Relu", ["x"], name="r")
    stats = [g.const(f"s{i}", np.full((5,), v, np.float32)) for i, v in enumerate((2.0, 0.5, 0.1, 3.0))]
    y = g.op("BatchNormalization", [r] + stats, name="bn", epsilon=1e-3)
    g.add_output(y, None, FLOAT)
    a = nbm.analyze(g, {"x": [2, 5, 3, 4]})
    assert [e["op"] for e in a["exec"]][-1] == "BatchNormalization"


def test_sppf_cascade_planned_as_one_pass():
    """YOLO's SPPF (three 5x5/s1 MaxPools and the Concat of the four tensors)
    plans as one SPPF step reading only the first tensor; the pools' outputs
    get no buffer."""
    g = configs.yolov8n(2)
    a = nbm.analyze(g, {"images": [2, 3, 640, 640]})
    sppf = [e for e in a["exec"] if e["op"] == "SPPF"]
    assert len(sppf) == 1 and sppf[0]["name"] == "sppf.cat" and sppf[0]["group"] == 4
    assert not any(e["name"].startswith("sppf.m") for e in a["exec"])


def test_sppf_not_fused_when_a_pool_output_has_another_reader():
    g = Graph(opset=13)
    x = g.add_input("x", [1, 4, 8, 8])
    m1 = g.op("MaxPool", [x], name="m1", kernel_shape=[5, 5], strides=[1, 1], pads=[2, 2, 2, 2])
    m2 = g.op("MaxPool", [m1], name="m2", kernel_shape=[5, 5], strides=[1, 1], pads=[2, 2, 2, 2])
    c = g.op("Concat", [x, m1, m2], name="cat", axis=1)
    g.add_output(c, None, FLOAT)
    g.add_output(g.op("Relu", [m1], name="side"), None, FLOAT)
    a = nbm.analyze(g, {"x": [1, 4, 8, 8]})
    assert not any(e["op"] == "SPPF" for e in a["exec"])
    # a stride-2 pool in the chain is not a "same" window either
    g2 = Graph(opset=13)
    x = g2.add_input("x", [1, 4, 8, 8])
    m1 = g2.op("MaxPool", [x], name="m1", kernel_shape=[3, 3], strides=[1, 1], pads=[1, 1, 1, 1])
    c = g2.op("Concat", [x, m1], name="cat", axis=1)
    g2.add_output(c, None, FLOAT)
    assert any(e["op"] == "SPPF" for e in nbm.analyze(g2, {"x": [1, 4, 8, 8]})["exec"])


def test_attention_fusion_limits():
    """The fused attention step needs head dim 64 and at most 208 tokens;
    other chains stay MatMul / Softmax rows."""
    from nert_b200 import synth

    def chain(T, D, merge=True):
        g = Graph(opset=13)
        q = g.add_input("q", [2, 3, T, D])
        k = g.add_input("k", [2, 3, D, T])
        v = g.add_input("v", [2, 3, T, D])
        s = g.op("Div", [g.op("MatMul", [q, k], name="qk"), g.const("c", np.array(8.0, np.float32))], name="sc")
        o = g.op("MatMul", [g.op("Softmax", [s], name="sm", axis=-1), v], name="av")
        if merge:
            o = g.op("Reshape", [g.op("Transpose", [o], name="t", perm=[0, 2, 1, 3]),
                                 g.const("m", np.array([2, T, 3 * D], np.int64))], name="merge")
        g.add_output(o, None, FLOAT)
        return nbm.analyze(g, {"q": [2, 3, T, D], "k": [2, 3, D, T], "v": [2, 3, T, D]})["exec"]

    assert [e["op"] for e in chain(197, 64)] == ["Attention"]
    assert [e["op"] for e in chain(5, 64, merge=False)] == ["Attention"]
    assert "Attention" not in [e["op"] for e in chain(209, 64)]
    assert "Attention" not in [e["op"] for e in chain(50, 32)]
