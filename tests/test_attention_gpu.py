"""The fused attention step (ops_attn.cu) against the oracle's MatMul -> Div
-> Softmax -> MatMul rows (src/kernels/mat_mul.cpp, div.cpp, softmax.cpp),
within max|err| <= 1e-4 * max|ref|, through the C ABI and through the engine
(where the plan must have fused the chain)."""

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import synth
from nert_b200.onnx_io import FLOAT, Graph
from oracle import np_ref

pytestmark = pytest.mark.gpu


def chain_graph(B, H, T, D=64, merge=True, scale_op="Div", scale=8.0):
    g = Graph(opset=13)
    q = g.add_input("q", [B, H, T, D])
    k = g.add_input("k", [B, H, D, T])
    v = g.add_input("v", [B, H, T, D])
    s = g.op("MatMul", [q, k], name="qk")
    if scale_op:
        s = g.op(scale_op, [s, g.const("c", np.array(scale, np.float32))], name="sc")
    o = g.op("MatMul", [g.op("Softmax", [s], name="sm", axis=-1), v], name="av")
    if merge:
        o = g.op("Reshape", [g.op("Transpose", [o], name="t", perm=[0, 2, 1, 3]),
                             g.const("m", np.array([B, T, H * D], np.int64))], name="merge")
    g.add_output(o, None, FLOAT)
    return g


def feeds(B, H, T, D=64, seed=0, spread=1.0):
    return {"q": synth.normal((B, H, T, D), spread, 300 + seed), "k": synth.normal((B, H, D, T), spread, 400 + seed),
            "v": synth.normal((B, H, T, D), 1.0, 500 + seed)}


@pytest.mark.parametrize("T", [197, 1, 5, 16, 128, 129, 208])
@pytest.mark.parametrize("merge", [True, False], ids=["merged", "heads"])
def test_attention_c_abi(cuda, T, merge):
    import torch

    from nert_b200 import _lib
    from nert_b200._lib import i64s

    B, H, D = 2, 3, 64
    f = feeds(B, H, T)
    want = list(np_ref.run(chain_graph(B, H, T, merge=merge), f).values())[0]
    q, k, v = (torch.from_numpy(f[n]).cuda() for n in ("q", "k", "v"))
    out = torch.full(want.shape, float("nan"), device="cuda")
    os_ = [T * H * D, D, H * D] if merge else [H * T * D, T * D, D]
    L, dev = _lib.lib(), _lib.device(0)
    _lib.check(L.nb2_attention(dev, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, T, D,
                               i64s([H * T * D, T * D, D, 1]), i64s([H * D * T, D * T, 1, T]),
                               i64s([H * T * D, T * D, D, 1]), i64s(os_), 2, 8.0))
    _lib.check(L.nb2_device_synchronize(dev))
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= TOL


@pytest.mark.parametrize("B,T,spread", [(32, 197, 1.0), (2, 197, 4.0), (3, 50, 0.25)],
                         ids=["vit_b32", "peaked", "flat"])
def test_attention_engine_matches_rows(cuda, B, T, spread):
    """The engine's fused step against the oracle and against the same graph
    run as separate rows (fused_attention=False)."""
    from nert_b200 import model as nbm

    H = 12 if B == 32 else 3
    g = chain_graph(B, H, T)
    assert [e["op"] for e in nbm.analyze(g, {"q": [B, H, T, 64], "k": [B, H, 64, T], "v": [B, H, T, 64]})["exec"]] \
        == ["Attention"]
    f = feeds(B, H, T, spread=spread, seed=B)
    dims = {n: list(a.shape) for n, a in f.items()}
    fused = nbm.Model(g, dims)
    rows = nbm.Model(g, dims, fused_attention=False)
    try:
        got = list(fused.run(f).values())[0]
        unfused = list(rows.run(f).values())[0]
    finally:
        fused.close()
        rows.close()
    if B == 32:
        # the oracle on a slice of images (each (b, h) is independent)
        sl = {n: a[:2] for n, a in f.items()}
        want = list(np_ref.run(chain_graph(2, H, T), sl).values())[0]
        assert rel_err(got[:2], want) <= TOL
    else:
        want = list(np_ref.run(g, f).values())[0]
        assert rel_err(got, want) <= TOL
    assert rel_err(got, unfused) <= TOL


def test_attention_mul_scale_and_no_scale(cuda):
    from nert_b200 import model as nbm

    for op, c in (("Mul", 0.125), (None, 1.0)):
        g = chain_graph(2, 2, 31, merge=False, scale_op=op, scale=c)
        f = feeds(2, 2, 31, seed=7)
        m = nbm.Model(g, {n: list(a.shape) for n, a in f.items()})
        try:
            got = list(m.run(f).values())[0]
        finally:
            m.close()
        assert rel_err(got, list(np_ref.run(g, f).values())[0]) <= TOL


def test_attention_rejects_unsupported(cuda):
    from nert_b200 import _lib
    from nert_b200._lib import i64s

    L, dev = _lib.lib(), _lib.device(0)
    s4 = i64s([0, 0, 0, 1])
    assert L.nb2_attention(dev, 8, 8, 8, 8, 1, 1, 209, 64, s4, s4, s4, i64s([0, 0, 0]), 0, 1.0) != 0
    assert L.nb2_attention(dev, 8, 8, 8, 8, 1, 1, 10, 32, s4, s4, s4, i64s([0, 0, 0]), 0, 1.0) != 0
