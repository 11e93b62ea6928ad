"""Per-row parity of the B200 kernels (through the C ABI) against the oracle.

* known answers ported from the reference's tests (tests/golden/known_answers.py);
* seeded random cases at the config-1 geometries (reduced batch) checked
  against the numpy restatement of the reference kernels, with the north-star
  bound max|err| <= 1e-4 * max|ref| for the default 3xTF32 mode.
"""

import numpy as np
import pytest

from conftest import TOL, rel_err
from golden.known_answers import CASES
from nert_b200 import synth
from oracle import np_ref

pytestmark = pytest.mark.gpu

SUPPORTED = {"Relu", "Add", "Mul", "Sub", "Div", "Gemm", "MatMul", "Conv", "MaxPool", "GlobalAveragePool"}


def _run_case(op, attrs, arrs):
    import torch

    from nert_b200 import _lib, ops

    t = [torch.from_numpy(a).cuda() for a in arrs]
    if op == "Relu":
        return ops.unary(0, t[0])
    if op in ("Add", "Sub", "Mul", "Div"):
        return ops.binary({"Add": 0, "Sub": 1, "Mul": 2, "Div": 3}[op], t[0], t[1])
    if op == "Gemm":
        return ops.gemm(t[0], t[1], t[2] if len(t) > 2 else None, attrs.get("transA", 0), attrs.get("transB", 0),
                        attrs.get("alpha", 1.0), attrs.get("beta", 1.0))
    if op == "MatMul":
        return ops.matmul(t[0], t[1])
    if op == "Conv":
        sp = attrs.get("pads", [0, 0, 0, 0])
        return ops.conv2d(t[0], t[1], t[2] if len(t) > 2 else None, attrs.get("strides", [1, 1]), sp,
                          attrs.get("dilations", [1, 1]), attrs.get("group", 1))
    if op == "MaxPool":
        return ops.maxpool2d(t[0], attrs["kernel_shape"], attrs.get("strides", [1, 1]), attrs.get("pads", [0] * 4),
                             attrs.get("dilations", [1, 1]), attrs.get("ceil_mode", 0))
    if op == "GlobalAveragePool":
        return ops.global_avgpool(t[0])
    raise KeyError(op)


@pytest.mark.parametrize("case", [c for c in CASES if c[1] in SUPPORTED], ids=lambda c: c[0].split()[1])
def test_known_answers(cuda, case):
    cite, op, attrs, ins, exp, edims = case
    arrs = [np.array(v, np.float32).reshape(d) for v, d in ins]
    got = _run_case(op, attrs, arrs).cpu().numpy()
    assert list(got.shape) == edims, cite
    np.testing.assert_allclose(got.ravel(), np.array(exp, np.float32), rtol=1e-6, atol=1e-6, err_msg=cite)


# (name, N, C, H, W, M, k, stride, pad, group) — the config-1 sweep at reduced batch
CONV_CASES = [
    ("stem_3_64_k7s2", 2, 3, 224, 224, 64, 7, 2, 3, 1),
    ("c64_k3_56", 2, 64, 56, 56, 64, 3, 1, 1, 1),
    ("c128_k3_28", 2, 128, 28, 28, 128, 3, 1, 1, 1),
    ("c256_k3_14", 2, 256, 14, 14, 256, 3, 1, 1, 1),
    ("c512_k3_7", 4, 512, 7, 7, 512, 3, 1, 1, 1),
    ("ds_64_128_s2", 2, 64, 56, 56, 128, 1, 2, 0, 1),
    ("ds_128_256_s2", 2, 128, 28, 28, 256, 1, 2, 0, 1),
    ("ds_256_512_s2", 2, 256, 14, 14, 512, 1, 2, 0, 1),
    ("r50_64_256", 2, 64, 56, 56, 256, 1, 1, 0, 1),
    ("r50_256_64", 2, 256, 56, 56, 64, 1, 1, 0, 1),
    ("s2_k3_64_128", 2, 64, 56, 56, 128, 3, 2, 1, 1),
    ("odd_c48_k3", 2, 48, 17, 19, 40, 3, 1, 1, 1),
    ("group2_c64", 2, 64, 20, 20, 96, 3, 1, 1, 2),
    ("patch16_vit", 2, 3, 224, 224, 768, 16, 16, 0, 1),
]


@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: c[0])
def test_conv_parity(cuda, case):
    import torch

    from nert_b200 import ops

    name, n, c, h, w, m, k, s, p, g = case
    x = synth.normal((n, c, h, w), 1.0, synth.seed_of("sweep", name + ".x"))
    wt = synth.normal((m, c // g, k, k), 1.0 / np.sqrt(c // g * k * k), synth.seed_of("sweep", name + ".w"))
    b = synth.normal((m,), 1.0, synth.seed_of("sweep", name + ".b"))
    attrs = {"strides": [s, s], "pads": [p] * 4, "group": g}
    ref = np_ref.run_op("Conv", attrs, [x, wt, b])
    got = ops.conv2d(torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda(), torch.from_numpy(b).cuda(),
                     [s, s], [p] * 4, [1, 1], g).cpu().numpy()
    assert got.shape == ref.shape
    assert rel_err(got, ref) <= TOL, rel_err(got, ref)


def test_conv_fused_residual_relu(cuda):
    import torch

    from nert_b200 import ops

    x = synth.normal((2, 64, 28, 28), 1.0, 11)
    wt = synth.normal((64, 64, 3, 3), 1.0 / 24, 12)
    b = synth.normal((64,), 1.0, 13)
    r = synth.normal((2, 64, 28, 28), 1.0, 14)
    conv = np_ref.run_op("Conv", {"pads": [1] * 4}, [x, wt, b])
    ref = np.maximum(conv + r, 0)
    got = ops.conv2d(torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda(), torch.from_numpy(b).cuda(),
                     [1, 1], [1] * 4, residual=torch.from_numpy(r).cuda(), act=1).cpu().numpy()
    assert rel_err(got, ref) <= TOL


GEMM_CASES = [
    (64, 1000, 512, 0, 1),
    (256, 384, 768, 0, 0),
    (200, 136, 100, 1, 0),
    (129, 65, 33, 1, 1),
    (1024, 1024, 1024, 0, 0),
]


@pytest.mark.parametrize("case", GEMM_CASES, ids=lambda c: "x".join(map(str, c)))
def test_gemm_parity(cuda, case):
    import torch

    from nert_b200 import ops

    m, n, k, ta, tb = case
    a = synth.normal((k, m) if ta else (m, k), 1.0, synth.seed_of("gemm", f"{case}.a"))
    b = synth.normal((n, k) if tb else (k, n), 1.0 / np.sqrt(k), synth.seed_of("gemm", f"{case}.b"))
    c = synth.normal((n,), 1.0, synth.seed_of("gemm", f"{case}.c"))
    attrs = {"transA": ta, "transB": tb, "alpha": 1.5, "beta": 0.5}
    ref = np_ref.run_op("Gemm", attrs, [a, b, c])
    got = ops.gemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(c).cuda(), ta, tb,
                   1.5, 0.5).cpu().numpy()
    assert rel_err(got, ref) <= TOL, rel_err(got, ref)


def test_gemm_rank2_bias(cuda):
    import torch

    from nert_b200 import ops

    a = synth.normal((70, 90), 1.0, 21)
    b = synth.normal((90, 50), 1.0, 22)
    c = synth.normal((70, 50), 1.0, 23)
    ref = np_ref.run_op("Gemm", {"beta": 2.0}, [a, b, c])
    got = ops.gemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(c).cuda(),
                   beta=2.0).cpu().numpy()
    assert rel_err(got, ref) <= TOL


@pytest.mark.parametrize("shapes", [((4, 12, 197, 64), (4, 12, 64, 197)), ((4, 197, 768), (768, 256)),
                                    ((3, 50, 40), (40, 30))], ids=["qk", "linear", "b3"])
def test_matmul_parity(cuda, shapes):
    import torch

    from nert_b200 import ops

    a = synth.normal(shapes[0], 1.0, 31)
    b = synth.normal(shapes[1], 0.1, 32)
    ref = np_ref.run_op("MatMul", {}, [a, b])
    got = ops.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert got.shape == ref.shape
    assert rel_err(got, ref) <= TOL


def test_one_tf32_mode_is_separate(cuda):
    """1xTF32 is opt-in and visibly less accurate than the 3xTF32 default."""
    import torch

    from nert_b200 import _lib, ops

    a = synth.normal((256, 512), 1.0, 41)
    b = synth.normal((512, 256), 1.0, 42)
    ref = np_ref.run_op("Gemm", {}, [a, b])
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    e3 = rel_err(ops.gemm(ta, tb).cpu().numpy(), ref)
    ops.set_precision(_lib.PREC_1XTF32)
    try:
        e1 = rel_err(ops.gemm(ta, tb).cpu().numpy(), ref)
    finally:
        ops.set_precision(_lib.PREC_3XTF32)
    assert e3 <= TOL
    assert e1 > e3
    assert e1 < 1e-2


def test_maxpool_resnet_geometry(cuda):
    import torch

    from nert_b200 import ops

    x = synth.normal((2, 64, 112, 112), 1.0, 51)
    attrs = {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]}
    ref = np_ref.run_op("MaxPool", attrs, [x])
    got = ops.maxpool2d(torch.from_numpy(x).cuda(), [3, 3], [2, 2], [1, 1, 1, 1]).cpu().numpy()
    np.testing.assert_array_equal(got, ref)


def test_gap_and_relu_add(cuda):
    import torch

    from nert_b200 import ops

    x = synth.normal((4, 512, 7, 7), 1.0, 61)
    np.testing.assert_allclose(ops.global_avgpool(torch.from_numpy(x).cuda()).cpu().numpy(),
                               np_ref.run_op("GlobalAveragePool", {}, [x]), rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(ops.unary(0, torch.from_numpy(x).cuda()).cpu().numpy(),
                                  np_ref.run_op("Relu", {}, [x]))
    y = synth.normal((4, 512, 7, 7), 1.0, 62)
    np.testing.assert_array_equal(ops.binary(0, torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()).cpu().numpy(),
                                  np_ref.run_op("Add", {}, [x, y]))
