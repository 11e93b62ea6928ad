"""The direct CUDA-core Conv (conv_direct.cu) for narrow outputs (<= 32
channels, few multiply-adds per pixel) against the oracle's Conv row
(src/kernels/conv.cpp:138-295), within max|err| <= 1e-4 * max|ref|: through
the C ABI, with the fused epilogue, and inside the engine on the YOLO-style
graph (whose cheap narrow layers must take it)."""

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import synth
from oracle import np_ref

pytestmark = pytest.mark.gpu

# (name, N, C, H, W, M, kh, kw, stride, pad, dilation)
CASES = [
    ("yolo_b0_stem", 2, 3, 64, 64, 16, 3, 3, 2, 1, 1),
    ("c2f_pointwise_32", 2, 32, 40, 40, 32, 1, 1, 1, 0, 1),
    ("yolo_c2f_bottleneck", 2, 16, 33, 31, 16, 3, 3, 1, 1, 1),
    ("pointwise_48_to_32", 3, 48, 20, 20, 32, 1, 1, 1, 0, 1),
    ("dfl_1x1_one_channel", 2, 16, 4, 70, 1, 1, 1, 1, 0, 1),
    ("odd_m_5_dilated", 1, 7, 17, 19, 5, 3, 3, 1, 2, 2),
    ("rect_kernel_stride", 2, 4, 23, 29, 9, 5, 3, 3, 2, 1),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0])
def test_direct_conv_c_abi(cuda, case):
    import torch

    from nert_b200 import _lib, ops

    name, n, c, h, w, m, kh, kw, s, p, d = case
    seed = synth.seed_of("direct", name)
    x = synth.normal((n, c, h, w), 1.0, seed)
    wt = synth.normal((m, c, kh, kw), 1.0 / np.sqrt(c * kh * kw), seed ^ 1)
    b = synth.normal((m,), 0.5, seed ^ 2)
    y = ops.conv2d(torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda(), torch.from_numpy(b).cuda(), (s, s),
                   (p, p, p, p), (d, d)).cpu().numpy()
    attrs = {"strides": [s, s], "pads": [p, p, p, p], "dilations": [d, d], "kernel_shape": [kh, kw]}
    want = np_ref.run_op("Conv", attrs, [x, wt, b])
    assert y.shape == want.shape
    assert rel_err(y, want) <= TOL


def test_direct_conv_fused_residual_and_silu(cuda):
    import torch

    from nert_b200 import _lib, ops

    seed = synth.seed_of("direct", "epilogue")
    x = synth.normal((2, 16, 24, 24), 1.0, seed)
    wt = synth.normal((16, 16, 3, 3), 0.08, seed ^ 1)
    b = synth.normal((16,), 0.5, seed ^ 2)
    r = synth.normal((2, 16, 24, 24), 1.0, seed ^ 3)
    t = lambda a: torch.from_numpy(a).cuda()
    y = ops.conv2d(t(x), t(wt), t(b), (1, 1), (1, 1, 1, 1), residual=t(r), act=_lib.ACT_SILU).cpu().numpy()
    z = np_ref.run_op("Conv", {"strides": [1, 1], "pads": [1, 1, 1, 1], "kernel_shape": [3, 3]}, [x, wt, b]) + r
    want = z * (1.0 / (1.0 + np.exp(-z.astype(np.float64))))
    assert rel_err(y, want.astype(np.float32)) <= TOL


def test_yolo_narrow_layers_take_the_direct_path(cuda):
    """The YOLO-style graph's <= 32-channel convs run as [direct] steps, and
    its outputs still match the rows run one by one."""
    from nert_b200 import configs
    from nert_b200 import model as nbm

    g = configs.yolov8n(1, expose_scores=True)
    x = configs.yolo_input(1)
    m = nbm.Model(g, {"images": list(x.shape)})
    try:
        labels = [lab for lab, _ in m.profile()]
        got = m.run({"images": x})
    finally:
        m.close()
    direct = [lab for lab in labels if "[direct]" in lab]
    assert any(":b0" in lab for lab in direct) and any(":b2.cv1" in lab for lab in direct), direct
    assert not any(":b1" in lab or ":b4.m0" in lab for lab in direct), direct  # FMA-heavy: tensor cores
    assert any("dfl" in lab for lab in direct), direct
    plain = nbm.Model(g, {"images": list(x.shape)}, fuse=False, channels_last=False)
    try:
        want = plain.run({"images": x})
    finally:
        plain.close()
    for name, v in got.items():
        if v.dtype == np.float32:
            assert rel_err(v, want[name]) <= TOL, name
