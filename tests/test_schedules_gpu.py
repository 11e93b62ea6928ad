"""Every schedule of the tensor-core contraction kernel against the oracle.

The host picks, per launch, the output tile width (64 or 128 columns), whether
two 128-wide tiles are kept in flight (the two MMA issuers take alternate
tiles and hand off through a barrier), whether K is split into slices
reduced by a second kernel, and whether the (tile, K block) pairs are cut
into one equal span per CTA (the balanced split, k_slices == 0, for tile
counts that leave the last wave short; the tiles cut at a span boundary are
finished by a second kernel). Each case below is sized so that one schedule is
taken, asserts through nb2_device_last_contraction that it was, and compares
the result with the numpy restatement of the reference rows
(src/kernels/gemm.cpp:122-136, conv.cpp:263-289: float64 accumulation, one
rounding) at max|err| <= 1e-4 * max|ref|.

The large cases are checked on rows sampled from every 128-row tile (a
different lane of each tile) plus a size-independent property over the whole
output: the column sums of Y equal (1^T A) B, and for a Conv each channel's
sum over images and pixels equals the weights applied to the window sums of
the padded input.
"""

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import synth
from oracle import np_ref

pytestmark = pytest.mark.gpu


def _sample_rows(m: int) -> np.ndarray:
    """Two rows of every 128-row tile, at lanes that differ from tile to tile."""
    rows = []
    for t in range((m + 127) // 128):
        for off in ((t * 37) % 128, (t * 37 + 71) % 128):
            r = t * 128 + off
            if r < m:
                rows.append(r)
    return np.array(rows, np.int64)


def _check_gemm(y, a, b, bias=None):
    """y = a @ b (+ bias) on sampled rows, and its column sums in full."""
    rows = _sample_rows(a.shape[0])
    want = a[rows].astype(np.float64) @ b.astype(np.float64)
    if bias is not None:
        want = want + bias.astype(np.float64)
    assert rel_err(y[rows], want.astype(np.float32)) <= TOL
    colsum_want = a.astype(np.float64).sum(axis=0) @ b.astype(np.float64)
    if bias is not None:
        colsum_want = colsum_want + a.shape[0] * bias.astype(np.float64)
    colsum = y.astype(np.float64).sum(axis=0)
    assert np.abs(colsum - colsum_want).max() <= TOL * np.abs(y.astype(np.float64)).sum(axis=0).max()


def _sched():
    from nert_b200 import _lib

    return _lib.last_contraction(0)


# (name, M, N, K, expected schedule)
GEMMS = [
    ("two_in_flight_4096x4096x1024", 4096, 4096, 1024, dict(tile_n=128, two_in_flight=1, k_slices=1)),
    ("two_in_flight_sweep_8192x3072x768", 8192, 3072, 768, dict(tile_n=128, two_in_flight=1, k_slices=1)),
    ("long_k_sweep_4096_cubed", 4096, 4096, 4096, dict(tile_n=128, two_in_flight=0, k_slices=1)),
    ("long_k_sweep_25088x768x3072", 25088, 768, 3072, dict(tile_n=128, two_in_flight=0, k_slices=1)),
    ("split_k_sweep_64x1000x512", 64, 1000, 512, dict(tile_n=128, two_in_flight=0, k_slices=4)),
    ("narrow_64_many_tiles", 30000, 64, 576, dict(tile_n=64, two_in_flight=0, k_slices=1)),
    ("short_k_64_wide", 2000, 256, 128, dict(tile_n=64, two_in_flight=0, k_slices=1)),
    # 100 and 196 tiles on 148 SMs: the balanced split
    ("balanced_100_tiles_2560x640x4096", 2560, 640, 4096, dict(tile_n=128, two_in_flight=0, k_slices=0)),
    ("balanced_196_tiles_1792x1792x2304", 1792, 1792, 2304, dict(tile_n=128, two_in_flight=0, k_slices=0)),
    # 300 tiles of 24 K blocks (ViT-B/16 b32 q/k/v/proj): a last wave of 4
    # tiles after two full ones stays unsplit (the balanced split measured 5%
    # slower per ViT forward there)
    ("sparse_tail_unsplit_6304x768x768", 6304, 768, 768, dict(tile_n=128, two_in_flight=0, k_slices=1)),
]


@pytest.mark.parametrize("case", GEMMS, ids=lambda c: c[0])
def test_gemm_schedule(cuda, case):
    import torch

    from nert_b200 import ops

    name, m, n, k, want = case
    seed = synth.seed_of("schedules", name)
    a = synth.normal((m, k), 1.0, seed)
    b = synth.normal((k, n), 1.0 / np.sqrt(k), seed ^ 1)
    bias = synth.normal((n,), 1.0, seed ^ 2)
    y = ops.gemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(bias).cuda())
    got = _sched()
    for key, v in want.items():
        assert got[key] == v, (name, got)
    _check_gemm(y.cpu().numpy(), a, b, bias)


def test_matmul_vit_fc1_b32_two_in_flight(cuda):
    """ViT-B/16 fc1 at batch 32: [32,197,768] x [768,3072], the 2-D weight
    folded into one GEMM of 6304 rows (1200 tiles, 24 K blocks)."""
    import torch

    from nert_b200 import ops

    seed = synth.seed_of("schedules", "vit_fc1")
    a = synth.normal((32, 197, 768), 1.0, seed)
    b = synth.normal((768, 3072), 0.02, seed ^ 1)
    y = ops.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    got = _sched()
    assert (got["tile_n"], got["two_in_flight"], got["k_slices"]) == (128, 1, 1), got
    _check_gemm(y.reshape(-1, 3072), a.reshape(-1, 768), b)


def _conv_channel_sums(x, w, b, stride, pad, oh, ow):
    """sum over (n, oh, ow) of Conv(x, w) + b per output channel, by linearity:
    the weights applied to the window sums of the padded input."""
    n, c = x.shape[:2]
    m, _, kh, kw = w.shape
    xp = np.pad(x.astype(np.float64), [(0, 0), (0, 0), (pad, pad), (pad, pad)])
    s = np.zeros((c, kh, kw))
    for i in range(kh):
        for j in range(kw):
            s[:, i, j] = xp[:, :, i:i + stride * (oh - 1) + 1:stride, j:j + stride * (ow - 1) + 1:stride].sum(
                axis=(0, 2, 3))
    return np.einsum("mcij,cij->m", w.astype(np.float64), s) + b.astype(np.float64) * n * oh * ow


# (name, N, C, H, W, M, k, stride, pad, expected schedule)
CONVS = [
    # ResNet-18 bs64 layer 2: 392 tiles of 128 on 148 SMs, 36 K blocks
    ("resnet18_b64_layer2", 64, 128, 28, 28, 128, 3, 1, 1, dict(tile_n=128, two_in_flight=0, k_slices=1)),
    # ResNet-50 1x1 expansion at bs32: 1568 tiles, 2 K blocks
    ("resnet50_b32_1x1_expand", 32, 64, 56, 56, 256, 1, 1, 0, dict(tile_n=128, two_in_flight=1, k_slices=1)),
    # ResNet-18 bs64 layer 1: 64 channels, double-buffered 64-wide tiles
    ("resnet18_b64_layer1", 64, 64, 56, 56, 64, 3, 1, 1, dict(tile_n=64, two_in_flight=0, k_slices=1)),
    # ResNet-18 bs64 layers 3 and 4: 196 and 100 tiles, 72 and 144 K blocks
    ("resnet18_b64_layer3", 64, 256, 14, 14, 256, 3, 1, 1, dict(tile_n=128, two_in_flight=0, k_slices=0)),
    ("resnet18_b64_layer4", 64, 512, 7, 7, 512, 3, 1, 1, dict(tile_n=128, two_in_flight=0, k_slices=0)),
]


@pytest.mark.parametrize("case", CONVS, ids=lambda c: c[0])
def test_conv_schedule(cuda, case):
    import torch

    from nert_b200 import ops

    name, n, c, h, w, m, k, s, p, want = case
    seed = synth.seed_of("schedules", name)
    x = synth.normal((n, c, h, w), 1.0, seed)
    wt = synth.normal((m, c, k, k), 1.0 / np.sqrt(c * k * k), seed ^ 1)
    b = synth.normal((m,), 1.0, seed ^ 2)
    y = ops.conv2d(torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda(), torch.from_numpy(b).cuda(), (s, s),
                   (p, p, p, p)).cpu().numpy()
    got = _sched()
    for key, v in want.items():
        assert got[key] == v, (name, got)
    attrs = {"strides": [s, s], "pads": [p, p, p, p], "kernel_shape": [k, k]}
    for i in (0, n // 2, n - 1):
        ref = np_ref.run_op("Conv", attrs, [x[i:i + 1], wt, b])
        assert rel_err(y[i:i + 1], ref) <= TOL, (name, i)
    sums = y.astype(np.float64).sum(axis=(0, 2, 3))
    want_sums = _conv_channel_sums(x, wt, b, s, p, y.shape[2], y.shape[3])
    assert np.abs(sums - want_sums).max() <= TOL * np.abs(y.astype(np.float64)).sum(axis=(0, 2, 3)).max()


def test_wait_bound_expiry_reports_device_error_then_recovers(cuda):
    """A pipeline wait that runs out of its bound makes the kernel record a
    device error and unwind (no trap, no hang); the context stays usable and
    the same Gemm at the default bound then matches the oracle."""
    import torch

    from nert_b200 import _lib, ops

    lib = _lib.lib()
    dev = _lib.device(0)
    default = lib.nb2_device_get_wait_bound(dev)
    assert default > 10 ** 8
    seed = synth.seed_of("schedules", "wait_bound")
    # six K blocks: below the split-K threshold, so one kernel
    a = synth.normal((512, 192), 1.0, seed)
    b = synth.normal((192, 384), 1.0 / 14, seed ^ 1)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    _lib.check(lib.nb2_device_set_wait_bound(dev, 64))
    try:
        with pytest.raises(_lib.NB2Error) as err:
            ops.gemm(ta, tb)
        assert err.value.status == _lib.ERR_DEVICE
        assert "bounded wait expired" in str(err.value)
    finally:
        _lib.check(lib.nb2_device_set_wait_bound(dev, 0))
    assert lib.nb2_device_get_wait_bound(dev) == default
    y = ops.gemm(ta, tb).cpu().numpy()
    assert rel_err(y, np_ref.run_op("Gemm", {}, [a, b])) <= TOL


def test_balanced_split_through_output_map(cuda):
    """A MatMul whose head-split Transpose the engine absorbs (the epilogue
    writes through an output map) and whose 100 tiles of 144 K blocks take
    the balanced split: the reduce writes the cut tiles through the same map.
    Checked against the oracle's MatMul -> Reshape -> Transpose rows."""
    from nert_b200 import _lib
    from nert_b200 import model as nbm
    from nert_b200.onnx_io import FLOAT, Graph

    seed = synth.seed_of("schedules", "balanced_omap")
    g = Graph(opset=13)
    x = g.add_input("x", [1280, 4608])
    y = g.op("MatMul", [x, g.const("w", synth.normal((4608, 1280), 1.0 / 68, seed))], name="mm")
    y = g.op("Reshape", [y, g.const("s", np.array([1280, 10, 128], np.int64))], name="rs")
    y = g.op("Transpose", [y], name="tr", perm=[1, 0, 2])
    g.add_output(y, None, FLOAT)
    ex = nbm.analyze(g, {"x": [1280, 4608]})["exec"]
    assert [e["op"] for e in ex] == ["MatMul"] and ex[0]["perm"] == [1, 0, 2]
    feed = {"x": synth.normal((1280, 4608), 1.0, seed ^ 1)}
    m = nbm.Model(g, {"x": [1280, 4608]})
    try:
        got = list(m.run(feed).values())[0]
        sched = _lib.last_contraction(0)
    finally:
        m.close()
    assert (sched["tile_n"], sched["k_slices"], sched["tiles"]) == (128, 0, 100), sched
    want = list(np_ref.run(g, feed).values())[0]
    assert rel_err(got, want) <= TOL
