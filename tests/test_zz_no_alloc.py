"""nb2_conv2d_noalloc: the Conv entry point for callers that cannot allocate
device memory (code recording a CUDA graph, frameworks that own all device
memory). It must give the same results as nb2_conv2d while keeping its
scratch in the library's fixed static device array.

Collected last (file name) so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import _lib, synth
from nert_b200.ops import conv_geom

pytestmark = pytest.mark.gpu


def _call(fn_name, dev, g, x, w, b, y):
    fn = getattr(_lib.lib(), fn_name)
    return fn(dev, ctypes.byref(g), x.data_ptr(), w.data_ptr(), b.data_ptr() if b is not None else None, None,
              _lib.ACT_NONE, y.data_ptr())


@pytest.mark.parametrize("order", ["generic_then_tap", "tap_then_generic"])
def test_noalloc_matches_conv2d_on_two_calls_in_a_row(cuda, order):
    import torch

    lib = _lib.lib()
    dev = _lib.device(0)
    cases = [
        # (N, C, H, W, M, k, stride, pad): a stem-like generic-layout conv and a
        # channel-tap conv, so the second call finds the first call's data
        (2, 3, 64, 64, 32, 7, 2, 3),
        (2, 64, 28, 28, 96, 3, 1, 1),
    ]
    if order == "tap_then_generic":
        cases = cases[::-1]
    for i, (n, c, h, w, m, k, s, p) in enumerate(cases):
        x = torch.from_numpy(synth.normal((n, c, h, w), 1.0, 100 + i)).cuda()
        wt = torch.from_numpy(synth.normal((m, c, k, k), 1.0 / np.sqrt(c * k * k), 200 + i)).cuda()
        b = torch.from_numpy(synth.normal((m,), 1.0, 300 + i)).cuda()
        g = conv_geom(tuple(x.shape), tuple(wt.shape), (s, s), (p, p, p, p))
        y_ref = torch.empty((g.n, g.m, g.oh, g.ow), device="cuda")
        y_new = torch.full((g.n, g.m, g.oh, g.ow), float("nan"), device="cuda")
        torch.cuda.synchronize()
        _lib.check(_call("nb2_conv2d", dev, g, x, wt, b, y_ref))
        _lib.check(lib.nb2_device_synchronize(dev))
        _lib.check(_call("nb2_conv2d_noalloc", dev, g, x, wt, b, y_new))
        _lib.check(lib.nb2_device_synchronize(dev))
        got, want = y_new.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) <= TOL


def test_noalloc_rejects_weights_above_capacity(cuda):
    import torch

    lib = _lib.lib()
    dev = _lib.device(0)
    cap = lib.nb2_conv2d_noalloc_capacity()
    assert cap == 8 << 20
    # 512 x 4608 packed hi+lo = 18.9 MB > 8 MiB
    g = conv_geom((1, 512, 7, 7), (512, 512, 3, 3), (1, 1), (1, 1, 1, 1))
    x = torch.zeros((1, 512, 7, 7), device="cuda")
    w = torch.zeros((512, 512, 3, 3), device="cuda")
    y = torch.zeros((1, 512, 7, 7), device="cuda")
    st = _call("nb2_conv2d_noalloc", dev, g, x, w, None, y)
    assert st == _lib.ERR_INVALID
    assert "static scratch" in lib.nb2_last_error().decode()


def test_noalloc_long_k_layer_matches_conv2d(cuda):
    """A layer with one output tile and a long K, which nb2_conv2d runs with
    split K in a growable workspace: the no-alloc call never grows that
    workspace (it runs unsplit when the workspace is absent or too small),
    and both orders of the two calls agree with each other."""
    import torch

    lib = _lib.lib()
    dev = _lib.device(0)
    n, c, h, w, m, k = 1, 256, 7, 7, 96, 3
    x = torch.from_numpy(synth.normal((n, c, h, w), 1.0, 400)).cuda()
    wt = torch.from_numpy(synth.normal((m, c, k, k), 1.0 / np.sqrt(c * k * k), 401)).cuda()
    b = torch.from_numpy(synth.normal((m,), 1.0, 402)).cuda()
    g = conv_geom(tuple(x.shape), tuple(wt.shape), (1, 1), (1, 1, 1, 1))
    outs = []
    for name in ("nb2_conv2d_noalloc", "nb2_conv2d", "nb2_conv2d_noalloc"):
        y = torch.full((g.n, g.m, g.oh, g.ow), float("nan"), device="cuda")
        torch.cuda.synchronize()
        _lib.check(_call(name, dev, g, x, wt, b, y))
        _lib.check(lib.nb2_device_synchronize(dev))
        outs.append(y.cpu().numpy())
    for got in (outs[0], outs[2]):
        assert np.isfinite(got).all()
        assert rel_err(got, outs[1]) <= TOL
