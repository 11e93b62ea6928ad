"""nb2_conv2d_noalloc: the Conv entry point for callers that cannot allocate
device memory, such as a plug-in run inside a host framework that owns all
device memory and forbids allocation while it runs, or a service held to a
fixed memory budget. It must give the same results as nb2_conv2d (and the
oracle) while keeping its scratch in the library's fixed static device array,
and must leave the device's free memory unchanged.

Collected last (file name) so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import _lib, synth
from nert_b200.ops import conv_geom
from oracle import np_ref

pytestmark = pytest.mark.gpu


def _call(fn_name, dev, g, x, w, b, y):
    fn = getattr(_lib.lib(), fn_name)
    return fn(dev, ctypes.byref(g), x.data_ptr(), w.data_ptr(), b.data_ptr() if b is not None else None, None,
              _lib.ACT_NONE, y.data_ptr())


def _oracle(x, w, b, s, p):
    attrs = {"strides": [s, s], "pads": [p, p, p, p], "kernel_shape": list(w.shape[2:])}
    return np_ref.run_op("Conv", attrs, [x, w, b])


def _case(i, n, c, h, w, m, k):
    x = synth.normal((n, c, h, w), 1.0, 100 + i)
    wt = synth.normal((m, c, k, k), 1.0 / np.sqrt(c * k * k), 200 + i)
    b = synth.normal((m,), 1.0, 300 + i)
    return x, wt, b


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
        xh, wh, bh = _case(i, n, c, h, w, m, k)
        x, wt, b = (torch.from_numpy(a).cuda() for a in (xh, wh, bh))
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
        assert rel_err(got, _oracle(xh, wh, bh, s, p)) <= TOL


def test_noalloc_allocates_nothing(cuda):
    """After the first call on the device (which resolves the static array's
    address), further calls leave the device's free memory unchanged."""
    import torch

    lib = _lib.lib()
    dev = _lib.device(0)
    xh, wh, bh = _case(7, 2, 64, 28, 28, 128, 3)
    x, wt, b = (torch.from_numpy(a).cuda() for a in (xh, wh, bh))
    g = conv_geom(tuple(x.shape), tuple(wt.shape), (1, 1), (1, 1, 1, 1))
    y = torch.empty((g.n, g.m, g.oh, g.ow), device="cuda")
    torch.cuda.synchronize()
    _lib.check(_call("nb2_conv2d_noalloc", dev, g, x, wt, b, y))
    _lib.check(lib.nb2_device_synchronize(dev))
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        _lib.check(_call("nb2_conv2d_noalloc", dev, g, x, wt, b, y))
        _lib.check(lib.nb2_device_synchronize(dev))
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert rel_err(y.cpu().numpy(), _oracle(xh, wh, bh, 1, 1)) <= TOL


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


def test_noalloc_long_k_layer_runs_unsplit(cuda):
    """A layer with one output tile and a long K, which nb2_conv2d runs with
    split K in its growable workspace: the no-alloc call never splits K, in
    either order of the calls, and all agree with the oracle."""
    import torch

    lib = _lib.lib()
    dev = _lib.device(0)
    n, c, h, w, m, k = 1, 256, 7, 7, 96, 3
    xh, wh, bh = _case(40, n, c, h, w, m, k)
    x, wt, b = (torch.from_numpy(a).cuda() for a in (xh, wh, bh))
    g = conv_geom(tuple(x.shape), tuple(wt.shape), (1, 1), (1, 1, 1, 1))
    want = _oracle(xh, wh, bh, 1, 1)
    for name, slices in (("nb2_conv2d_noalloc", 1), ("nb2_conv2d", None), ("nb2_conv2d_noalloc", 1)):
        y = torch.full((g.n, g.m, g.oh, g.ow), float("nan"), device="cuda")
        torch.cuda.synchronize()
        _lib.check(_call(name, dev, g, x, wt, b, y))
        _lib.check(lib.nb2_device_synchronize(dev))
        sched = _lib.last_contraction(0)
        if slices is None:
            assert sched["k_slices"] > 1  # the allocating entry point does split this layer
        else:
            assert sched["k_slices"] == slices
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) <= TOL
