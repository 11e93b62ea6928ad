"""Python wrappers of the B200 op rows over torch CUDA tensors.

torch provides device memory only; every computation is a kernel of
libnert_b200.so reached through the C ABI. The wrappers mirror the reference
operators' attribute semantics (ONNX names, NCHW, explicit begin/end pads).
Each call synchronises torch's stream before launching on the layer's own
stream and synchronises the layer's stream after, so results are ready for
torch and device-recorded errors surface as exceptions.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, i64s, lib


def _dev(t: torch.Tensor) -> int:
    return _lib.device(t.device.index or 0)


def _p(t):
    return None if t is None else t.data_ptr()


def _prep(*ts):
    torch.cuda.synchronize()
    for t in ts:
        if t is not None:
            assert t.is_cuda and t.is_contiguous(), "expected contiguous CUDA tensors"


def _finish(dev):
    check(lib().nb2_device_synchronize(dev))


def set_precision(precision: int, ordinal: int = 0) -> None:
    check(lib().nb2_device_set_precision(_lib.device(ordinal), precision))


def conv_out_dim(n, k, s, pb, pe, d):
    return (n + pb + pe - (d * (k - 1) + 1)) // s + 1


def conv_geom(x_shape, w_shape, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1):
    n, c, h, w = x_shape
    m, _, kh, kw = w_shape
    oh = conv_out_dim(h, kh, strides[0], pads[0], pads[2], dilations[0])
    ow = conv_out_dim(w, kw, strides[1], pads[1], pads[3], dilations[1])
    return _lib.ConvGeom(n, c, h, w, m, kh, kw, oh, ow, strides[0], strides[1], pads[0], pads[1], pads[2], pads[3],
                         dilations[0], dilations[1], group)


def conv2d(x, w, b=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1, residual=None,
           act=_lib.ACT_NONE):
    g = conv_geom(tuple(x.shape), tuple(w.shape), strides, pads, dilations, group)
    y = torch.empty((g.n, g.m, g.oh, g.ow), device=x.device, dtype=torch.float32)
    _prep(x, w, b, residual)
    dev = _dev(x)
    check(lib().nb2_conv2d(dev, ctypes.byref(g), _p(x), _p(w), _p(b), _p(residual), act, _p(y)))
    _finish(dev)
    return y


def gemm(a, b, c=None, trans_a=0, trans_b=0, alpha=1.0, beta=1.0, act=_lib.ACT_NONE):
    m = a.shape[1] if trans_a else a.shape[0]
    k = a.shape[0] if trans_a else a.shape[1]
    n = b.shape[0] if trans_b else b.shape[1]
    y = torch.empty((m, n), device=a.device, dtype=torch.float32)
    _prep(a, b, c)
    dev = _dev(a)
    c_rank = 0 if c is None else c.dim()
    check(lib().nb2_gemm(dev, _p(a), _p(b), _p(c), c_rank, _p(y), m, n, k, trans_a, trans_b, alpha, beta, act))
    _finish(dev)
    return y


def matmul(a, b):
    out_shape = torch.matmul(torch.empty(a.shape, device="meta"), torch.empty(b.shape, device="meta")).shape
    y = torch.empty(out_shape, device=a.device, dtype=torch.float32)
    _prep(a, b)
    dev = _dev(a)
    check(lib().nb2_matmul(dev, _p(a), i64s(a.shape), a.dim(), _p(b), i64s(b.shape), b.dim(), _p(y)))
    _finish(dev)
    return y


def unary(op, x):
    y = torch.empty_like(x)
    _prep(x)
    dev = _dev(x)
    check(lib().nb2_unary(dev, op, _p(x), _p(y), x.numel()))
    _finish(dev)
    return y


def binary(op, a, b):
    out_shape = torch.broadcast_shapes(a.shape, b.shape)
    y = torch.empty(out_shape, device=a.device, dtype=a.dtype)
    _prep(a, b)
    dev = _dev(a)
    dt = _lib.I64 if a.dtype == torch.int64 else _lib.F32
    check(lib().nb2_binary(dev, op, dt, _p(a), i64s(a.shape), a.dim(), _p(b), i64s(b.shape), b.dim(), _p(y),
                           i64s(out_shape), len(out_shape)))
    _finish(dev)
    return y


def maxpool2d(x, kernel, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), ceil_mode=0):
    n, c, h, w = x.shape

    def od(i, k, s, pb, pe, d):
        numer = i + pb + pe - (d * (k - 1) + 1)
        return ((numer + s - 1) // s if ceil_mode else numer // s) + 1

    oh = od(h, kernel[0], strides[0], pads[0], pads[2], dilations[0])
    ow = od(w, kernel[1], strides[1], pads[1], pads[3], dilations[1])
    y = torch.empty((n, c, oh, ow), device=x.device, dtype=torch.float32)
    _prep(x)
    dev = _dev(x)
    check(lib().nb2_maxpool2d(dev, _p(x), i64s(x.shape), _p(y), i64s(y.shape), i64s(kernel), i64s(strides),
                              i64s(pads), i64s(dilations)))
    _finish(dev)
    return y


def global_avgpool(x):
    rows = x.shape[0] * x.shape[1]
    inner = x.numel() // rows
    y = torch.empty(tuple(x.shape[:2]) + (1,) * (x.dim() - 2), device=x.device, dtype=torch.float32)
    _prep(x)
    dev = _dev(x)
    check(lib().nb2_row_mean(dev, _p(x), rows, inner, _p(y)))
    _finish(dev)
    return y
