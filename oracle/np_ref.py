"""TEST INFRASTRUCTURE ONLY: a numpy restatement of the reference CPU kernels.

This is the checker for the B200 path, never the thing measured or shipped.
Each op function restates the arithmetic of the reference's naive CPU kernel
(the oracle of NERT itself) and cites the file:line it follows. Contractions
and reductions accumulate in float64 and round once to float32, as the
reference does; elementwise ops compute in float32, as the reference does.

The restatement is pinned two ways (see tests/test_oracle.py): against the
hand-computed known answers of the reference's own tests
(tests/golden/known_answers.py), and against the reference library itself
(oracle/_ref/libnert_ref.so, compiled from the reference sources) on seeded
graphs.

``run(graph, inputs)`` interprets an ``nert_b200.onnx_io.Graph`` node by node.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def _attr(node, name, default):
    return node.attrs.get(name, default)


def _window_pads(auto_pad, in_sp, k, d, s, pads):
    """Per-axis (begin, end) padding; reference ResolvePads,
    src/kernels/conv.cpp:78-119 (MaxPool uses the same rule)."""
    r = len(in_sp)
    if auto_pad == "VALID":
        return [0] * r, [0] * r
    if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
        pb, pe = [], []
        for i in range(r):
            out = (in_sp[i] + s[i] - 1) // s[i]
            eff = d[i] * (k[i] - 1) + 1
            total = max(0, (out - 1) * s[i] + eff - in_sp[i])
            if auto_pad == "SAME_UPPER":
                pb.append(total // 2)
                pe.append(total - total // 2)
            else:
                pe.append(total // 2)
                pb.append(total - total // 2)
        return pb, pe
    if not pads:
        return [0] * r, [0] * r
    return list(pads[:r]), list(pads[r:])


def _out_dim(n, k, d, pb, pe, s, ceil_mode):
    """reference WindowOutput, src/kernels/conv.cpp:122-135."""
    eff = d * (k - 1) + 1
    numer = n + pb + pe - eff
    return ((numer + s - 1) // s if ceil_mode else numer // s) + 1


def conv(node, x, w, b=None):
    """reference kernels::Conv, src/kernels/conv.cpp:138-295 (float64
    accumulation from the bias, one float32 rounding per output)."""
    sp = x.ndim - 2
    group = _attr(node, "group", 1)
    s = _attr(node, "strides", [1] * sp)
    d = _attr(node, "dilations", [1] * sp)
    k = list(w.shape[2:])
    pb, pe = _window_pads(_attr(node, "auto_pad", "NOTSET"), list(x.shape[2:]), k, d, s, _attr(node, "pads", []))
    outs = [_out_dim(x.shape[2 + i], k[i], d[i], pb[i], pe[i], s[i], False) for i in range(sp)]
    n, c = x.shape[:2]
    m = w.shape[0]
    cg, mg = c // group, m // group
    xp = np.pad(x.astype(np.float64), [(0, 0), (0, 0)] + [(pb[i], pe[i]) for i in range(sp)])
    y = np.zeros([n, m] + outs, np.float64)
    w64 = w.astype(np.float64)
    for gi in range(group):
        xg = xp[:, gi * cg:(gi + 1) * cg]
        wg = w64[gi * mg:(gi + 1) * mg]
        # gather the window taps: cols[n, cg, *k, *outs]
        taps = []
        for idx in np.ndindex(*k):
            sl = [slice(None), slice(None)]
            for i in range(sp):
                start = idx[i] * d[i]
                sl.append(slice(start, start + s[i] * (outs[i] - 1) + 1, s[i]))
            taps.append(xg[tuple(sl)])
        cols = np.stack(taps, axis=2)  # [n, cg, K, *outs]
        wk = wg.reshape(mg, cg, -1)  # [mg, cg, K]
        y[:, gi * mg:(gi + 1) * mg] = np.einsum("ncq...,mcq->nm...", cols, wk, optimize=True)
    if b is not None:
        y += b.astype(np.float64).reshape([1, m] + [1] * sp)
    return y.astype(F32)


def conv_transpose(node, x, w, b=None):
    """reference kernels::ConvTranspose, src/kernels/conv_transpose.cpp:76-191:
    every input pixel scattered through the [C, M/group, KH, KW] weight to
    oh = ih*s - pad_begin + kh*d (kept when inside the output), bias first;
    summed here in float64 and rounded once (the reference sums in float32)."""
    group = _attr(node, "group", 1)
    s = _attr(node, "strides", [1, 1])
    d = _attr(node, "dilations", [1, 1])
    op = _attr(node, "output_padding", [0, 0])
    p = _attr(node, "pads", [0, 0, 0, 0])
    if _attr(node, "auto_pad", "NOTSET") == "VALID":
        p = [0, 0, 0, 0]
    n, c, H, W = x.shape
    kh, kw = w.shape[2], w.shape[3]
    mg = w.shape[1]
    m = mg * group
    cg = c // group
    oh = s[0] * (H - 1) + op[0] + d[0] * (kh - 1) + 1 - p[0] - p[2]
    ow = s[1] * (W - 1) + op[1] + d[1] * (kw - 1) + 1 - p[1] - p[3]
    # full (uncropped) canvas, then the window [p_begin, p_begin + out)
    fh = s[0] * (H - 1) + d[0] * (kh - 1) + 1 + op[0] + p[0] + p[2]
    fw = s[1] * (W - 1) + d[1] * (kw - 1) + 1 + op[1] + p[1] + p[3]
    full = np.zeros((n, m, fh, fw), np.float64)
    x64, w64 = x.astype(np.float64), w.astype(np.float64)
    for gi in range(group):
        xg = x64[:, gi * cg:(gi + 1) * cg]
        wg = w64[gi * cg:(gi + 1) * cg]  # [cg, mg, kh, kw]
        for i in range(kh):
            for j in range(kw):
                contrib = np.einsum("nchw,cm->nmhw", xg, wg[:, :, i, j])
                full[:, gi * mg:(gi + 1) * mg, i * d[0]:i * d[0] + s[0] * (H - 1) + 1:s[0],
                     j * d[1]:j * d[1] + s[1] * (W - 1) + 1:s[1]] += contrib
    y = full[:, :, p[0]:p[0] + oh, p[1]:p[1] + ow]
    if b is not None:
        y = y + b.astype(np.float64)[None, :, None, None]
    return y.astype(F32)


def gemm(node, a, b, c=None):
    """reference kernels::Gemm, src/kernels/gemm.cpp:59-137."""
    a = a.T if _attr(node, "transA", 0) else a
    b = b.T if _attr(node, "transB", 0) else b
    alpha = float(np.float32(_attr(node, "alpha", 1.0)))
    beta = float(np.float32(_attr(node, "beta", 1.0)))
    acc = a.astype(np.float64) @ b.astype(np.float64)
    v = alpha * acc
    if c is not None:
        v = v + beta * np.broadcast_to(c.astype(np.float64), v.shape)
    return v.astype(F32)


def matmul(node, a, b):
    """reference kernels::MatMul, src/kernels/mat_mul.cpp:79-169 (NumPy
    broadcasting, 1-D promotion, float64 accumulation)."""
    return np.matmul(a.astype(np.float64), b.astype(np.float64)).astype(F32)


def relu(node, x):
    """reference kernels::Relu, src/kernels/relu.cpp:29-54: max(0, x)."""
    return np.where(x > 0, x, F32(0)).astype(F32)


def _binary(fn):
    def op(node, a, b):
        """reference broadcast binaries, src/kernels/add.cpp:96-130 (and
        mul.cpp, sub.cpp, div.cpp): float32 arithmetic per element."""
        with np.errstate(all="ignore"):
            if a.dtype == np.int64:
                return fn(a, b, True)
            return fn(a.astype(F32), b.astype(F32), False).astype(F32)
    return op


def _div(a, b, is_int):
    if is_int:
        # int64 Div truncates toward zero (src/kernels/div.cpp:96-115)
        q = np.abs(a) // np.abs(b)
        return (np.sign(a) * np.sign(b) * q).astype(np.int64)
    return a / b


add = _binary(lambda a, b, i: a + b)
sub = _binary(lambda a, b, i: a - b)
mul = _binary(lambda a, b, i: a * b)
div = _binary(_div)


def sigmoid(node, x):
    """reference kernels::Sigmoid, src/kernels/sigmoid.cpp:52:
    1 / (1 + exp(-x)) in float32."""
    with np.errstate(over="ignore"):
        return (F32(1) / (F32(1) + np.exp(-x.astype(F32)))).astype(F32)


def maxpool(node, x):
    """reference kernels::MaxPool, src/kernels/max_pool.cpp:138-239:
    -inf outside the input, ceil_mode, dilation."""
    k = _attr(node, "kernel_shape", None)
    s = _attr(node, "strides", [1, 1])
    d = _attr(node, "dilations", [1, 1])
    ceil_mode = bool(_attr(node, "ceil_mode", 0))
    pb, pe = _window_pads(_attr(node, "auto_pad", "NOTSET"), list(x.shape[2:]), k, d, s, _attr(node, "pads", []))
    oh = _out_dim(x.shape[2], k[0], d[0], pb[0], pe[0], s[0], ceil_mode)
    ow = _out_dim(x.shape[3], k[1], d[1], pb[1], pe[1], s[1], ceil_mode)
    # pad generously so ceil_mode windows stay in range
    need_h = max(0, (oh - 1) * s[0] + d[0] * (k[0] - 1) + 1 - (x.shape[2] + pb[0]))
    need_w = max(0, (ow - 1) * s[1] + d[1] * (k[1] - 1) + 1 - (x.shape[3] + pb[1]))
    xp = np.pad(x, [(0, 0), (0, 0), (pb[0], need_h), (pb[1], need_w)], constant_values=-np.inf)
    y = np.full(x.shape[:2] + (oh, ow), -np.inf, F32)
    for i in range(k[0]):
        for j in range(k[1]):
            t = xp[:, :, i * d[0]:i * d[0] + s[0] * (oh - 1) + 1:s[0], j * d[1]:j * d[1] + s[1] * (ow - 1) + 1:s[1]]
            y = np.where(t > y, t, y)
    return y.astype(F32)


def average_pool(node, x):
    """reference kernels::AveragePool, src/kernels/average_pool.cpp:128-225:
    dilation 1, the window clipped to [start, min(start + k, in + pad_end)),
    in-range taps summed in float32 in row-major order, divided by the padded
    window size (count_include_pad) or the in-range tap count."""
    k = _attr(node, "kernel_shape", None)
    s = _attr(node, "strides", [1, 1])
    ceil_mode = bool(_attr(node, "ceil_mode", 0))
    include = bool(_attr(node, "count_include_pad", 0))
    pb, pe = _window_pads(_attr(node, "auto_pad", "NOTSET"), list(x.shape[2:]), k, [1, 1], s, _attr(node, "pads", []))
    H, W = x.shape[2], x.shape[3]
    oh = _out_dim(H, k[0], 1, pb[0], pe[0], s[0], ceil_mode)
    ow = _out_dim(W, k[1], 1, pb[1], pe[1], s[1], ceil_mode)
    hs = np.arange(oh) * s[0] - pb[0]
    he = np.minimum(hs + k[0], H + pe[0])
    h0, h1 = np.maximum(hs, 0), np.minimum(he, H)
    ws = np.arange(ow) * s[1] - pb[1]
    we = np.minimum(ws + k[1], W + pe[1])
    w0, w1 = np.maximum(ws, 0), np.minimum(we, W)
    acc = np.zeros(x.shape[:2] + (oh, ow), F32)
    for i in range(k[0]):
        ih = hs + i
        vh = (ih >= h0) & (ih < h1)
        rows = x[:, :, np.clip(ih, 0, H - 1), :]
        for j in range(k[1]):
            iw = ws + j
            vw = (iw >= w0) & (iw < w1)
            vals = rows[:, :, :, np.clip(iw, 0, W - 1)]
            acc = np.where(vh[:, None] & vw[None, :], (acc + vals).astype(F32), acc)
    div = ((he - hs)[:, None] * (we - ws)[None, :]) if include else ((h1 - h0)[:, None] * (w1 - w0)[None, :])
    with np.errstate(divide="ignore", invalid="ignore"):
        y = np.where(div > 0, acc / div.astype(F32), np.float32(0.0))
    return y.astype(F32)


def global_average_pool(node, x):
    """reference kernels::GlobalAveragePool, src/kernels/global_average_pool.cpp:32-68:
    float64 sum divided by the spatial size."""
    axes = tuple(range(2, x.ndim))
    sp = int(np.prod(x.shape[2:]))
    tot = x.astype(np.float64).sum(axis=axes, keepdims=True)
    return (tot / sp).astype(F32)


def flatten(node, x):
    """reference kernels::Flatten, src/kernels/flatten.cpp:31."""
    axis = _attr(node, "axis", 1)
    if axis < 0:
        axis += x.ndim
    return x.reshape(int(np.prod(x.shape[:axis])), -1)


def reshape(node, x, shape):
    """reference kernels::Reshape, src/kernels/reshape.cpp:32 (0 copies the
    input dim unless allowzero, -1 is inferred)."""
    shape = [int(v) for v in shape]
    allowzero = _attr(node, "allowzero", 0)
    out = [x.shape[i] if (v == 0 and not allowzero) else v for i, v in enumerate(shape)]
    return x.reshape(out)


def softmax(node, x):
    """reference kernels::Softmax, src/kernels/softmax.cpp:47-120: max shift,
    float64 exp and sum (opset >= 13 form: one axis)."""
    axis = _attr(node, "axis", -1)
    x64 = x.astype(np.float64)
    m = x64.max(axis=axis, keepdims=True)
    e = np.exp(x64 - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(F32)


def _unary32(fn, cite):
    def op(node, x):
        with np.errstate(all="ignore"):
            return fn(x.astype(F32)).astype(F32)
    op.__doc__ = f"reference {cite}: float32 std:: math per element."
    return op


def _erf32(x):
    import math as _m

    flat = x.astype(np.float64).ravel()
    return np.array([_m.erf(v) for v in flat], np.float64).astype(F32).reshape(x.shape)


erf = _unary32(_erf32, "kernels::Erf, src/kernels/erf.cpp:27-50")
sqrt = _unary32(np.sqrt, "kernels::Sqrt, src/kernels/sqrt.cpp")
tanh = _unary32(np.tanh, "kernels::Tanh, src/kernels/tanh.cpp")
exp = _unary32(np.exp, "kernels::Exp, src/kernels/exp.cpp")
neg = _unary32(np.negative, "kernels::Neg, src/kernels/neg.cpp")
absolute = _unary32(np.abs, "kernels::Abs, src/kernels/abs.cpp")


def power(node, a, b):
    """reference kernels::Pow, src/kernels/pow.cpp: float32 std::pow with broadcasting."""
    with np.errstate(all="ignore"):
        return np.power(a.astype(F32), b.astype(F32)).astype(F32)


def identity(node, x):
    return x.copy()


def layer_norm(node, x, scale, bias=None):
    """reference kernels::LayerNormalization, src/kernels/layer_normalization.cpp:77-160:
    float64 mean and population variance over the axes from `axis`."""
    axis = _attr(node, "axis", -1)
    if axis < 0:
        axis += x.ndim
    eps = float(np.float32(_attr(node, "epsilon", 1e-5)))
    axes = tuple(range(axis, x.ndim))
    x64 = x.astype(np.float64)
    mean = x64.mean(axis=axes, keepdims=True)
    var = ((x64 - mean) ** 2).mean(axis=axes, keepdims=True)
    inv = 1.0 / np.sqrt(var + eps)
    y = (x64 - mean) * inv * scale.astype(np.float64)
    if bias is not None:
        y = y + bias.astype(np.float64)
    return y.astype(F32), mean.astype(F32), inv.astype(F32)


def transpose(node, x):
    """reference kernels::Transpose, src/kernels/transpose.cpp:54 (default: reverse)."""
    perm = _attr(node, "perm", None)
    return np.ascontiguousarray(np.transpose(x, perm))


def concat(node, *xs):
    """reference kernels::Concat, src/kernels/concat.cpp:64."""
    return np.concatenate(xs, axis=_attr(node, "axis", 0))


def split(node, x, sizes=None):
    """reference kernels::Split, src/kernels/split.cpp:65 (sizes input from
    opset 13, 'split' attribute before, else even split)."""
    axis = _attr(node, "axis", 0)
    n_out = len(node.outputs)
    if sizes is None:
        sizes = _attr(node, "split", None)
    if sizes is None or len(sizes) == 0:
        dim = x.shape[axis]
        each = -(-dim // n_out)
        sizes = [min(each, dim - i * each) for i in range(n_out)]
    idx = np.cumsum(sizes)[:-1]
    return [np.ascontiguousarray(p) for p in np.split(x, idx, axis=axis)]


def slice_op(node, x, starts, ends, axes=None, steps=None):
    """reference kernels::Slice, src/kernels/slice.cpp (ONNX clamping)."""
    starts, ends = [int(v) for v in starts], [int(v) for v in ends]
    axes = list(range(len(starts))) if axes is None else [int(v) for v in axes]
    steps = [1] * len(starts) if steps is None else [int(v) for v in steps]
    sl = [slice(None)] * x.ndim
    for s, e, a, st in zip(starts, ends, axes, steps):
        a = a + x.ndim if a < 0 else a
        dim = x.shape[a]
        s = s + dim if s < 0 else s
        e = e + dim if e < 0 else e
        if st > 0:
            s, e = min(max(s, 0), dim), min(max(e, 0), dim)
        else:
            s, e = min(max(s, 0), dim - 1), min(max(e, -1), dim - 1)
            e = None if e < 0 else e
        sl[a] = slice(s, e, st)
    return np.ascontiguousarray(x[tuple(sl)])


def gather(node, x, idx):
    """reference kernels::Gather, src/kernels/gather.cpp:49-129: negative
    indices wrap; out-of-range indices are an error."""
    axis = _attr(node, "axis", 0)
    if axis < 0:
        axis += x.ndim
    dim = x.shape[axis]
    idx = np.asarray(idx, np.int64)
    if ((idx < -dim) | (idx >= dim)).any():
        raise IndexError("Gather: index out of range")
    return np.take(x, np.where(idx < 0, idx + dim, idx), axis=axis)


def topk(node, x, k):
    """reference kernels::TopK, src/kernels/top_k.cpp:53-142: largest, sorted,
    order (value desc, index asc)."""
    k = int(np.asarray(k).ravel()[0])
    axis = _attr(node, "axis", -1)
    xm = np.moveaxis(x, axis, -1)
    flat = xm.reshape(-1, xm.shape[-1])
    vals = np.empty((flat.shape[0], k), F32)
    inds = np.empty((flat.shape[0], k), np.int64)
    for r in range(flat.shape[0]):
        order = np.lexsort((np.arange(flat.shape[1]), -flat[r].astype(np.float64)))[:k]
        inds[r] = order
        vals[r] = flat[r][order]
    shape = xm.shape[:-1] + (k,)
    return (np.moveaxis(vals.reshape(shape), -1, axis), np.moveaxis(inds.reshape(shape), -1, axis))


def _cround(x):
    """C++ std::round: halves away from zero."""
    return math.floor(abs(x) + 0.5) * (1 if x >= 0 else -1)


def _nearest(mode, x, n):
    """reference NearestIndex, src/kernels/resize.cpp:78-93."""
    f = math.floor(x)
    if mode == "round_prefer_floor":
        i = f if x - f == 0.5 else _cround(x)
    elif mode == "round_prefer_ceil":
        i = _cround(x)
    elif mode == "floor":
        i = f
    else:
        i = math.ceil(x)
    return min(max(int(i), 0), n - 1)


def resize(node, x, roi=None, scales=None, sizes=None):
    """reference kernels::Resize, src/kernels/resize.cpp:62-290: per-axis
    tables from the coordinate transform; nearest or (multi)linear."""
    mode = _attr(node, "mode", "nearest")
    tr = _attr(node, "coordinate_transformation_mode", "half_pixel")
    nm = _attr(node, "nearest_mode", "round_prefer_floor")
    r = x.ndim
    if sizes is not None and np.size(sizes) > 0:
        out = [int(v) for v in sizes]
        sc = [float(np.float32(out[i]) / np.float32(x.shape[i])) for i in range(r)]
    else:
        sc = [float(v) for v in np.asarray(scales, F32)]
        out = [int(math.floor(x.shape[i] * sc[i])) for i in range(r)]
    tables = []
    for d in range(r):
        tab = []
        for o in range(out[d]):
            xo = float(o)
            if tr == "half_pixel":
                xs = (xo + 0.5) / sc[d] - 0.5
            elif tr == "pytorch_half_pixel":
                xs = (xo + 0.5) / sc[d] - 0.5 if out[d] > 1 else 0.0
            elif tr == "align_corners":
                xs = 0.0 if out[d] == 1 else xo * (x.shape[d] - 1) / (out[d] - 1)
            else:
                xs = xo / sc[d]
            if mode == "nearest":
                i = _nearest(nm, xs, x.shape[d])
                tab.append((i, i, 0.0))
            else:
                cl = min(max(xs, 0.0), float(x.shape[d] - 1))
                lo = int(math.floor(cl))
                hi = min(lo + 1, x.shape[d] - 1)
                tab.append((lo, hi, 0.0 if hi == lo else cl - lo))
        tables.append(tab)
    if mode == "nearest":
        idx = [np.array([t[0] for t in tab]) for tab in tables]
        return np.ascontiguousarray(x[np.ix_(*idx)])
    y = np.zeros(out, np.float64)
    x64 = x.astype(np.float64)
    for pos in np.ndindex(*out):
        taps = [((), 1.0)]
        for d in range(r):
            lo, hi, w = tables[d][pos[d]]
            if w == 0.0:
                taps = [(p + (lo,), wt) for p, wt in taps]
            else:
                taps = [(p + (lo,), wt * (1 - w)) for p, wt in taps] + [(p + (hi,), wt * w) for p, wt in taps]
        y[pos] = sum(wt * x64[p] for p, wt in taps)
    return y.astype(x.dtype)


def cast(node, x):
    """reference kernels::Cast, src/kernels/cast.cpp: float->int64 truncates."""
    to = _attr(node, "to", 1)
    if to == 7:
        return np.trunc(x).astype(np.int64) if x.dtype != np.int64 else x.copy()
    if to == 9:
        return x != 0
    return x.astype(F32)


def unsqueeze(node, x, axes=None):
    """reference kernels::Unsqueeze, src/kernels/unsqueeze.cpp."""
    axes = _attr(node, "axes", None) if axes is None else axes
    r = x.ndim + len(axes)
    axes = sorted(int(a) + r if a < 0 else int(a) for a in axes)
    y = x
    for a in axes:
        y = np.expand_dims(y, a)
    return y


def squeeze(node, x, axes=None):
    """reference kernels::Squeeze, src/kernels/squeeze.cpp."""
    axes = _attr(node, "axes", None) if axes is None else axes
    if axes is None or len(axes) == 0:
        return np.squeeze(x)
    return np.squeeze(x, axis=tuple(int(a) + x.ndim if a < 0 else int(a) for a in axes))


def reduce_mean(node, x, axes=None):
    """reference kernels::ReduceMean, src/kernels/reduce_mean.cpp:44 (float64 sum)."""
    axes = _attr(node, "axes", None) if axes is None else axes
    keep = bool(_attr(node, "keepdims", 1))
    ax = tuple(range(x.ndim)) if axes is None or len(axes) == 0 else tuple(int(a) % x.ndim for a in axes)
    return x.astype(np.float64).mean(axis=ax, keepdims=keep).astype(F32)


def _softmax_versioned(node, x):
    """Softmax: opset < 13 coerces to 2-D at `axis` (default 1,
    src/softmax_form.hpp); opset >= 13 normalises one axis (default -1)."""
    if getattr(node, "opset", 13) < 13:
        axis = _attr(node, "axis", 1)
        if axis < 0:
            axis += x.ndim
        flat = x.reshape(int(np.prod(x.shape[:axis])), -1).astype(np.float64)
        m = flat.max(axis=1, keepdims=True)
        e = np.exp(flat - m)
        return (e / e.sum(axis=1, keepdims=True)).astype(F32).reshape(x.shape)
    return softmax(node, x)


OPS = {
    "Erf": erf,
    "Sqrt": sqrt,
    "Tanh": tanh,
    "Exp": exp,
    "Neg": neg,
    "Abs": absolute,
    "Pow": power,
    "Identity": identity,
    "LayerNormalization": layer_norm,
    "Transpose": transpose,
    "Concat": concat,
    "Split": split,
    "Slice": slice_op,
    "Gather": gather,
    "TopK": topk,
    "Resize": resize,
    "Cast": cast,
    "Unsqueeze": unsqueeze,
    "Squeeze": squeeze,
    "ReduceMean": reduce_mean,
    "Conv": conv,
    "Gemm": gemm,
    "MatMul": matmul,
    "Relu": relu,
    "Add": add,
    "Sub": sub,
    "Mul": mul,
    "Div": div,
    "Sigmoid": sigmoid,
    "MaxPool": maxpool,
    "ConvTranspose": conv_transpose,
    "AveragePool": average_pool,
    "GlobalAveragePool": global_average_pool,
    "Flatten": flatten,
    "Reshape": reshape,
    "Softmax": _softmax_versioned,
}


def run(graph, inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Interpret ``graph`` in node order (the reference executor's loop,
    src/executor.cpp:480-535) and return its declared outputs."""
    env = dict(graph.initializers)
    env.update(inputs)
    for node in graph.nodes:
        node.opset = graph.opset
        fn = OPS.get(node.op_type)
        if fn is None:
            raise NotImplementedError(f"np_ref: no restatement of {node.op_type}")
        args = [env[n] if n else None for n in node.inputs]
        res = fn(node, *args)
        if isinstance(res, (list, tuple)):
            for name, r in zip(node.outputs, res):
                env[name] = r
        else:
            env[node.outputs[0]] = res
    return {name: env[name] for name, _, _ in graph.outputs}


def run_op(op_type: str, attrs: dict, inputs: list, opset: int = 13, n_out: int = 1):
    """Run one op on explicit arrays (None for an omitted optional input)."""
    from nert_b200.onnx_io import Node

    node = Node(op_type, [], [f"o{i}" for i in range(n_out)], "op", dict(attrs))
    node.opset = opset
    return OPS[op_type](node, *inputs)


__all__ = ["run", "run_op", "OPS", "math"]
