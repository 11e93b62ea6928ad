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


OPS = {
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
    "GlobalAveragePool": global_average_pool,
    "Flatten": flatten,
    "Reshape": reshape,
    "Softmax": softmax,
}


def run(graph, inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Interpret ``graph`` in node order (the reference executor's loop,
    src/executor.cpp:480-535) and return its declared outputs."""
    env = dict(graph.initializers)
    env.update(inputs)
    for node in graph.nodes:
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


def run_op(op_type: str, attrs: dict, inputs: list[np.ndarray]) -> np.ndarray:
    """Run one op on explicit arrays (for the known-answer checks)."""
    from nert_b200.onnx_io import Node

    return OPS[op_type](Node(op_type, [], [], "op", dict(attrs)), *inputs)


__all__ = ["run", "run_op", "OPS", "math"]
