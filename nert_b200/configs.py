"""Synthetic graphs for the five benchmark configurations.

Each builder returns an :class:`onnx_io.Graph` whose weights come from the
seeded generator in :mod:`synth`, so the reference loader, the numpy oracle
and the B200 engine all see identical bits.

BatchNormalization has no row in the reference (its loader rejects it,
``src/model_loader.cpp:1677-1690``); the reference only ever meets BN folded
into Conv by the exporter. The builders therefore fold BN at construction:
``W' = W * gamma / sqrt(var + eps)``, ``b' = beta - mean * gamma / sqrt(var + eps)``
with gamma=1, beta=0, mean=0, var ~ U[0.5, 1.5], eps=1e-5. The folded bias is
zero but is kept as an explicit Conv bias input.
"""

from __future__ import annotations

import math

import numpy as np

from . import synth
from .onnx_io import FLOAT, Graph


class _Builder:
    def __init__(self, config: str, opset: int = 13, bn_nodes: bool = False):
        self.config = config
        self.g = Graph(name=config, opset=opset)
        self.bn_nodes = bn_nodes

    def seed(self, name: str) -> int:
        return synth.seed_of(self.config, name)

    def conv_bn(self, x: str, cin: int, cout: int, k: int, stride: int = 1, pad: int = 0,
                name: str = "conv", groups: int = 1) -> str:
        """Conv + folded BatchNorm (Kaiming-normal weights, std sqrt(2/fan_in))."""
        fan_in = (cin // groups) * k * k
        w = synth.normal((cout, cin // groups, k, k), math.sqrt(2.0 / fan_in), self.seed(name + ".w"))
        var = synth.uniform((cout,), 0.5, 1.5, self.seed(name + ".bn_var"))
        if self.bn_nodes:
            # the unfolded export: Conv without bias, then BatchNormalization
            # (gamma 1, beta 0, mean 0, the seeded variance, epsilon 1e-5)
            y = self.g.op("Conv", [x, self.g.const(name + ".weight", w)], name=name, kernel_shape=[k, k],
                          strides=[stride, stride], pads=[pad, pad, pad, pad], dilations=[1, 1], group=groups)
            stats = [self.g.const(name + ".bn_" + t, v) for t, v in
                     (("scale", np.ones((cout,), np.float32)), ("bias", np.zeros((cout,), np.float32)),
                      ("mean", np.zeros((cout,), np.float32)), ("var", var))]
            return self.g.op("BatchNormalization", [y] + stats, name=name + ".bn", epsilon=1e-5)
        scale = (1.0 / np.sqrt(var.astype(np.float64) + 1e-5)).astype(np.float32)
        w = (w * scale[:, None, None, None]).astype(np.float32)
        b = np.zeros((cout,), np.float32)
        wn = self.g.const(name + ".weight", w)
        bn = self.g.const(name + ".bias", b)
        return self.g.op("Conv", [x, wn, bn], name=name, kernel_shape=[k, k], strides=[stride, stride],
                         pads=[pad, pad, pad, pad], dilations=[1, 1], group=groups)

    def relu(self, x: str, name: str) -> str:
        return self.g.op("Relu", [x], name=name)


def resnet18(batch: int = 1, config: str = "resnet18", bn_nodes: bool = False) -> Graph:
    """torchvision-style ResNet-18 (BasicBlock 2/2/2/2, widths 64-512).
    bn_nodes=True keeps every BatchNormalization as a node after its Conv (an
    export without the fold); the same seeds give the folded graph's values."""
    return _resnet(batch, config, bottleneck=False, blocks=(2, 2, 2, 2), bn_nodes=bn_nodes)


def resnet50(batch: int = 1, config: str = "resnet50", softmax: bool = True, expose_logits: bool = False) -> Graph:
    """torchvision-style ResNet-50 (Bottleneck 3/4/6/3, widths 64-2048) + Softmax.

    With random Kaiming weights the logits spread over hundreds, so the
    softmax is nearly one-hot; ``expose_logits`` adds the Gemm output
    ``fc_out`` as a second graph output so parity checks see every logit."""
    return _resnet(batch, config, bottleneck=True, blocks=(3, 4, 6, 3), softmax=softmax, expose_logits=expose_logits)


def _resnet(batch: int, config: str, bottleneck: bool, blocks, softmax: bool = False,
            expose_logits: bool = False, bn_nodes: bool = False) -> Graph:
    b = _Builder(config, bn_nodes=bn_nodes)
    g = b.g
    x = g.add_input("input", [batch, 3, 224, 224])
    y = b.relu(b.conv_bn(x, 3, 64, 7, 2, 3, name="conv1"), "relu1")
    y = g.op("MaxPool", [y], name="maxpool", kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])
    cin = 64
    widths = (64, 128, 256, 512)
    expansion = 4 if bottleneck else 1
    for li, (nblk, width) in enumerate(zip(blocks, widths)):
        for bi in range(nblk):
            stride = 2 if (li > 0 and bi == 0) else 1
            pre = f"layer{li + 1}.{bi}"
            cout = width * expansion
            if bottleneck:
                t = b.relu(b.conv_bn(y, cin, width, 1, 1, 0, name=pre + ".conv1"), pre + ".relu1")
                t = b.relu(b.conv_bn(t, width, width, 3, stride, 1, name=pre + ".conv2"), pre + ".relu2")
                t = b.conv_bn(t, width, cout, 1, 1, 0, name=pre + ".conv3")
            else:
                t = b.relu(b.conv_bn(y, cin, width, 3, stride, 1, name=pre + ".conv1"), pre + ".relu1")
                t = b.conv_bn(t, width, cout, 3, 1, 1, name=pre + ".conv2")
            if stride != 1 or cin != cout:
                sc = b.conv_bn(y, cin, cout, 1, stride, 0, name=pre + ".downsample")
            else:
                sc = y
            y = g.op("Add", [t, sc], name=pre + ".add")
            y = b.relu(y, pre + ".relu_out")
            cin = cout
    y = g.op("GlobalAveragePool", [y], name="avgpool")
    y = g.op("Flatten", [y], name="flatten", axis=1)
    wfc = synth.normal((1000, cin), math.sqrt(2.0 / cin), b.seed("fc.w"))
    bound = 1.0 / math.sqrt(cin)
    bfc = synth.uniform((1000,), -bound, bound, b.seed("fc.b"))
    y = g.op("Gemm", [y, g.const("fc.weight", wfc), g.const("fc.bias", bfc)], name="fc", transB=1)
    logits = y
    if softmax:
        y = g.op("Softmax", [y], name="softmax", axis=-1)
    g.add_output(y, None, FLOAT)
    if softmax and expose_logits:
        g.add_output(logits, None, FLOAT)
    return g


def resnet_input(batch: int, config: str = "resnet18") -> np.ndarray:
    """The seeded U[-1, 1] input image batch for the ResNet configs."""
    return synth.uniform((batch, 3, 224, 224), -1.0, 1.0, synth.seed_of(config, "input"))


# ---- ViT-B/16 (config 4) --------------------------------------------------------

def vit_b16(batch: int = 32, config: str = "vit_b16", layers: int = 12, d: int = 768, heads: int = 12,
            mlp: int = 3072, classes: int = 1000) -> Graph:
    """ViT-B/16-style encoder at opset 17 (LayerNormalization exists from 17).

    Patch Conv 16x16/s16 -> tokens, cls token + learned positional embedding,
    `layers` pre-LN blocks (MatMul Q/K/V, QK^T / 8, Softmax, MatMul V,
    projection + residual; MLP with GELU written as x*0.5*(1+Erf(x/sqrt 2)) +
    residual), final LN, Gather of the cls token, Gemm head. Weights N(0, 0.02),
    LN gamma=1, beta=0. The cls token is stored pre-tiled to the batch so the
    graph needs no Expand."""
    b = _Builder(config, opset=17)
    g = b.g
    hd = d // heads
    n_tok = 197

    def w(name, shape, std=0.02):
        return g.const(name, synth.normal(shape, std, b.seed(name)))

    def linear(x, din, dout, name):
        y = g.op("MatMul", [x, w(name + ".w", (din, dout))], name=name)
        return g.op("Add", [y, w(name + ".b", (dout,))], name=name + ".bias")

    def ln(x, name):
        return g.op("LayerNormalization", [x, g.const(name + ".g", np.ones((d,), np.float32)),
                                           g.const(name + ".b", np.zeros((d,), np.float32))],
                    name=name, axis=-1, epsilon=1e-6)

    def i64(name, vals):
        return g.const(name, np.array(vals, np.int64))

    x = g.add_input("input", [batch, 3, 224, 224])
    p = g.op("Conv", [x, w("patch.w", (d, 3, 16, 16)), w("patch.b", (d,))], name="patch", kernel_shape=[16, 16],
             strides=[16, 16])
    p = g.op("Reshape", [p, i64("patch.shape", [batch, d, 196])], name="patch.flat")
    p = g.op("Transpose", [p], name="patch.tokens", perm=[0, 2, 1])
    cls = np.repeat(synth.normal((1, 1, d), 0.02, b.seed("cls")), batch, axis=0)
    t = g.op("Concat", [g.const("cls", cls), p], name="tokens", axis=1)
    t = g.op("Add", [t, w("pos", (1, n_tok, d))], name="pos_add")
    heads_shape = i64("heads.shape", [batch, n_tok, heads, hd])
    merge_shape = i64("merge.shape", [batch, n_tok, d])
    for li in range(layers):
        pre = f"blk{li}"
        h = ln(t, pre + ".ln1")
        q = g.op("Transpose", [g.op("Reshape", [linear(h, d, d, pre + ".q"), heads_shape], name=pre + ".q.r")],
                 name=pre + ".q.t", perm=[0, 2, 1, 3])
        k = g.op("Transpose", [g.op("Reshape", [linear(h, d, d, pre + ".k"), heads_shape], name=pre + ".k.r")],
                 name=pre + ".k.t", perm=[0, 2, 3, 1])
        v = g.op("Transpose", [g.op("Reshape", [linear(h, d, d, pre + ".v"), heads_shape], name=pre + ".v.r")],
                 name=pre + ".v.t", perm=[0, 2, 1, 3])
        s = g.op("MatMul", [q, k], name=pre + ".qk")
        s = g.op("Div", [s, g.const(pre + ".scale", np.array(np.sqrt(hd), np.float32))], name=pre + ".scaled")
        a = g.op("Softmax", [s], name=pre + ".softmax", axis=-1)
        c = g.op("MatMul", [a, v], name=pre + ".av")
        c = g.op("Reshape", [g.op("Transpose", [c], name=pre + ".ctx.t", perm=[0, 2, 1, 3]), merge_shape],
                 name=pre + ".ctx")
        t = g.op("Add", [linear(c, d, d, pre + ".proj"), t], name=pre + ".res1")
        h = ln(t, pre + ".ln2")
        f = linear(h, d, mlp, pre + ".fc1")
        e = g.op("Erf", [g.op("Div", [f, g.const(pre + ".sqrt2", np.array(np.sqrt(2.0), np.float32))],
                              name=pre + ".gelu.div")], name=pre + ".gelu.erf")
        e = g.op("Add", [e, g.const(pre + ".one", np.array(1.0, np.float32))], name=pre + ".gelu.add")
        f = g.op("Mul", [g.op("Mul", [f, e], name=pre + ".gelu.mul"), g.const(pre + ".half", np.array(0.5, np.float32))],
                 name=pre + ".gelu.half")
        t = g.op("Add", [linear(f, mlp, d, pre + ".fc2"), t], name=pre + ".res2")
    t = ln(t, "ln_f")
    c = g.op("Gather", [t, g.const("cls_index", np.array(0, np.int64))], name="cls_token", axis=1)
    y = g.op("Gemm", [c, w("head.w", (classes, d)), w("head.b", (classes,))], name="head", transB=1)
    g.add_output(y, None, FLOAT)
    return g


def vit_input(batch: int, config: str = "vit_b16") -> np.ndarray:
    return synth.uniform((batch, 3, 224, 224), -1.0, 1.0, synth.seed_of(config, "input"))


# ---- YOLOv8n-style detector (config 3) -------------------------------------------

# The Kaiming-initialised SiLU stack shrinks activations (x*sigmoid(x) ~ x/2
# near 0), leaving class logits around 0.006 std; this factor on the last
# class conv brings them to O(1) so the sigmoid scores are spread out and the
# TopK boundary is not a pile of near-ties.
CLS_HEAD_SCALE = 90.0

def yolov8n(batch: int = 1, config: str = "yolov8n", size: int = 640, classes: int = 80, topk: int = 300,
            expose_scores: bool = False) -> Graph:
    """YOLOv8n-style detector at opset 13.

    CSP backbone of Conv + SiLU (Sigmoid * Mul), C2f blocks built from Split /
    bottlenecks / Concat, SPPF with three MaxPool 5x5 s1; PAN neck with nearest
    Resize x2 and Concat; decoupled head over the 80x80 + 40x40 + 20x20 = 8400
    anchors with 4x16 DFL bins and 80 class logits; DFL as Softmax over the 16
    bins + 1x1 Conv with weights 0..15; boxes decoded from anchor points and
    strides; TopK k=300 over the 8400*80 sigmoid scores; Gather of the chosen
    boxes (anchor = index // 80, class = index - 80 * anchor, int64).
    Kaiming weights; the class-head output conv is scaled so logits are O(1).
    ``expose_scores`` adds three more graph outputs, the flattened pre-TopK
    scores ``scores.flat_out`` [B, 8400*80], the decoded boxes ``boxes_out``
    [B, 4, 8400] and the TopK indices ``topk_out1`` [B, k] (int64), so the
    selection can be checked against the scores and boxes the same run
    computed."""
    b = _Builder(config)
    g = b.g

    def conv(x, cin, cout, k, s, name, act=True, scale=1.0):
        fan = cin * k * k
        wt = synth.normal((cout, cin, k, k), scale * math.sqrt(2.0 / fan), b.seed(name + ".w"))
        bi = synth.normal((cout,), 0.01 * scale, b.seed(name + ".b"))
        y = g.op("Conv", [x, g.const(name + ".w", wt), g.const(name + ".b", bi)], name=name, kernel_shape=[k, k],
                 strides=[s, s], pads=[k // 2] * 4)
        if act:
            y = g.op("Mul", [y, g.op("Sigmoid", [y], name=name + ".sig")], name=name + ".silu")
        return y

    def c2f(x, cin, cout, n, shortcut, name):
        c = cout // 2
        y = conv(x, cin, 2 * c, 1, 1, name + ".cv1")
        parts = g.op("Split", [y, g.const(name + ".split", np.array([c, c], np.int64))], n_out=2, name=name + ".split",
                     axis=1)
        outs = list(parts)
        cur = parts[1]
        for i in range(n):
            t = conv(cur, c, c, 3, 1, f"{name}.m{i}.cv1")
            t = conv(t, c, c, 3, 1, f"{name}.m{i}.cv2")
            cur = g.op("Add", [cur, t], name=f"{name}.m{i}.add") if shortcut else t
            outs.append(cur)
        y = g.op("Concat", outs, name=name + ".cat", axis=1)
        return conv(y, (2 + n) * c, cout, 1, 1, name + ".cv2")

    x = g.add_input("images", [batch, 3, size, size])
    x = conv(x, 3, 16, 3, 2, "b0")
    x = conv(x, 16, 32, 3, 2, "b1")
    x = c2f(x, 32, 32, 1, True, "b2")
    x = conv(x, 32, 64, 3, 2, "b3")
    p3 = c2f(x, 64, 64, 2, True, "b4")
    x = conv(p3, 64, 128, 3, 2, "b5")
    p4 = c2f(x, 128, 128, 2, True, "b6")
    x = conv(p4, 128, 256, 3, 2, "b7")
    x = c2f(x, 256, 256, 1, True, "b8")
    # SPPF
    t = conv(x, 256, 128, 1, 1, "sppf.cv1")
    m1 = g.op("MaxPool", [t], name="sppf.m1", kernel_shape=[5, 5], strides=[1, 1], pads=[2, 2, 2, 2])
    m2 = g.op("MaxPool", [m1], name="sppf.m2", kernel_shape=[5, 5], strides=[1, 1], pads=[2, 2, 2, 2])
    m3 = g.op("MaxPool", [m2], name="sppf.m3", kernel_shape=[5, 5], strides=[1, 1], pads=[2, 2, 2, 2])
    p5 = conv(g.op("Concat", [t, m1, m2, m3], name="sppf.cat", axis=1), 512, 256, 1, 1, "sppf.cv2")
    # PAN neck
    empty = g.const("roi", np.zeros((0,), np.float32))
    up = g.const("up2", np.array([1, 1, 2, 2], np.float32))
    u = g.op("Resize", [p5, empty, up], name="up1", mode="nearest")
    n4 = c2f(g.op("Concat", [u, p4], name="cat1", axis=1), 384, 128, 1, False, "n12")
    u = g.op("Resize", [n4, empty, up], name="up2", mode="nearest")
    o3 = c2f(g.op("Concat", [u, p3], name="cat2", axis=1), 192, 64, 1, False, "n15")
    d = conv(o3, 64, 64, 3, 2, "n16")
    o4 = c2f(g.op("Concat", [d, n4], name="cat3", axis=1), 192, 128, 1, False, "n18")
    d = conv(o4, 128, 128, 3, 2, "n19")
    o5 = c2f(g.op("Concat", [d, p5], name="cat4", axis=1), 384, 256, 1, False, "n21")
    # decoupled head
    levels = []
    for i, (feat, c) in enumerate(((o3, 64), (o4, 128), (o5, 256))):
        bx = conv(conv(feat, c, 64, 3, 1, f"h{i}.box0"), 64, 64, 3, 1, f"h{i}.box1")
        bx = conv(bx, 64, 64, 1, 1, f"h{i}.box2", act=False)
        cl = conv(conv(feat, c, 80, 3, 1, f"h{i}.cls0"), 80, 80, 3, 1, f"h{i}.cls1")
        cl = conv(cl, 80, classes, 1, 1, f"h{i}.cls2", act=False, scale=CLS_HEAD_SCALE)
        hw = (size // (8 << i)) ** 2
        cat = g.op("Concat", [bx, cl], name=f"h{i}.cat", axis=1)
        levels.append(g.op("Reshape", [cat, g.const(f"h{i}.shape", np.array([batch, 64 + classes, hw], np.int64))],
                           name=f"h{i}.flat"))
    na = sum((size // s) ** 2 for s in (8, 16, 32))
    out = g.op("Concat", levels, name="head.cat", axis=2)
    box, cls = g.op("Split", [out, g.const("head.split", np.array([64, classes], np.int64))], n_out=2,
                    name="head.split", axis=1)
    # DFL: softmax over 16 bins, expectation by a fixed 1x1 conv
    dfl = g.op("Reshape", [box, g.const("dfl.shape", np.array([batch, 4, 16, na], np.int64))], name="dfl.r")
    dfl = g.op("Softmax", [g.op("Transpose", [dfl], name="dfl.t", perm=[0, 2, 1, 3])], name="dfl.softmax", axis=1)
    dfl = g.op("Conv", [dfl, g.const("dfl.w", np.arange(16, dtype=np.float32).reshape(1, 16, 1, 1))], name="dfl.conv")
    dist = g.op("Reshape", [dfl, g.const("dist.shape", np.array([batch, 4, na], np.int64))], name="dist")
    # dist2bbox (xywh) * stride
    anchors, strides = [], []
    for s in (8, 16, 32):
        n = size // s
        ys, xs = np.meshgrid(np.arange(n) + 0.5, np.arange(n) + 0.5, indexing="ij")
        anchors.append(np.stack([xs.ravel(), ys.ravel()]))
        strides.append(np.full((n * n,), s, np.float32))
    anc = g.const("anchors", np.concatenate(anchors, axis=1).astype(np.float32)[None])   # [1,2,na]
    st = g.const("strides", np.concatenate(strides)[None, None])                            # [1,1,na]
    lt, rb = g.op("Split", [dist, g.const("dist.split", np.array([2, 2], np.int64))], n_out=2, name="dist.split",
                  axis=1)
    x1y1 = g.op("Sub", [anc, lt], name="x1y1")
    x2y2 = g.op("Add", [anc, rb], name="x2y2")
    cxy = g.op("Div", [g.op("Add", [x1y1, x2y2], name="cxy.sum"), g.const("two", np.array(2.0, np.float32))],
               name="cxy")
    wh = g.op("Sub", [x2y2, x1y1], name="wh")
    boxes = g.op("Mul", [g.op("Concat", [cxy, wh], name="xywh", axis=1), st], name="boxes")   # [B,4,na]
    # scores and selection
    scores = g.op("Sigmoid", [cls], name="scores")                                            # [B,80,na]
    flat = g.op("Reshape", [g.op("Transpose", [scores], name="scores.t", perm=[0, 2, 1]),
                            g.const("scores.shape", np.array([batch, na * classes], np.int64))], name="scores.flat")
    top_v, top_i = g.op("TopK", [flat, g.const("k", np.array([topk], np.int64))], n_out=2, name="topk", axis=-1)
    anchor_i = g.op("Div", [top_i, g.const("ncls", np.array(classes, np.int64))], name="anchor_idx")
    class_i = g.op("Sub", [top_i, g.op("Mul", [anchor_i, g.const("ncls2", np.array(classes, np.int64))],
                                       name="anchor_base")], name="class_idx")
    offs = g.const("batch_off", (np.arange(batch, dtype=np.int64) * na)[:, None])
    flat_i = g.op("Reshape", [g.op("Add", [anchor_i, offs], name="flat_idx"),
                              g.const("flat_idx.shape", np.array([batch * topk], np.int64))], name="flat_idx.r")
    box_rows = g.op("Reshape", [g.op("Transpose", [boxes], name="boxes.t", perm=[0, 2, 1]),
                                g.const("boxes.shape", np.array([batch * na, 4], np.int64))], name="box_rows")
    sel = g.op("Gather", [box_rows, flat_i], name="box_gather", axis=0)
    sel = g.op("Reshape", [sel, g.const("sel.shape", np.array([batch, topk, 4], np.int64))], name="det_boxes")
    g.add_output(top_v, None, FLOAT)
    g.add_output(sel, None, FLOAT)
    g.add_output(class_i, None, 7)
    if expose_scores:
        g.add_output(flat, None, FLOAT)
        g.add_output(boxes, None, FLOAT)
        g.add_output(top_i, None, 7)
    return g


def yolo_input(batch: int, config: str = "yolov8n", size: int = 640) -> np.ndarray:
    return synth.uniform((batch, 3, size, size), 0.0, 1.0, synth.seed_of(config, "input"))


# ---- single-op sweep (config 1) ---------------------------------------------------

# (name, C, H, W, M, k, stride, pad) at batch 32
SWEEP_CONVS = [
    ("stem_3_64_k7s2_224", 3, 224, 224, 64, 7, 2, 3),
    ("c64_k3_56", 64, 56, 56, 64, 3, 1, 1),
    ("c128_k3_28", 128, 28, 28, 128, 3, 1, 1),
    ("c256_k3_14", 256, 14, 14, 256, 3, 1, 1),
    ("c512_k3_7", 512, 7, 7, 512, 3, 1, 1),
    ("proj_64_128_s2", 64, 56, 56, 128, 1, 2, 0),
    ("proj_128_256_s2", 128, 28, 28, 256, 1, 2, 0),
    ("proj_256_512_s2", 256, 14, 14, 512, 1, 2, 0),
    ("r50_64_256_56", 64, 56, 56, 256, 1, 1, 0),
    ("r50_256_64_56", 256, 56, 56, 64, 1, 1, 0),
]
SWEEP_GEMMS = [(64, 1000, 512), (4096, 4096, 4096), (8192, 3072, 768), (25088, 768, 3072)]


def sweep_conv(name: str, batch: int = 32):
    """One config-1 Conv as a graph with N(0,1) input and N(0,1)/sqrt(fan_in) weights."""
    spec = {s[0]: s for s in SWEEP_CONVS}[name]
    _, c, h, w, m, k, s, p = spec
    b = _Builder("sweep")
    g = b.g
    x = g.add_input("x", [batch, c, h, w])
    wt = synth.normal((m, c, k, k), 1.0 / math.sqrt(c * k * k), b.seed(name + ".w"))
    bi = synth.normal((m,), 1.0, b.seed(name + ".b"))
    y = g.op("Conv", [x, g.const("w", wt), g.const("b", bi)], name=name, kernel_shape=[k, k], strides=[s, s],
             pads=[p] * 4)
    g.add_output(y, None, FLOAT)
    feed = {"x": synth.normal((batch, c, h, w), 1.0, b.seed(name + ".x"))}
    return g, feed


def sweep_gemm(m: int, n: int, k: int):
    """One config-1 Gemm (runtime A and B operands, as in the sweep)."""
    g = Graph(name="gemm", opset=13)
    g.add_input("a", [m, k])
    g.add_input("b", [k, n])
    y = g.op("Gemm", ["a", "b"], name=f"gemm_{m}x{n}x{k}")
    g.add_output(y, None, FLOAT)
    seed = synth.seed_of("sweep", f"gemm{m}x{n}x{k}")
    feed = {"a": synth.normal((m, k), 1.0, seed), "b": synth.normal((k, n), 1.0 / math.sqrt(k), seed ^ 1)}
    return g, feed


def _conv_out(n: int, k: int, s: int, d: int, p0: int, p1: int) -> int:
    return (n + p0 + p1 - d * (k - 1) - 1) // s + 1


def conv_chain(batch: int, cin: int, h: int, w: int, c: int, m: int, kernel=(3, 3), strides=(1, 1),
               pads=(1, 1, 1, 1), dilations=(1, 1), residual: bool = False, pool: bool = False,
               gap: bool = False, tag: str = "chain"):
    """A small Conv trunk around one Conv of the given geometry.

    input [N,cin,H,W] -> Conv 1x1 (cin->c) + Relu [-> MaxPool 3x3/2 pad 1]
    -> Conv(kernel, strides, pads, dilations; c->m) [+ 1x1 strided skip] + Relu
    -> Conv 1x1 (m->16) [-> GlobalAveragePool] -> output.
    Inside the engine the middle Conv reads channels-last when c % 4 == 0
    (the first Conv writes it that way). Returns
    (graph, feed).
    """
    b = _Builder(tag)
    g = b.g
    x = g.add_input("x", [batch, cin, h, w])

    def conv(src, ci, co, k, s, p, d, name):
        fan_in = ci * k[0] * k[1]
        wt = synth.normal((co, ci, k[0], k[1]), math.sqrt(2.0 / fan_in), b.seed(name + ".w"))
        bi = synth.normal((co,), 0.1, b.seed(name + ".b"))
        return g.op("Conv", [src, g.const(name + ".w", wt), g.const(name + ".b", bi)], name=name,
                    kernel_shape=list(k), strides=list(s), pads=list(p), dilations=list(d))

    t = g.op("Relu", [conv(x, cin, c, (1, 1), (1, 1), (0, 0, 0, 0), (1, 1), "head")], name="head_relu")
    if pool:
        t = g.op("MaxPool", [t], name="pool", kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])
        h, w = _conv_out(h, 3, 2, 1, 1, 1), _conv_out(w, 3, 2, 1, 1, 1)
    y = conv(t, c, m, kernel, strides, pads, dilations, "mid")
    oh = _conv_out(h, kernel[0], strides[0], dilations[0], pads[0], pads[2])
    ow = _conv_out(w, kernel[1], strides[1], dilations[1], pads[1], pads[3])
    if residual:
        sh, sw = _conv_out(h, 1, strides[0], 1, 0, 0), _conv_out(w, 1, strides[1], 1, 0, 0)
        if (sh, sw) != (oh, ow):
            raise ValueError("residual needs a skip of the same extent")
        skip = conv(t, c, m, (1, 1), strides, (0, 0, 0, 0), (1, 1), "skip")
        y = g.op("Add", [y, skip], name="add")
    y = g.op("Relu", [y], name="mid_relu")
    y = conv(y, m, 16, (1, 1), (1, 1), (0, 0, 0, 0), (1, 1), "tail")
    if gap:
        y = g.op("GlobalAveragePool", [y], name="gap")
    g.add_output(y, None, FLOAT)
    feed = {"x": synth.normal(tuple(g.inputs[0][1]), 1.0, b.seed("x"))}
    return g, feed
