"""Run one row or one model repeatedly, for external profilers (ncu).

    python -m nert_b200.probe conv N C H W M K STRIDE PAD [REPS]
    python -m nert_b200.probe gemm M N K [REPS]
    python -m nert_b200.probe maxpool N C H W K STRIDE PAD [REPS]
    python -m nert_b200.probe resnet18 BATCH [REPS]
    python -m nert_b200.probe engine_conv N C H W M K STRIDE PAD [REPS]
        (one Conv as an engine graph: C <= 4 takes the 4-channel input path)
    python -m nert_b200.probe chain N C H W M K STRIDE PAD [REPS]
        (engine graph: 1x1 Conv 16->C, the KxK Conv C->M reading and writing
        channels-last, 1x1 Conv M->16; the middle Conv is the second igemm
        launch of each run)

Inputs are seeded synthetic data; each mode prints one line with the
geometry and exits 0 on success.
"""

from __future__ import annotations

import sys

import numpy as np


def main(argv):
    import torch

    from . import ops, synth

    mode = argv[0]
    if mode == "conv":
        n, c, h, w, m, k, s, p = (int(v) for v in argv[1:9])
        reps = int(argv[9]) if len(argv) > 9 else 3
        x = torch.from_numpy(synth.normal((n, c, h, w), 1.0, 1)).cuda()
        wt = torch.from_numpy(synth.normal((m, c, k, k), (2.0 / (c * k * k)) ** 0.5, 2)).cuda()
        b = torch.from_numpy(synth.normal((m,), 0.1, 3)).cuda()
        for _ in range(reps):
            y = ops.conv2d(x, wt, b, [s, s], [p] * 4)
        print("conv", tuple(y.shape))
    elif mode == "gemm":
        m, n, k = (int(v) for v in argv[1:4])
        reps = int(argv[4]) if len(argv) > 4 else 3
        a = torch.from_numpy(synth.normal((m, k), 1.0, 1)).cuda()
        b = torch.from_numpy(synth.normal((k, n), 1.0 / np.sqrt(k), 2)).cuda()
        for _ in range(reps):
            y = ops.gemm(a, b)
        print("gemm", tuple(y.shape))
    elif mode == "maxpool":
        n, c, h, w, k, s, p = (int(v) for v in argv[1:8])
        reps = int(argv[8]) if len(argv) > 8 else 3
        x = torch.from_numpy(synth.normal((n, c, h, w), 1.0, 1)).cuda()
        for _ in range(reps):
            y = ops.maxpool2d(x, [k, k], [s, s], [p] * 4)
        print("maxpool", tuple(y.shape))
    elif mode == "resnet18":
        from . import configs
        from .model import Model

        b = int(argv[1])
        reps = int(argv[2]) if len(argv) > 2 else 3
        m = Model(configs.resnet18(b), {"input": [b, 3, 224, 224]})
        x = configs.resnet_input(b)
        for _ in range(reps):
            out = m.run({"input": x})
        print("resnet18", out["fc_out"].shape)
    elif mode == "engine_conv":
        from .model import Model
        from .onnx_io import FLOAT, Graph

        n, c, h, w, m_, k, s, p = (int(v) for v in argv[1:9])
        reps = int(argv[9]) if len(argv) > 9 else 3
        g = Graph(opset=13)
        x = g.add_input("x", [n, c, h, w])
        wt = g.const("w", synth.normal((m_, c, k, k), (2.0 / (c * k * k)) ** 0.5, 2))
        g.add_output(g.op("Conv", [x, wt], name="conv", kernel_shape=[k, k], strides=[s, s], pads=[p] * 4),
                     None, FLOAT)
        m = Model(g, {"x": [n, c, h, w]})
        feed = {"x": synth.uniform((n, c, h, w), -1.0, 1.0, 1)}
        for _ in range(reps):
            out = m.run(feed)
        m.close()
        print("engine_conv", next(iter(out.values())).shape)
    elif mode == "chain":
        from . import configs
        from .model import Model

        n, c, h, w, m_, k, s, p = (int(v) for v in argv[1:9])
        reps = int(argv[9]) if len(argv) > 9 else 3
        g, feed = configs.conv_chain(n, 16, h, w, c, m_, kernel=(k, k), strides=(s, s), pads=(p,) * 4,
                                     tag="probe")
        m = Model(g, {"x": list(feed["x"].shape)})
        for _ in range(reps):
            out = m.run(feed)
        m.close()
        print("chain", next(iter(out.values())).shape)
    else:
        raise SystemExit(__doc__)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
