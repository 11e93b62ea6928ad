"""Shared test helpers: single-op graphs from the known-answer tables."""

import numpy as np

from nert_b200.onnx_io import FLOAT, INT64, Graph

NP = {"f32": np.float32, "i64": np.int64}
CODE = {"f32": FLOAT, "i64": INT64}


def case2_graph(case):
    """(graph, feeds, expected) for one CASES2 entry: constant operands become
    initializers, the others graph inputs."""
    cite, op, attrs, ins, outs, atol, opset = case
    g = Graph(name="case", opset=opset)
    names, feeds = [], {}
    for i, item in enumerate(ins):
        vals, dims, dt = item[:3]
        const = len(item) > 3 and item[3]
        arr = np.array(vals, dtype=NP[dt]).reshape(dims)
        if const:
            names.append(g.const(f"c{i}", arr))
        else:
            names.append(g.add_input(f"in{i}", list(dims), CODE[dt]))
            feeds[f"in{i}"] = arr
    produced = g.op(op, names, n_out=len(outs), name="node", **attrs)
    produced = produced if isinstance(produced, list) else [produced]
    expected = {}
    for name, (vals, dims, dt) in zip(produced, outs):
        g.add_output(name, list(dims), CODE[dt])
        expected[name] = np.array(vals, dtype=NP[dt]).reshape(dims)
    return g, feeds, expected


def check_outputs(got: dict, expected: dict, atol: float, cite: str):
    for name, want in expected.items():
        have = np.asarray(got[name])
        assert have.shape == want.shape, (cite, name, have.shape, want.shape)
        if want.dtype == np.int64 or atol == 0:
            np.testing.assert_array_equal(have, want, err_msg=cite)
        else:
            np.testing.assert_allclose(have, want, atol=atol, rtol=0, err_msg=cite)
