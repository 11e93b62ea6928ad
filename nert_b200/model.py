"""Python face of the B200 engine, mirroring NERT's host API.

    graph = load_graph_from_file("model.onnx")        # nert::LoadGraphFromFile
    model = Model(graph, {"input": [64, 3, 224, 224]}, device=0)   # nert::Model
    out = model.run({"input": x})                      # Model::Run / RunTyped

Everything runs in libnert_b200.so (C++ host engine + sm_100a kernels); this
module only marshals numpy arrays across the C ABI.
"""

from __future__ import annotations

import ctypes
import json

import numpy as np

from . import _lib, onnx_io
from ._lib import check, lib

NO_FUSION, NO_GRAPH, NCHW_ONLY, NO_ATTENTION = 1, 2, 4, 8
_NP = {0: np.float32, 1: np.int64, 2: np.bool_}

_EXTRA = {
    "nb2_model_create": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_int64),
                                        ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_void_p)]),
    "nb2_model_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "nb2_model_num_io": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "nb2_model_io": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                    ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                    ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_void_p)]),
    "nb2_model_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                     ctypes.POINTER(ctypes.c_void_p)]),
    "nb2_model_run_async": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                           ctypes.POINTER(ctypes.c_void_p)]),
    "nb2_model_launch": (ctypes.c_int, [ctypes.c_void_p]),
    "nb2_model_synchronize": (ctypes.c_int, [ctypes.c_void_p]),
    "nb2_model_stats": (ctypes.c_int, [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_int64)] * 5),
    "nb2_model_profile": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                         ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int)]),
    "nb2_model_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "nb2_graph_analyze": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                         ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_int64),
                                         ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_char_p, ctypes.c_int64,
                                         ctypes.POINTER(ctypes.c_int64)]),
    "nb2_host_alloc": (ctypes.c_int, [ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p)]),
    "nb2_host_free": (ctypes.c_int, [ctypes.c_void_p]),
}
_lib._SIGS.update(_EXTRA)
if _lib._lib is not None:  # already loaded: bind the extra signatures too
    for _n, (_r, _a) in _EXTRA.items():
        getattr(_lib._lib, _n).restype = _r
        getattr(_lib._lib, _n).argtypes = _a


def load_graph_from_file(path: str) -> onnx_io.Graph:
    """Read an ONNX file (the counterpart of nert::LoadGraphFromFile)."""
    return onnx_io.load(path)


def _onnx_bytes(graph) -> bytes:
    if isinstance(graph, (bytes, bytearray)):
        return bytes(graph)
    if isinstance(graph, str):
        with open(graph, "rb") as f:
            return f.read()
    return onnx_io.to_onnx_bytes(graph)


def _dims_args(input_dims: dict):
    names = list(input_dims)
    c_names = (ctypes.c_char_p * max(1, len(names)))(*[n.encode() for n in names])
    flat = [int(d) for n in names for d in input_dims[n]]
    c_dims = (ctypes.c_int64 * max(1, len(flat)))(*flat)
    c_ranks = (ctypes.c_int * max(1, len(names)))(*[len(input_dims[n]) for n in names])
    return len(names), c_names, c_dims, c_ranks


def analyze(graph, input_dims: dict, flags: int = 0) -> dict:
    """Shapes, fused rows and the arena plan of a graph (host only, no GPU)."""
    data = _onnx_bytes(graph)
    n, c_names, c_dims, c_ranks = _dims_args(input_dims)
    need = ctypes.c_int64()
    check(lib().nb2_graph_analyze(data, len(data), n, c_names, c_dims, c_ranks, flags, None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    check(lib().nb2_graph_analyze(data, len(data), n, c_names, c_dims, c_ranks, flags, buf, need.value,
                                  ctypes.byref(need)))
    return json.loads(buf.value.decode())


class HostBuffer:
    """Pinned host memory exposed as a numpy array."""

    def __init__(self, shape, dtype=np.float32):
        self.nbytes = int(np.prod(shape)) * np.dtype(dtype).itemsize
        p = ctypes.c_void_p()
        check(lib().nb2_host_alloc(self.nbytes, ctypes.byref(p)))
        self.ptr = p.value
        buf = (ctypes.c_char * self.nbytes).from_address(self.ptr)
        self.array = np.frombuffer(buf, dtype=dtype).reshape(shape)

    def free(self):
        if self.ptr:
            self.array = None
            lib().nb2_host_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Model:
    """One graph on one GPU for one input shape (nert::Model on B200)."""

    def __init__(self, graph, input_dims: dict, device: int = 0, fuse: bool = True, cuda_graph: bool = True,
                 channels_last: bool = True, fused_attention: bool = True):
        """channels_last=False keeps every activation NCHW (no NHWC conv trunk);
        fused_attention=False runs attention chains as separate rows."""
        data = _onnx_bytes(graph)
        n, c_names, c_dims, c_ranks = _dims_args(input_dims)
        flags = ((0 if fuse else NO_FUSION) | (0 if cuda_graph else NO_GRAPH) |
                 (0 if channels_last else NCHW_ONLY) | (0 if fused_attention else NO_ATTENTION))
        h = ctypes.c_void_p()
        check(lib().nb2_model_create(data, len(data), n, c_names, c_dims, c_ranks, device, flags, ctypes.byref(h)))
        self._h = h.value
        ni, no = ctypes.c_int(), ctypes.c_int()
        check(lib().nb2_model_num_io(self._h, ctypes.byref(ni), ctypes.byref(no)))
        self.inputs = [self._io(0, i) for i in range(ni.value)]
        self.outputs = [self._io(1, i) for i in range(no.value)]

    def _io(self, is_out, i):
        name, dt, rank = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 8)()
        ptr = ctypes.c_void_p()
        check(lib().nb2_model_io(self._h, is_out, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(rank), dims,
                                 ctypes.byref(ptr)))
        return {"name": name.value.decode(), "dtype": _NP[dt.value], "shape": tuple(dims[d] for d in range(rank.value)),
                "device_ptr": ptr.value}

    def run(self, inputs: dict) -> dict:
        """End-to-end run from host arrays (Model::Run)."""
        arrs = []
        for io in self.inputs:
            a = np.ascontiguousarray(inputs[io["name"]], dtype=io["dtype"])
            if a.shape != io["shape"]:
                raise ValueError(f"input '{io['name']}' has shape {a.shape}, expected {io['shape']}")
            arrs.append(a)
        outs = [np.empty(io["shape"], dtype=io["dtype"]) for io in self.outputs]
        self.run_into([a.ctypes.data for a in arrs], [o.ctypes.data for o in outs])
        return {io["name"]: o for io, o in zip(self.outputs, outs)}

    def run_into(self, in_ptrs, out_ptrs):
        c_in = (ctypes.c_void_p * max(1, len(in_ptrs)))(*in_ptrs)
        c_out = (ctypes.c_void_p * max(1, len(out_ptrs)))(*out_ptrs)
        check(lib().nb2_model_run(self._h, c_in, c_out))

    def run_async(self, in_ptrs, out_ptrs):
        """Queue H2D copies, the run and D2H copies; pair with synchronize()."""
        c_in = (ctypes.c_void_p * max(1, len(in_ptrs)))(*in_ptrs)
        c_out = (ctypes.c_void_p * max(1, len(out_ptrs)))(*out_ptrs)
        check(lib().nb2_model_run_async(self._h, c_in, c_out))

    def launch(self):
        check(lib().nb2_model_launch(self._h))

    def synchronize(self):
        check(lib().nb2_model_synchronize(self._h))

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(lib().nb2_model_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def stats(self) -> dict:
        v = [ctypes.c_int64() for _ in range(5)]
        check(lib().nb2_model_stats(self._h, *[ctypes.byref(x) for x in v]))
        return dict(zip(["kernels_per_run", "arena_bytes", "weight_bytes", "fused_groups", "exec_nodes"],
                        [x.value for x in v]))

    def profile(self, max_steps: int = 4096) -> list[tuple[str, float]]:
        L = 96
        labels = ctypes.create_string_buffer(max_steps * L)
        ms = (ctypes.c_float * max_steps)()
        cnt = ctypes.c_int()
        check(lib().nb2_model_profile(self._h, max_steps, labels, L, ms, ctypes.byref(cnt)))
        raw = labels.raw
        return [(raw[i * L:(i + 1) * L].split(b"\0", 1)[0].decode(), ms[i]) for i in range(min(cnt.value, max_steps))]

    def close(self):
        if getattr(self, "_h", None):
            lib().nb2_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
