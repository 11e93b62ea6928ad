"""A small ONNX graph description with a protobuf writer and reader.

The ``onnx`` package is not a dependency: models are written and read with a
hand-written protobuf wire codec over the subset of ``onnx.proto`` that NERT's
loader reads (ModelProto, GraphProto, NodeProto, AttributeProto, TensorProto,
ValueInfoProto; field numbers as in the public ONNX schema and as decoded by
the reference loader, ``src/model_loader.cpp:41-97``).

The same ``Graph`` object feeds three consumers, so every one of them sees the
same graph and the same weights:

* the B200 engine (``nb2_model_load_onnx``), which parses the bytes in C++;
* the reference's own loader (``nert::LoadGraphFromFile``) in the oracle;
* the numpy restatement in ``oracle/np_ref.py``.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

# TensorProto.DataType values.
FLOAT, INT64, BOOL = 1, 7, 9
_NP_OF = {FLOAT: np.float32, INT64: np.int64, BOOL: np.bool_}
_CODE_OF = {np.dtype(np.float32): FLOAT, np.dtype(np.int64): INT64, np.dtype(np.bool_): BOOL}

# AttributeProto.AttributeType values.
A_FLOAT, A_INT, A_STRING, A_TENSOR, A_FLOATS, A_INTS = 1, 2, 3, 4, 6, 7


@dataclass
class Node:
    op_type: str
    inputs: list[str]
    outputs: list[str]
    name: str = ""
    attrs: dict[str, Any] = field(default_factory=dict)


@dataclass
class Graph:
    name: str = "graph"
    nodes: list[Node] = field(default_factory=list)
    initializers: dict[str, np.ndarray] = field(default_factory=dict)
    inputs: list[tuple[str, list[int], int]] = field(default_factory=list)
    outputs: list[tuple[str, list[int] | None, int]] = field(default_factory=list)
    opset: int = 13

    # ---- builder helpers -------------------------------------------------
    _counter: int = 0

    def fresh(self, stem: str) -> str:
        self._counter += 1
        return f"{stem}_{self._counter}"

    def add_input(self, name: str, dims: list[int], dtype: int = FLOAT) -> str:
        self.inputs.append((name, list(dims), dtype))
        return name

    def add_output(self, name: str, dims: list[int] | None = None, dtype: int = FLOAT) -> None:
        self.outputs.append((name, None if dims is None else list(dims), dtype))

    def const(self, name: str, value: np.ndarray) -> str:
        # np.ascontiguousarray would turn a 0-d scalar into shape (1,)
        self.initializers[name] = np.array(value, order="C", copy=True)
        return name

    def op(self, op_type: str, inputs: list[str], n_out: int = 1, name: str | None = None, **attrs) -> Any:
        name = name or self.fresh(op_type.lower())
        outs = [f"{name}_out{i}" if n_out > 1 else f"{name}_out" for i in range(n_out)]
        self.nodes.append(Node(op_type, list(inputs), outs, name, dict(attrs)))
        return outs if n_out > 1 else outs[0]


# ---- protobuf wire encoding ----------------------------------------------

def _varint(v: int) -> bytes:
    if v < 0:
        v += 1 << 64
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(fieldno: int, wire: int) -> bytes:
    return _varint((fieldno << 3) | wire)


def _ld(fieldno: int, payload: bytes) -> bytes:
    return _key(fieldno, 2) + _varint(len(payload)) + payload


def _vi(fieldno: int, v: int) -> bytes:
    return _key(fieldno, 0) + _varint(v)


def _f32(fieldno: int, v: float) -> bytes:
    return _key(fieldno, 5) + struct.pack("<f", v)


def _tensor(name: str, arr: np.ndarray) -> bytes:
    arr = np.array(arr, order="C", copy=False) if arr.ndim == 0 else np.ascontiguousarray(arr)
    code = _CODE_OF[arr.dtype]
    out = b"".join(_vi(1, int(d)) for d in arr.shape)
    out += _vi(2, code) + _ld(8, name.encode())
    raw = arr.astype(arr.dtype.newbyteorder("<"), copy=False).tobytes()
    return out + _ld(9, raw)


def _attr(name: str, value: Any) -> bytes:
    out = _ld(1, name.encode())
    if isinstance(value, bool):
        value = int(value)
    if isinstance(value, (int, np.integer)):
        return out + _vi(3, int(value)) + _vi(20, A_INT)
    if isinstance(value, (float, np.floating)):
        return out + _f32(2, float(value)) + _vi(20, A_FLOAT)
    if isinstance(value, str):
        return out + _ld(4, value.encode()) + _vi(20, A_STRING)
    if isinstance(value, np.ndarray):
        return out + _ld(5, _tensor("", value)) + _vi(20, A_TENSOR)
    if isinstance(value, (list, tuple)):
        if all(isinstance(v, (int, np.integer)) for v in value):
            return out + b"".join(_vi(8, int(v)) for v in value) + _vi(20, A_INTS)
        return out + b"".join(_f32(7, float(v)) for v in value) + _vi(20, A_FLOATS)
    raise TypeError(f"attribute {name}: unsupported value {value!r}")


def _value_info(name: str, dims: list[int] | None, dtype: int) -> bytes:
    tt = _vi(1, dtype)
    if dims is not None:
        shape = b"".join(_ld(1, _vi(1, int(d))) for d in dims)
        tt += _ld(2, shape)
    return _ld(1, name.encode()) + _ld(2, _ld(1, tt))


def to_onnx_bytes(g: Graph) -> bytes:
    body = b""
    for n in g.nodes:
        nb = b"".join(_ld(1, s.encode()) for s in n.inputs)
        nb += b"".join(_ld(2, s.encode()) for s in n.outputs)
        nb += _ld(3, n.name.encode()) + _ld(4, n.op_type.encode())
        nb += b"".join(_ld(5, _attr(k, v)) for k, v in n.attrs.items())
        body += _ld(1, nb)
    body += _ld(2, g.name.encode())
    for k, v in g.initializers.items():
        body += _ld(5, _tensor(k, v))
    for name, dims, dt in g.inputs:
        body += _ld(11, _value_info(name, dims, dt))
    for name, dims, dt in g.outputs:
        body += _ld(12, _value_info(name, dims, dt))
    model = _vi(1, 8) + _ld(2, b"nert_b200") + _ld(8, _ld(1, b"") + _vi(2, g.opset)) + _ld(7, body)
    return model


def save(g: Graph, path: str) -> str:
    with open(path, "wb") as f:
        f.write(to_onnx_bytes(g))
    return path


# ---- protobuf wire decoding ----------------------------------------------

class _Reader:
    def __init__(self, data: bytes):
        self.d = memoryview(data)
        self.i = 0

    def done(self) -> bool:
        return self.i >= len(self.d)

    def varint(self) -> int:
        shift = v = 0
        while True:
            b = self.d[self.i]
            self.i += 1
            v |= (b & 0x7F) << shift
            if not b & 0x80:
                return v
            shift += 7

    def field(self) -> tuple[int, int]:
        k = self.varint()
        return k >> 3, k & 7

    def value(self, wire: int) -> Any:
        if wire == 0:
            return self.varint()
        if wire == 1:
            v = bytes(self.d[self.i:self.i + 8])
            self.i += 8
            return v
        if wire == 5:
            v = bytes(self.d[self.i:self.i + 4])
            self.i += 4
            return v
        if wire == 2:
            n = self.varint()
            v = bytes(self.d[self.i:self.i + n])
            self.i += n
            return v
        raise ValueError(f"unsupported wire type {wire}")


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _fields(data: bytes):
    r = _Reader(data)
    while not r.done():
        f, w = r.field()
        yield f, w, r.value(w)


def _read_ints(w: int, v: Any) -> list[int]:
    if w == 0:
        return [_signed(v)]
    r = _Reader(v)
    out = []
    while not r.done():
        out.append(_signed(r.varint()))
    return out


def _read_tensor(data: bytes) -> tuple[str, np.ndarray]:
    dims, code, name, raw, floats, ints = [], FLOAT, "", None, [], []
    for f, w, v in _fields(data):
        if f == 1:
            dims += _read_ints(w, v)
        elif f == 2:
            code = v
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = v
        elif f == 4:
            floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if w == 2 else [struct.unpack("<f", v)[0]]
        elif f == 7:
            ints += _read_ints(w, v)
    dt = _NP_OF[code]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=np.dtype(dt).newbyteorder("<")).astype(dt)
    elif code == FLOAT:
        arr = np.array(floats, dtype=np.float32)
    else:
        arr = np.array(ints, dtype=dt)
    return name, arr.reshape(dims)


def _read_value_info(data: bytes) -> tuple[str, list[int] | None, int]:
    name, dims, code = "", None, FLOAT
    for f, _, v in _fields(data):
        if f == 1:
            name = v.decode()
        elif f == 2:
            for f2, _, v2 in _fields(v):
                if f2 == 1:
                    for f3, _, v3 in _fields(v2):
                        if f3 == 1:
                            code = v3
                        elif f3 == 2:
                            dims = []
                            for f4, _, v4 in _fields(v3):
                                if f4 == 1:
                                    d = -1
                                    for f5, _, v5 in _fields(v4):
                                        if f5 == 1:
                                            d = _signed(v5)
                                    dims.append(d)
    return name, dims, code


def from_onnx_bytes(data: bytes) -> Graph:
    g = Graph()
    graph_bytes = b""
    for f, _, v in _fields(data):
        if f == 7:
            graph_bytes = v
        elif f == 8:
            dom, ver = "", 0
            for f2, _, v2 in _fields(v):
                if f2 == 1:
                    dom = v2.decode()
                elif f2 == 2:
                    ver = v2
            if dom in ("", "ai.onnx"):
                g.opset = ver
    for f, w, v in _fields(graph_bytes):
        if f == 1:
            n = Node("", [], [])
            for f2, w2, v2 in _fields(v):
                if f2 == 1:
                    n.inputs.append(v2.decode())
                elif f2 == 2:
                    n.outputs.append(v2.decode())
                elif f2 == 3:
                    n.name = v2.decode()
                elif f2 == 4:
                    n.op_type = v2.decode()
                elif f2 == 5:
                    an, av, at, ints, floats = "", None, 0, [], []
                    for f3, w3, v3 in _fields(v2):
                        if f3 == 1:
                            an = v3.decode()
                        elif f3 == 2:
                            av = struct.unpack("<f", v3)[0]
                        elif f3 == 3:
                            av = _signed(v3)
                        elif f3 == 4:
                            av = v3.decode()
                        elif f3 == 5:
                            av = _read_tensor(v3)[1]
                        elif f3 == 7:
                            floats += (list(struct.unpack(f"<{len(v3) // 4}f", v3)) if w3 == 2
                                       else [struct.unpack("<f", v3)[0]])
                        elif f3 == 8:
                            ints += _read_ints(w3, v3)
                        elif f3 == 20:
                            at = v3
                    if at == A_INTS:
                        av = ints
                    elif at == A_FLOATS:
                        av = floats
                    n.attrs[an] = av
            g.nodes.append(n)
        elif f == 2:
            g.name = v.decode()
        elif f == 5:
            name, arr = _read_tensor(v)
            g.initializers[name] = arr
        elif f == 11:
            name, dims, code = _read_value_info(v)
            if name not in g.initializers:
                g.inputs.append((name, dims or [], code))
        elif f == 12:
            g.outputs.append(_read_value_info(v))
    return g


def load(path: str) -> Graph:
    with open(path, "rb") as f:
        return from_onnx_bytes(f.read())
