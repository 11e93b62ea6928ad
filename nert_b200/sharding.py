"""Batch sharding over several GPUs.

* ``shard_plan(batch, n)`` — the contiguous slices (offset, count) of a batch
  over n GPUs, computed by the library (``nb2_shard_plan``), so the in-process
  runner and the one-process-per-GPU launch split a batch the same way.
* ``ShardedModel`` — one graph run over several GPUs from ONE process: a plan
  per GPU for its slice, one native host thread and stream per shard,
  scatter from / gather into the caller's host arrays (``nb2_sharded_*``).
* ``rank_slice`` / ``gather_rows`` — the same split for a job launched as one
  process per GPU (torchrun): each rank takes its slice of the global batch,
  and the slices are gathered in rank order over ``torch.distributed``.

Every op on the path is per image once BatchNormalization is folded, so no
data crosses between GPUs while a batch runs; there is no collective on the
data path.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import check, lib
from .model import _NP, NO_FUSION, NO_GRAPH, NCHW_ONLY, _dims_args, _onnx_bytes

_i64p = ctypes.POINTER(ctypes.c_int64)
_EXTRA = {
    "nb2_shard_plan": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int, _i64p, _i64p]),
    "nb2_sharded_create": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_char_p), _i64p, ctypes.POINTER(ctypes.c_int),
                                          ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_void_p)]),
    "nb2_sharded_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "nb2_sharded_num_io": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int),
                                          ctypes.POINTER(ctypes.c_int)]),
    "nb2_sharded_io": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                      ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), _i64p]),
    "nb2_sharded_shard": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int), _i64p,
                                         _i64p]),
    "nb2_sharded_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                       ctypes.POINTER(ctypes.c_void_p)]),
}
_lib._SIGS.update(_EXTRA)
if _lib._lib is not None:
    for _n, (_r, _a) in _EXTRA.items():
        getattr(_lib._lib, _n).restype = _r
        getattr(_lib._lib, _n).argtypes = _a


def shard_plan(batch: int, n: int) -> list[tuple[int, int]]:
    """[(offset, count)] of each of n shards (the first batch % n take one more)."""
    offs = (ctypes.c_int64 * n)()
    counts = (ctypes.c_int64 * n)()
    check(lib().nb2_shard_plan(batch, n, offs, counts))
    return [(offs[i], counts[i]) for i in range(n)]


def rank_slice(batch: int, rank: int, world: int) -> slice:
    """This rank's slice of a global batch (one process per GPU)."""
    off, cnt = shard_plan(batch, world)[rank]
    return slice(off, off + cnt)


def gather_rows(local: np.ndarray, batch: int, dist) -> np.ndarray | None:
    """Concatenate every rank's slice along axis 0 in rank order (on every
    rank); ``dist`` is an initialised ``torch.distributed``. The slices may be
    ragged (``shard_plan``), so each is padded to the largest before the
    all-gather and trimmed after."""
    import torch

    world = dist.get_world_size()
    plan = shard_plan(batch, world)
    widest = max(c for _, c in plan)
    pad = np.zeros((widest,) + local.shape[1:], local.dtype)
    pad[:local.shape[0]] = local
    t = torch.from_numpy(pad)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return np.concatenate([p.numpy()[:c] for p, (_, c) in zip(parts, plan)], axis=0)


class ShardedModel:
    """One graph batch-sharded over GPUs ``devices`` (a list of ordinals; an
    ordinal may repeat, e.g. two shards on one GPU)."""

    def __init__(self, graph, input_dims: dict, devices, fuse: bool = True, cuda_graph: bool = True,
                 channels_last: bool = True):
        data = _onnx_bytes(graph)
        n, c_names, c_dims, c_ranks = _dims_args(input_dims)
        devs = (ctypes.c_int * len(devices))(*devices)
        flags = ((0 if fuse else NO_FUSION) | (0 if cuda_graph else NO_GRAPH) |
                 (0 if channels_last else NCHW_ONLY))
        h = ctypes.c_void_p()
        check(lib().nb2_sharded_create(data, len(data), n, c_names, c_dims, c_ranks, devs, len(devices), flags,
                                       ctypes.byref(h)))
        self._h = h.value
        ni, no = ctypes.c_int(), ctypes.c_int()
        check(lib().nb2_sharded_num_io(self._h, ctypes.byref(ni), ctypes.byref(no)))
        self.inputs = [self._io(0, i) for i in range(ni.value)]
        self.outputs = [self._io(1, i) for i in range(no.value)]
        self.shards = []
        for i in range(len(devices)):
            o, off, cnt = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
            check(lib().nb2_sharded_shard(self._h, i, ctypes.byref(o), ctypes.byref(off), ctypes.byref(cnt)))
            self.shards.append({"device": o.value, "offset": off.value, "count": cnt.value})

    def _io(self, is_out, i):
        name, dt, rank = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 8)()
        check(lib().nb2_sharded_io(self._h, is_out, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(rank),
                                   dims))
        return {"name": name.value.decode(), "dtype": _NP[dt.value],
                "shape": tuple(dims[d] for d in range(rank.value))}

    def run(self, inputs: dict) -> dict:
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
        check(lib().nb2_sharded_run(self._h, c_in, c_out))

    def close(self):
        if getattr(self, "_h", None):
            lib().nb2_sharded_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
