"""TEST INFRASTRUCTURE ONLY: ctypes access to the reference NERT library.

``oracle/_ref/libnert_ref.so`` is the reference's own CPU library, compiled
from its sources by ``oracle/Makefile`` (see ``oracle/ref_capi.cpp`` for the C
ABI). Only the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg use this module, and only as the checker / the timed reference.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libnert_ref.so")
# the same library with the reference's CUDA device (cuDNN/cuBLAS rows), the
# GPU baseline; built only where nvcc and cuDNN are present
CUDA_LIB_PATH = os.path.join(HERE, "_ref", "libnert_ref_cuda.so")
# the reference checkout: NERT_REFERENCE, else a sibling of this repository
REFERENCE_SRC = os.environ.get("NERT_REFERENCE",
                               os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

_libs: dict = {}
_NP = {0: np.float32, 1: np.int64, 2: np.bool_}
_CODE = {np.dtype(np.float32): 0, np.dtype(np.int64): 1, np.dtype(np.bool_): 2}


def build(quiet: bool = True) -> bool:
    """Compile oracle/_ref from the reference sources when they are present
    (the CPU library, and the CUDA-device library where nvcc and cuDNN are)."""
    if not os.path.isdir(os.path.join(REFERENCE_SRC, "src")):
        return os.path.exists(LIB_PATH)
    targets = ["all"]
    if os.path.exists(os.path.join(HERE, "..", "nert_b200", "lib", "libnert_b200_device.so")):
        targets.append("bench_runtime")  # the reference's runtime bench harness on the B200 handle
    out = subprocess.run(["make", "-C", HERE, "-j8", f"REF={REFERENCE_SRC}"] + targets, capture_output=True,
                         text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout[-2000:] + out.stderr[-2000:])
    return True


def available(cuda: bool = False) -> bool:
    return os.path.exists(CUDA_LIB_PATH if cuda else LIB_PATH)


def lib(cuda: bool = False):
    """The reference library: CPU only, or (cuda=True) with its CudaDevice."""
    key = "cuda" if cuda else "cpu"
    if key not in _libs:
        path = CUDA_LIB_PATH if cuda else LIB_PATH
        if not os.path.exists(path):
            raise RuntimeError(f"reference oracle library missing: {path} (run make -C oracle)")
        L = ctypes.CDLL(path)
        L.nref_open.restype = ctypes.c_void_p
        L.nref_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
        L.nref_last_error.restype = ctypes.c_char_p
        L.nref_last_error.argtypes = [ctypes.c_void_p]
        L.nref_close.argtypes = [ctypes.c_void_p]
        L.nref_open_folded.restype = ctypes.c_void_p
        L.nref_open_folded.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                       ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int), ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
        L.nref_run.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                               ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_void_p),
                               ctypes.POINTER(ctypes.c_int64)]
        L.nref_last_run_ms.restype = ctypes.c_double
        L.nref_last_run_ms.argtypes = [ctypes.c_void_p]
        L.nref_num_outputs.argtypes = [ctypes.c_void_p]
        L.nref_output_name.restype = ctypes.c_char_p
        L.nref_output_name.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.nref_output_info.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                       ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64)]
        L.nref_output_copy.restype = ctypes.c_int64
        L.nref_output_copy.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
        L.nref_arena_bytes.restype = ctypes.c_int64
        L.nref_arena_bytes.argtypes = [ctypes.c_void_p]
        if cuda:
            L.nref_cuda_device.restype = ctypes.c_void_p
            L.nref_cuda_device.argtypes = []
        _libs[key] = L
    return _libs[key]


class RefModel:
    """The reference's nert::Model over an ONNX file, on CpuDevice or on any
    other ``const nert::Device*`` handed in as an integer address."""

    def __init__(self, onnx_path: str, input_dims: dict[str, list[int]], device: int | None = None,
                 cuda: bool = False, fold_device: int | None = None, fold: bool = False):
        """cuda=True: the library built with the reference's CudaDevice, and
        (when `device` is None) that device."""
        self._L = L = lib(cuda)
        if cuda and device is None:
            device = L.nref_cuda_device()
            if not device:
                raise RuntimeError("reference CudaDevice unavailable: " + L.nref_last_error(None).decode())
        names = list(input_dims)
        c_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        flat = [d for n in names for d in input_dims[n]]
        c_dims = (ctypes.c_int64 * max(1, len(flat)))(*flat)
        c_ranks = (ctypes.c_int * len(names))(*[len(input_dims[n]) for n in names])
        self.folded = 0
        if fold:
            # nert::FoldConstants with `fold_device`'s rows first (CpuDevice when None)
            n_fold = ctypes.c_int(0)
            self._h = L.nref_open_folded(onnx_path.encode(), len(names), c_names, c_dims, c_ranks, fold_device,
                                         device, ctypes.byref(n_fold))
            self.folded = n_fold.value
        else:
            self._h = L.nref_open(onnx_path.encode(), len(names), c_names, c_dims, c_ranks, device)
        if not self._h:
            raise RuntimeError("reference load failed: " + L.nref_last_error(None).decode())
        self.last_ms = 0.0

    def run(self, inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
        L = self._L
        names = list(inputs)
        arrs = [np.ascontiguousarray(inputs[n]) for n in names]
        c_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        c_dt = (ctypes.c_int * len(names))(*[_CODE[a.dtype] for a in arrs])
        c_data = (ctypes.c_void_p * len(names))(*[a.ctypes.data for a in arrs])
        c_nb = (ctypes.c_int64 * len(names))(*[a.nbytes for a in arrs])
        if L.nref_run(self._h, len(names), c_names, c_dt, c_data, c_nb) != 0:
            raise RuntimeError("reference run failed: " + L.nref_last_error(self._h).decode())
        self.last_ms = L.nref_last_run_ms(self._h)
        out = {}
        for i in range(L.nref_num_outputs(self._h)):
            dt, rank = ctypes.c_int(), ctypes.c_int()
            dims = (ctypes.c_int64 * 8)()
            if L.nref_output_info(self._h, i, ctypes.byref(dt), ctypes.byref(rank), dims) != 0:
                raise RuntimeError(L.nref_last_error(self._h).decode())
            shape = [dims[d] for d in range(rank.value)]
            arr = np.empty(shape, dtype=_NP[dt.value])
            L.nref_output_copy(self._h, i, arr.ctypes.data, arr.nbytes)
            out[L.nref_output_name(self._h, i).decode()] = arr
        return out

    def arena_bytes(self) -> int:
        return self._L.nref_arena_bytes(self._h)

    def close(self):
        if self._h:
            self._L.nref_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def run_graph(graph, inputs: dict[str, np.ndarray], device: int | None = None,
              cuda: bool = False) -> dict[str, np.ndarray]:
    """Write ``graph`` (an nert_b200.onnx_io.Graph) to a temp ONNX file and run
    it once through the reference loader + executor (cuda=True: on the
    reference's own CudaDevice)."""
    from nert_b200 import onnx_io

    with tempfile.TemporaryDirectory() as d:
        path = onnx_io.save(graph, os.path.join(d, "model.onnx"))
        m = RefModel(path, {k: list(v.shape) for k, v in inputs.items()}, device, cuda)
        try:
            return m.run(inputs)
        finally:
            m.close()
