"""ctypes binding of ``include/nert_b200.h`` (libnert_b200.so).

There is no fallback: if the native library is missing or fails to load,
every entry point raises. Build it with ``python nert_b200/build.py`` (or
``__graft_entry__.build()``).
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libnert_b200.so")
DEVICE_LIB_PATH = os.path.join(HERE, "lib", "libnert_b200_device.so")

OK, ERR_INVALID, ERR_CUDA, ERR_DEVICE, ERR_UNSUPPORTED, ERR_NOMEM = 0, -1, -2, -3, -4, -5
PREC_3XTF32, PREC_1XTF32 = 0, 1
ACT_NONE, ACT_RELU, ACT_SILU, ACT_SIGMOID = 0, 1, 2, 3
F32, I64, BOOL = 0, 1, 2

c_i64p = ctypes.POINTER(ctypes.c_int64)
vp = ctypes.c_void_p


class NB2Error(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"nert_b200 error {status}: {msg}")
        self.status = status


class ConvGeom(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "n", "c", "h", "w", "m", "kh", "kw", "oh", "ow", "stride_h", "stride_w",
        "pad_top", "pad_left", "pad_bottom", "pad_right", "dil_h", "dil_w", "group")]


class ConvTGeom(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "n", "c", "h", "w", "m", "kh", "kw", "oh", "ow", "stride_h", "stride_w", "pad_top", "pad_left",
        "pad_bottom", "pad_right", "dil_h", "dil_w", "out_pad_h", "out_pad_w", "group")]


# name -> (restype, argtypes)
_SIGS = {
    "nb2_last_error": (ctypes.c_char_p, []),
    "nb2_device_open": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(vp)]),
    "nb2_device_ordinal": (ctypes.c_int, [vp]),
    "nb2_device_stream": (vp, [vp]),
    "nb2_device_set_precision": (ctypes.c_int, [vp, ctypes.c_int]),
    "nb2_device_get_precision": (ctypes.c_int, [vp]),
    "nb2_device_synchronize": (ctypes.c_int, [vp]),
    "nb2_device_set_wait_bound": (ctypes.c_int, [vp, ctypes.c_int64]),
    "nb2_device_get_wait_bound": (ctypes.c_int64, [vp]),
    "nb2_device_last_contraction": (ctypes.c_int, [vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                                   ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                                   c_i64p]),
    "nb2_pointer_on_device": (ctypes.c_int, [vp]),
    "nb2_device_malloc": (ctypes.c_int, [vp, ctypes.c_int64, ctypes.POINTER(vp)]),
    "nb2_device_free": (ctypes.c_int, [vp, vp]),
    "nb2_memcpy_h2d": (ctypes.c_int, [vp, vp, vp, ctypes.c_int64]),
    "nb2_memcpy_d2h": (ctypes.c_int, [vp, vp, vp, ctypes.c_int64]),
    "nb2_memcpy_d2d": (ctypes.c_int, [vp, vp, vp, ctypes.c_int64]),
    "nb2_conv2d": (ctypes.c_int, [vp, ctypes.POINTER(ConvGeom), vp, vp, vp, vp, ctypes.c_int, vp]),
    "nb2_conv2d_noalloc": (ctypes.c_int, [vp, ctypes.POINTER(ConvGeom), vp, vp, vp, vp, ctypes.c_int, vp]),
    "nb2_conv2d_noalloc_capacity": (ctypes.c_int64, []),
    "nb2_conv2d_packed_size": (ctypes.c_int, [ctypes.POINTER(ConvGeom), c_i64p]),
    "nb2_conv2d_pack": (ctypes.c_int, [vp, ctypes.POINTER(ConvGeom), vp, vp]),
    "nb2_conv2d_run_packed": (ctypes.c_int, [vp, ctypes.POINTER(ConvGeom), vp, vp, vp, vp, ctypes.c_int, vp]),
    "nb2_conv_transpose2d": (ctypes.c_int, [vp, ctypes.POINTER(ConvTGeom), vp, vp, vp, vp]),
    "nb2_gemm": (ctypes.c_int, [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int]),
    "nb2_gemm_packed_size": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, c_i64p]),
    "nb2_gemm_pack": (ctypes.c_int, [vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, vp]),
    "nb2_gemm_run_packed": (ctypes.c_int, [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                           ctypes.c_int]),
    "nb2_matmul": (ctypes.c_int, [vp, vp, c_i64p, ctypes.c_int, vp, c_i64p, ctypes.c_int, vp]),
    "nb2_unary": (ctypes.c_int, [vp, ctypes.c_int, vp, vp, ctypes.c_int64]),
    "nb2_binary": (ctypes.c_int, [vp, ctypes.c_int, ctypes.c_int, vp, c_i64p, ctypes.c_int, vp, c_i64p, ctypes.c_int,
                                  vp, c_i64p, ctypes.c_int]),
    "nb2_maxpool2d": (ctypes.c_int, [vp, vp, c_i64p, vp, c_i64p, c_i64p, c_i64p, c_i64p, c_i64p]),
    "nb2_avgpool2d": (ctypes.c_int, [vp, vp, c_i64p, vp, c_i64p, c_i64p, c_i64p, c_i64p, ctypes.c_int]),
    "nb2_sppf": (ctypes.c_int, [vp, vp, c_i64p, vp, ctypes.c_int64, ctypes.c_int64]),
    "nb2_attention": (ctypes.c_int, [vp, vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int64, c_i64p, c_i64p, c_i64p, c_i64p, ctypes.c_int, ctypes.c_float]),
    "nb2_row_mean": (ctypes.c_int, [vp, vp, ctypes.c_int64, ctypes.c_int64, vp]),
    "nb2_softmax": (ctypes.c_int, [vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]),
    "nb2_layernorm": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_float]),
    "nb2_transpose": (ctypes.c_int, [vp, vp, vp, c_i64p, c_i64p, ctypes.c_int, ctypes.c_int]),
    "nb2_concat_split": (ctypes.c_int, [vp, ctypes.c_int, vp, ctypes.POINTER(vp), c_i64p, ctypes.c_int,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int]),
    "nb2_slice": (ctypes.c_int, [vp, vp, vp, c_i64p, c_i64p, c_i64p, c_i64p, ctypes.c_int, ctypes.c_int]),
    "nb2_gather": (ctypes.c_int, [vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int]),
    "nb2_topk": (ctypes.c_int, [vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]),
    "nb2_resize": (ctypes.c_int, [vp, vp, vp, c_i64p, c_i64p, ctypes.POINTER(ctypes.c_double), ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "nb2_cast": (ctypes.c_int, [vp, vp, ctypes.c_int, vp, ctypes.c_int, ctypes.c_int64]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"native library missing: {LIB_PATH}; run python nert_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int) -> None:
    if status != OK:
        raise NB2Error(status, lib().nb2_last_error().decode())


def i64s(vals) -> ctypes.Array:
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)


def last_contraction(ordinal: int = 0) -> dict:
    """Schedule of the most recent Conv/Gemm/MatMul launch on the GPU."""
    tn, alt, ks, mode = (ctypes.c_int() for _ in range(4))
    tiles = ctypes.c_int64()
    check(lib().nb2_device_last_contraction(device(ordinal), ctypes.byref(tn), ctypes.byref(alt), ctypes.byref(ks),
                                            ctypes.byref(mode), ctypes.byref(tiles)))
    return {"tile_n": tn.value, "two_in_flight": alt.value, "k_slices": ks.value, "a_mode": mode.value,
            "tiles": tiles.value}


def device(ordinal: int = 0) -> int:
    h = vp()
    check(lib().nb2_device_open(ordinal, ctypes.byref(h)))
    return h.value
