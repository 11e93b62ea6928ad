"""Build the B200 layer's native libraries in-tree.

* ``nert_b200/lib/libnert_b200.so`` — every CUDA kernel and the C ABI of
  ``include/nert_b200.h`` plus the C++ engine (``csrc/engine``), compiled for
  sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
* ``nert_b200/lib/libnert_b200_device.so`` — the ``nert::Device`` plug-in
  (``device/b200_device.cpp``), compiled against the NERT public headers when
  they are available (``NERT_INCLUDE``, else the ``include/`` of the reference
  checkout named by ``NERT_REFERENCE`` or lying beside this repository).

Objects are rebuilt only when a source or header is newer than the object.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "lib")
OBJ_DIR = os.path.join(HERE, "lib", "obj")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xcompiler", "-Wall", "-diag-suppress", "177"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall"]

MAIN_LIB = os.path.join(LIB_DIR, "libnert_b200.so")
DEVICE_LIB = os.path.join(LIB_DIR, "libnert_b200_device.so")


def nert_include() -> str | None:
    ref = os.environ.get("NERT_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
    for cand in (os.environ.get("NERT_INCLUDE"), os.path.join(ref, "include")):
        if cand and os.path.exists(os.path.join(cand, "nert", "device.hpp")):
            return cand
    return None


def _newest(paths) -> float:
    return max((os.path.getmtime(p) for p in paths if os.path.exists(p)), default=0.0)


def _headers() -> list[str]:
    return (glob.glob(os.path.join(HERE, "csrc", "**", "*.cuh"), recursive=True)
            + glob.glob(os.path.join(HERE, "csrc", "**", "*.hpp"), recursive=True)
            + [os.path.join(ROOT, "include", "nert_b200.h")])


def _compile(src: str, obj: str, hdr_time: float) -> str | None:
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_time):
        return None
    os.makedirs(os.path.dirname(obj), exist_ok=True)
    inc = ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(HERE, "csrc")]
    if src.endswith(".cu"):
        cmd = [NVCC, *ARCH, *NVCC_FLAGS, *inc, "-c", src, "-o", obj]
    else:
        cmd = ["g++", *CXX_FLAGS, *inc, "-I", os.path.join(CUDA_HOME, "include"), "-c", src, "-o", obj]
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{out.stdout}\n{out.stderr}")
    return src


def build_main(verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu"))
                  + glob.glob(os.path.join(HERE, "csrc", "engine", "*.cpp")))
    hdr_time = _newest(_headers())
    objs = [os.path.join(OBJ_DIR, os.path.relpath(s, os.path.join(HERE, "csrc")) + ".o") for s in srcs]
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for done in ex.map(lambda so: _compile(so[0], so[1], hdr_time), zip(srcs, objs)):
            if done and verbose:
                print("compiled", os.path.relpath(done, ROOT))
    if not os.path.exists(MAIN_LIB) or os.path.getmtime(MAIN_LIB) < _newest(objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", MAIN_LIB, *objs, "-lpthread"]
        out = subprocess.run(cmd, capture_output=True, text=True)
        if out.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{out.stdout}\n{out.stderr}")
    return MAIN_LIB


def build_device_plugin(verbose: bool = False) -> str | None:
    """The nert::Device plug-in needs NERT's public headers at compile time."""
    src = os.path.join(HERE, "device", "b200_device.cpp")
    inc = nert_include()
    if not os.path.exists(src):
        return None
    if inc is None:
        return DEVICE_LIB if os.path.exists(DEVICE_LIB) else None
    if os.path.exists(DEVICE_LIB) and os.path.getmtime(DEVICE_LIB) >= max(
            os.path.getmtime(src), os.path.getmtime(MAIN_LIB), _newest(_headers())):
        return DEVICE_LIB
    cmd = ["g++", *CXX_FLAGS, "-shared", "-I", inc, "-I", os.path.join(ROOT, "include"), src, "-o", DEVICE_LIB,
           "-L", LIB_DIR, "-lnert_b200", "-Wl,-rpath,$ORIGIN"]
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"device plug-in build failed: {' '.join(cmd)}\n{out.stdout}\n{out.stderr}")
    if verbose:
        print("built", os.path.relpath(DEVICE_LIB, ROOT))
    return DEVICE_LIB


def build(verbose: bool = False) -> None:
    os.makedirs(LIB_DIR, exist_ok=True)
    build_main(verbose)
    build_device_plugin(verbose)


if __name__ == "__main__":
    build(verbose="-q" not in sys.argv)
