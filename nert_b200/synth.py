"""Seeded, toolchain-independent synthetic tensors.

Every tensor of every config is drawn from a counter-based generator so that
the same (config, tensor name) produces the same float32 bits on any host:

* a 64-bit seed is the FNV-1a hash of ``"<config>/<tensor>"``;
* element ``i`` is ``splitmix64(seed + (i + 1) * 0x9E3779B97F4A7C15)``
  (Steele, Lea & Flood, "Fast splittable pseudorandom number generators",
  OOPSLA 2014), evaluated with wrapping uint64 numpy arithmetic;
* uniform values take the top 24 bits (exact in float32);
* normal values use Box-Muller on two independent uniform streams, computed
  in float64 and rounded once to float32.
"""

from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def seed_of(config: str, tensor: str) -> int:
    """FNV-1a 64-bit hash of ``config/tensor``."""
    h = 0xCBF29CE484222325
    for b in f"{config}/{tensor}".encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _mix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _stream(seed: int, n: int) -> np.ndarray:
    idx = np.arange(1, n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + idx * _GOLDEN
    return _mix(z)


def uniform01(seed: int, n: int) -> np.ndarray:
    """n float64 values in [0, 1), each a multiple of 2**-24."""
    return (_stream(seed, n) >> np.uint64(40)).astype(np.float64) * (1.0 / (1 << 24))


def uniform(shape, lo: float, hi: float, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    u = uniform01(seed, n)
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def normal(shape, std: float, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    u1 = uniform01(seed, n)
    u2 = uniform01(seed ^ 0x5DEECE66D, n)
    u1 = np.maximum(u1, 2.0 ** -25)  # keep log finite
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (z * std).astype(np.float32).reshape(shape)
