"""Seeded synthetic inputs: splitmix64 + Box-Muller, N(0, 1) as float32.

Repo-owned so the same seed gives the same data on any machine and in any
language (std::normal_distribution is implementation-defined).  Vectorised
with numpy's wrapping uint64 arithmetic.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """Outputs offset+1 .. offset+n of splitmix64 seeded with `seed`."""
    i = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def normal(seed: int, shape, offset: int = 0) -> np.ndarray:
    """N(0, 1) float32 array of `shape` (Box-Muller on pairs of draws)."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    z = splitmix64(seed, 2 * m, 2 * offset)
    u1 = ((z[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
    u2 = (z[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * m, np.float64)
    out[0::2] = r * np.cos(2.0 * np.pi * u2)
    out[1::2] = r * np.sin(2.0 * np.pi * u2)
    return out[:n].astype(np.float32).reshape(shape)


def uniform_int(seed: int, n: int, lo: int, hi: int, offset: int = 0) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive)."""
    z = splitmix64(seed, n, offset)
    return (lo + (z % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int64)
