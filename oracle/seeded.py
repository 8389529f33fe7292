"""ORACLE — test infrastructure only (see oracle/__init__.py).

Deterministic, platform-independent input generator: a counter-based
splitmix64 hash of (seed, index) turned into uniform or normal floats.  The
golden fixtures in tests/golden/ store only the seed and shapes of their
inputs; the parity tests regenerate the identical bytes with these functions.
16-bit outputs are returned as uint16 words (fp16 via numpy, bf16 by
round-to-nearest-even of the fp32 value).
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def _splitmix(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + _GOLD
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def _bits(seed: int, n: int, stream: int = 0) -> np.ndarray:
    idx = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        base = _splitmix(np.array([seed * 2654435761 + stream * 40503 + 1], dtype=np.uint64))[0]
        return _splitmix(idx ^ base)


def uniform(seed: int, shape, lo: float = -1.0, hi: float = 1.0, stream: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    u = (_bits(seed, n, stream) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def normal(seed: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    u1 = (_bits(seed, n, 1) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    u2 = (_bits(seed, n, 2) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    u1 = np.maximum(u1, 1e-12)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return z.astype(np.float32).reshape(shape)


def randint(seed: int, shape, lo: int, hi: int) -> np.ndarray:
    """Integers uniform in [lo, hi)."""
    n = int(np.prod(shape))
    r = _bits(seed, n, 3) % np.uint64(hi - lo)
    return (r.astype(np.int64) + lo).reshape(shape)


def permutation(seed: int, n: int) -> np.ndarray:
    keys = _bits(seed, n, 4)
    return np.argsort(keys, kind="stable").astype(np.int64)


def to_f16_words(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_bf16_words(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return r.astype(np.uint16)


def words_to_f32(w: np.ndarray, dtype: str) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint16)
    if dtype == "f16":
        return w.view(np.float16).astype(np.float32)
    if dtype == "bf16":
        return (w.astype(np.uint32) << np.uint32(16)).view(np.float32)
    raise ValueError(dtype)


def to_words(x: np.ndarray, dtype: str) -> np.ndarray:
    return to_f16_words(x) if dtype == "f16" else to_bf16_words(x)
