"""ORACLE — test infrastructure only (see oracle/__init__.py).

e4m3 ("FP8 E4M3", OCP 8-bit floating point specification: sign, 4 exponent bits
with bias 7, 3 mantissa bits, subnormals, no infinities, S.1111.111 = NaN, largest
finite 448) in numpy, as the e4m3 KV cache uses it (vLLM's ``kv_cache_dtype="fp8"``
convention): ``stored = e4m3(x / scale)`` with IEEE fp32 division, round to nearest
even, finite saturation (|v| > 448 -> +-448); ``read = decode(stored) * scale``.

The reference stores its cache in fp16 only, so this is a restated encoding with
no reference counterpart; the GPU kernels are checked bit-exactly against it.
"""
from __future__ import annotations

import numpy as np


def _table():
    b = np.arange(256, dtype=np.uint16)
    s = (b >> 7) & 1
    e = (b >> 3) & 0xF
    m = b & 7
    mag = np.where(e == 0, m.astype(np.float64) * 2.0 ** -9,
                   (1.0 + m.astype(np.float64) / 8.0) * 2.0 ** (e.astype(np.float64) - 7))
    v = np.where(s == 1, -mag, mag)
    v[(e == 0xF) & (m == 7)] = np.nan
    return v


E4M3_VALUES = _table()                      # float64 [256]
_POS = E4M3_VALUES[:127]                    # 0 .. 448, increasing (codes 0x00..0x7e)


def decode(bits: np.ndarray) -> np.ndarray:
    """uint8 codes -> float32 values."""
    return E4M3_VALUES[np.asarray(bits, dtype=np.uint8)].astype(np.float32)


def encode(x: np.ndarray) -> np.ndarray:
    """float32 -> uint8 e4m3 codes: round to nearest even, saturate to +-448, NaN -> 0x7f."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    a = np.minimum(a, 448.0)
    hi = np.searchsorted(_POS, a, side="left")          # first code with value >= a
    hi = np.minimum(hi, 126)
    lo = np.maximum(hi - 1, 0)
    vhi, vlo = _POS[hi], _POS[lo]
    exact = vhi == a
    d_hi, d_lo = vhi - a, a - vlo
    pick_hi = exact | (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)
    code[np.isnan(x)] = 0x7F
    return code


def quantize(x: np.ndarray, scale: float) -> np.ndarray:
    """The cache write: e4m3(x / scale) with fp32 division."""
    return encode(np.asarray(x, np.float32) / np.float32(scale))


def dequantize(bits: np.ndarray, scale: float) -> np.ndarray:
    """The cache read: e4m3 value * scale (fp32)."""
    return decode(bits) * np.float32(scale)
