"""ORACLE — test infrastructure only (see oracle/__init__.py).

Python entry points of the reshape_and_cache golden
(test/zoo/teco/reshape_and_cache/reshape_and_cache.cpp:136-147): the C
restatement in ``reshape_and_cache.c`` (built by ``__graft_entry__.build()`` into
``oracle/liboracle_rc.so``) and an equivalent numpy version for cases where the C
library is not built.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle_rc.so")
        if not os.path.exists(path):
            return None
        lib = ctypes.CDLL(path)
        lib.oracle_reshape_and_cache.restype = ctypes.c_int
        lib.oracle_reshape_and_cache.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        _LIB = lib
    return _LIB


def reshape_and_cache(key, value, slot_mapping, key_cache, value_cache, threads: int = 1):
    """In-place scatter on numpy arrays of 16-bit words (uint16/int16/float16).

    key/value: [T, H, D]; slot_mapping: int64 [T]; caches: [NB, H, bs, D].
    Uses the C restatement when built, else :func:`reshape_and_cache_np`.
    """
    lib = _lib()
    T, H, D = key.shape
    NB, _, BS, _ = key_cache.shape
    for a in (key, value, key_cache, value_cache):
        assert a.dtype.itemsize == 2 and a.flags["C_CONTIGUOUS"]
    slot = np.ascontiguousarray(slot_mapping, dtype=np.int64)
    if lib is None:
        return reshape_and_cache_np(key, value, slot, key_cache, value_cache)
    lib.oracle_reshape_and_cache(key.ctypes.data, value.ctypes.data, slot.ctypes.data,
                                 key_cache.ctypes.data, value_cache.ctypes.data, T, H, D, NB,
                                 BS, threads)
    return key_cache, value_cache


def reshape_and_cache_np(key, value, slot_mapping, key_cache, value_cache):
    """numpy restatement (sequential semantics: for duplicate slots the last token wins)."""
    T, H, D = key.shape
    NB, _, BS, _ = key_cache.shape
    slot = np.asarray(slot_mapping, dtype=np.int64)
    for t in range(T):
        s = int(slot[t])
        if s < 0 or s >= NB * BS:
            continue
        key_cache[s // BS, :, s % BS, :] = key[t]
        value_cache[s // BS, :, s % BS, :] = value[t]
    return key_cache, value_cache


def reshape_bytes(slot_mapping, num_kv_heads: int, head_dim: int, elem: int = 2) -> int:
    """Algorithmic HBM bytes: read slot_mapping, read K and V rows of valid slots,
    write them to the caches."""
    slot = np.asarray(slot_mapping)
    valid = int((slot >= 0).sum())
    return 8 * slot.size + 4 * valid * num_kv_heads * head_dim * elem
