"""ctypes binding of the C ABI in include/tecoops.h (libteco_ops.so).

This is the binding a Python caller without the torch extension would use: plain
pointers and sizes, statuses returned as ints.  The parity tests call the
kernels through it.  Device pointers are plain integers (e.g. ``tensor.data_ptr()``).
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_HERE, "libteco_ops.so")

# tecoopsStatus_t
SUCCESS, NOT_INITIALIZED, ALLOC_FAILED, BAD_PARAM, INTERNAL_ERROR, INVALID_VALUE, \
    NOT_SUPPORTED = range(7)
# tecoopsDataType_t
DATA_FLOAT, DATA_HALF, DATA_INT8, DATA_INT16, DATA_INT32, DATA_INT64, DATA_UINT8, DATA_BOOL, \
    DATA_DOUBLE, DATA_BFLOAT16, DATA_COMPLEX_FLOAT = range(11)
DATA_FLOAT8_E4M3 = 32   # extension: e4m3 KV cache
# tecoopsKvLayout_t
KV_LAYOUT_HND, KV_LAYOUT_NHD = 0, 1
# tecoopsTensorFormat_t
TENSOR_NCHW, TENSOR_NHWC, TENSOR_CHWN, TENSOR_NWHC = range(4)

# every symbol declared in include/tecoops.h
EXPORTED = [
    "tecoopsCreate", "tecoopsDestroy", "tecoopsSetStream", "tecoopsGetStream",
    "tecoopsGetErrorString", "tecoopsCreateTensorDescriptor", "tecoopsSetTensor4dDescriptor",
    "tecoopsGetTensor4dDescriptor", "tecoopsSetTensorNdDescriptor",
    "tecoopsGetTensorNdDescriptor", "tecoopsDestroyTensorDescriptor", "tecoopsMemset",
    "tecoopsReshapeAndCache", "tecoopsReshapeAndCacheEx", "tecoopsFlashAttention", "tecoopsGetFlashAttentionWorkspaceSize",
    "tecoopsGetDeviceErrorStatus", "tecoopsSetDeviceWaitLimit",
    "tecoopsFlashAttentionDecodeNoAlloc", "tecoopsFlashAttentionEx",
    "tecoopsReshapeAndCacheFlashAttentionDecode", "tecoopsFlattenRays", "tecoopsReduceVariance",
    "tecoopsMorton3DInvert", "tecoopsRmsNorm", "tecoopsRmsNormEx", "tecoopsCausalConv1d",
]

_vp = ctypes.c_void_p
_i = ctypes.c_int
_lib = None


class FlashAttentionOptions(ctypes.Structure):
    """tecoopsFlashAttentionOptions_t."""
    _fields_ = [("softmax_scale", ctypes.c_float), ("causal", _i), ("window_left", _i),
                ("window_right", _i), ("kv_layout", _i), ("k_scale", ctypes.c_float),
                ("v_scale", ctypes.c_float)]


class KvCacheConfig(ctypes.Structure):
    """tecoopsKvCacheConfig_t."""
    _fields_ = [("kv_layout", _i), ("cache_dtype", _i), ("k_scale", ctypes.c_float),
                ("v_scale", ctypes.c_float)]


class TecoopsError(RuntimeError):
    def __init__(self, what: str, status: int):
        super().__init__(f"{what}: {error_string(status)} ({status})")
        self.status = status


def lib():
    """Load libteco_ops.so (raises OSError loudly when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIBRARY_PATH):
        raise OSError(f"libteco_ops.so not built at {LIBRARY_PATH}; run teco-ops_b200/build.py")
    L = ctypes.CDLL(LIBRARY_PATH)
    sig = {
        "tecoopsCreate": [ctypes.POINTER(_vp)],
        "tecoopsDestroy": [_vp],
        "tecoopsSetStream": [_vp, _vp],
        "tecoopsGetStream": [_vp, ctypes.POINTER(_vp)],
        "tecoopsCreateTensorDescriptor": [ctypes.POINTER(_vp)],
        "tecoopsSetTensor4dDescriptor": [_vp, _i, _i, _i, _i, _i, _i],
        "tecoopsGetTensor4dDescriptor": [_vp] + [ctypes.POINTER(_i)] * 9,
        "tecoopsSetTensorNdDescriptor": [_vp, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)],
        "tecoopsGetTensorNdDescriptor": [_vp, _i, ctypes.POINTER(_i), ctypes.POINTER(_i),
                                         ctypes.POINTER(_i), ctypes.POINTER(_i)],
        "tecoopsDestroyTensorDescriptor": [_vp],
        "tecoopsMemset": [_vp, _vp, _i, ctypes.c_size_t],
        "tecoopsReshapeAndCache": [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i],
        "tecoopsReshapeAndCacheEx": [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                                     ctypes.POINTER(KvCacheConfig)],
        "tecoopsFlashAttention": [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                  _vp, _vp, _vp, _vp],
        "tecoopsGetFlashAttentionWorkspaceSize": [_vp, _i, _i, _vp, _vp, _vp,
                                                  ctypes.POINTER(ctypes.c_size_t)],
        "tecoopsGetDeviceErrorStatus": [_vp, ctypes.POINTER(_i)],
        "tecoopsSetDeviceWaitLimit": [_vp, ctypes.c_ulonglong, _i],
        "tecoopsFlashAttentionDecodeNoAlloc": [_vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                               _vp, _vp, _vp, _vp],
        "tecoopsFlashAttentionEx": [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _vp, _vp, _vp, _vp,
                                    ctypes.POINTER(FlashAttentionOptions), _vp],
        "tecoopsReshapeAndCacheFlashAttentionDecode": [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp,
                                                       _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                                       _vp, _vp],
        "tecoopsRmsNorm": [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, ctypes.c_float],
        "tecoopsRmsNormEx": [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, ctypes.c_float, _i],
    }
    for name, args in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = _i
    L.tecoopsGetErrorString.argtypes = [_i]
    L.tecoopsGetErrorString.restype = ctypes.c_char_p
    _lib = L
    return L


def error_string(status: int) -> str:
    return lib().tecoopsGetErrorString(int(status)).decode()


def check(status: int, what: str):
    if status != SUCCESS:
        raise TecoopsError(what, status)


class Handle:
    """Owns a tecoopsHandle_t (created on the current CUDA device)."""

    def __init__(self, stream: int = 0):
        self.h = _vp()
        check(lib().tecoopsCreate(ctypes.byref(self.h)), "tecoopsCreate")
        if stream:
            check(lib().tecoopsSetStream(self.h, _vp(stream)), "tecoopsSetStream")

    def set_stream(self, stream: int):
        check(lib().tecoopsSetStream(self.h, _vp(stream)), "tecoopsSetStream")

    def close(self):
        if self.h:
            lib().tecoopsDestroy(self.h)
            self.h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Desc:
    """Owns a tecoopsTensorDescriptor_t set with packed Nd dims."""

    def __init__(self, dtype: int, dims):
        self.d = _vp()
        check(lib().tecoopsCreateTensorDescriptor(ctypes.byref(self.d)), "CreateTensorDescriptor")
        arr = (_i * len(dims))(*[int(x) for x in dims])
        check(lib().tecoopsSetTensorNdDescriptor(self.d, dtype, len(dims), arr, None),
              "SetTensorNdDescriptor")

    def __del__(self):
        try:
            lib().tecoopsDestroyTensorDescriptor(self.d)
        except Exception:
            pass


def reshape_and_cache(handle: Handle, key, value, slot_mapping, key_cache, value_cache,
                      num_tokens, num_kv_heads, head_size, num_blocks, block_size) -> int:
    """Raw C call; pointers are ints. Returns the tecoopsStatus_t."""
    return lib().tecoopsReshapeAndCache(handle.h, _vp(key), _vp(value), _vp(slot_mapping),
                                        _vp(key_cache), _vp(value_cache), num_tokens,
                                        num_kv_heads, head_size, num_blocks, block_size)


def reshape_and_cache_ex(handle: Handle, key, value, slot_mapping, key_cache, value_cache,
                         num_tokens, num_kv_heads, head_size, num_blocks, block_size, key_dtype,
                         kv_layout=KV_LAYOUT_HND, cache_dtype=None, k_scale=1.0,
                         v_scale=1.0) -> int:
    """tecoopsReshapeAndCacheEx: page layout and e4m3 caches (cache_dtype
    DATA_FLOAT8_E4M3 stores e4m3(x / scale))."""
    cfg = KvCacheConfig(int(kv_layout), int(key_dtype if cache_dtype is None else cache_dtype),
                        float(k_scale), float(v_scale))
    return lib().tecoopsReshapeAndCacheEx(handle.h, _vp(key), _vp(value), _vp(slot_mapping),
                                          _vp(key_cache), _vp(value_cache), num_tokens,
                                          num_kv_heads, head_size, num_blocks, block_size,
                                          int(key_dtype), ctypes.byref(cfg))


def flash_attention(handle: Handle, max_seqlen_q, max_seqlen_k, max_block_num, q_seq_lens,
                    kv_seq_lens, bt_desc: Desc, block_table, q_desc: Desc, q, k_desc: Desc,
                    k_cache, v_desc: Desc, v_cache, o_desc: Desc, out, workspace=0) -> int:
    return lib().tecoopsFlashAttention(handle.h, max_seqlen_q, max_seqlen_k, max_block_num,
                                       _vp(q_seq_lens), _vp(kv_seq_lens), bt_desc.d,
                                       _vp(block_table), q_desc.d, _vp(q), k_desc.d,
                                       _vp(k_cache), v_desc.d, _vp(v_cache), o_desc.d, _vp(out),
                                       _vp(workspace) if workspace else None)


def flash_attention_ex(handle: Handle, max_seqlen_q, max_seqlen_k, max_block_num, q_seq_lens,
                       kv_seq_lens, bt_desc: Desc, block_table, q_desc: Desc, q, k_desc: Desc,
                       k_cache, v_desc: Desc, v_cache, o_desc: Desc, out, workspace=0,
                       softmax_scale=0.0, causal=True, window=(-1, -1), softmax_lse=0,
                       kv_layout=KV_LAYOUT_HND, k_scale=1.0, v_scale=1.0) -> int:
    """tecoopsFlashAttentionEx: scale (<= 0: 1/sqrt(D)), causal, window (left, right;
    negative = unbounded), an optional fp32 [Hq, total_q] log-sum-exp output, the cache
    page layout and (e4m3 cache descriptors) the dequantisation scales."""
    opts = FlashAttentionOptions(float(softmax_scale), 1 if causal else 0, int(window[0]),
                                 int(window[1]), int(kv_layout), float(k_scale), float(v_scale))
    return lib().tecoopsFlashAttentionEx(handle.h, max_seqlen_q, max_seqlen_k, max_block_num,
                                         _vp(q_seq_lens), _vp(kv_seq_lens), bt_desc.d,
                                         _vp(block_table), q_desc.d, _vp(q), k_desc.d,
                                         _vp(k_cache), v_desc.d, _vp(v_cache), o_desc.d,
                                         _vp(out), _vp(workspace) if workspace else None,
                                         ctypes.byref(opts),
                                         _vp(softmax_lse) if softmax_lse else None)


def reshape_and_cache_flash_attention_decode(handle: Handle, key, value, slot_mapping,
                                             max_seqlen_k, q_seq_lens, kv_seq_lens,
                                             bt_desc: Desc, block_table, q_desc: Desc, q,
                                             k_desc: Desc, k_cache, v_desc: Desc, v_cache,
                                             o_desc: Desc, out, workspace=0) -> int:
    """One decode step: scatter of the new tokens' K/V and attention in one launch."""
    return lib().tecoopsReshapeAndCacheFlashAttentionDecode(
        handle.h, _vp(key), _vp(value), _vp(slot_mapping), max_seqlen_k, _vp(q_seq_lens),
        _vp(kv_seq_lens), bt_desc.d, _vp(block_table), q_desc.d, _vp(q), k_desc.d, _vp(k_cache),
        v_desc.d, _vp(v_cache), o_desc.d, _vp(out), _vp(workspace) if workspace else None)


def flash_attention_decode_noalloc(handle: Handle, max_seqlen_k, q_seq_lens, kv_seq_lens,
                                   bt_desc: Desc, block_table, q_desc: Desc, q, k_desc: Desc,
                                   k_cache, v_desc: Desc, v_cache, o_desc: Desc, out) -> int:
    """Decode for callers that cannot allocate: scratch is the library's static array."""
    return lib().tecoopsFlashAttentionDecodeNoAlloc(handle.h, max_seqlen_k, _vp(q_seq_lens),
                                                    _vp(kv_seq_lens), bt_desc.d, _vp(block_table),
                                                    q_desc.d, _vp(q), k_desc.d, _vp(k_cache),
                                                    v_desc.d, _vp(v_cache), o_desc.d, _vp(out))


def rms_norm(handle: Handle, input, weight, residual, output, residual_out, num_tokens,
             hidden_size, eps, dtype=None) -> int:
    """tecoopsRmsNorm (fp16) or, with dtype, tecoopsRmsNormEx; residual 0 = none."""
    args = (handle.h, _vp(input), _vp(weight), _vp(residual) if residual else None, _vp(output),
            _vp(residual_out) if residual_out else None, int(num_tokens), int(hidden_size),
            float(eps))
    if dtype is None:
        return lib().tecoopsRmsNorm(*args)
    return lib().tecoopsRmsNormEx(*args, int(dtype))


def workspace_size(handle: Handle, max_seqlen_q, max_seqlen_k, bt_desc: Desc, q_desc: Desc,
                   k_desc: Desc) -> int:
    n = ctypes.c_size_t(0)
    check(lib().tecoopsGetFlashAttentionWorkspaceSize(handle.h, max_seqlen_q, max_seqlen_k,
                                                      bt_desc.d, q_desc.d, k_desc.d,
                                                      ctypes.byref(n)),
          "GetFlashAttentionWorkspaceSize")
    return n.value


def device_error(handle: Handle):
    code = _i(0)
    st = lib().tecoopsGetDeviceErrorStatus(handle.h, ctypes.byref(code))
    return st, code.value


def set_device_wait_limit(handle: Handle, limit_ns: int, stall_test: bool = False) -> int:
    """Limit of the decode kernel's bounded waits; stall_test makes its first ring
    wait target a barrier nothing completes (tests of the give-up path)."""
    return lib().tecoopsSetDeviceWaitLimit(handle.h, int(limit_ns), 1 if stall_test else 0)
