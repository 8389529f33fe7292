"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and the host-side API (handles, descriptors, argument checks)
behaves like the reference's interface layer
(teco/interface/common/tecoops.cpp, teco/interface/ops/*.cpp)."""
import ctypes
import os
import re

import pytest

from tecoops import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "tecoops.h")).read()
    return sorted(set(re.findall(r"\b(tecoops[A-Z]\w*)\s*\(", src)))


def test_library_exports_every_header_symbol():
    L = capi.lib()
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), s
    assert sorted(capi.EXPORTED) == syms


def test_error_strings():
    assert capi.error_string(0) == "TECOOPS_STATUS_SUCCESS"
    assert capi.error_string(3) == "TECOOPS_STATUS_BAD_PARAM"
    assert capi.error_string(6) == "TECOOPS_STATUS_NOT_SUPPORTED"
    assert capi.error_string(99) == "UNKNOWN_ERROR"


def test_handle_stream_roundtrip():
    L = capi.lib()
    assert L.tecoopsCreate(None) == capi.BAD_PARAM
    h = capi.Handle()
    s = ctypes.c_void_p()
    assert L.tecoopsGetStream(h.h, ctypes.byref(s)) == capi.SUCCESS and not s.value
    assert L.tecoopsSetStream(h.h, ctypes.c_void_p(0x1234)) == capi.SUCCESS
    assert L.tecoopsGetStream(h.h, ctypes.byref(s)) == capi.SUCCESS and s.value == 0x1234
    assert L.tecoopsSetStream(None, None) == capi.BAD_PARAM
    assert L.tecoopsGetStream(h.h, None) == capi.BAD_PARAM
    h.set_stream(0)
    h.close()


def test_nd_descriptor_packed_strides_and_get():
    L = capi.lib()
    d = capi.Desc(capi.DATA_BFLOAT16, [5, 4, 3, 2])
    dt, nb = ctypes.c_int(), ctypes.c_int()
    dims, strides = (ctypes.c_int * 8)(), (ctypes.c_int * 8)()
    assert L.tecoopsGetTensorNdDescriptor(d.d, 8, ctypes.byref(dt), ctypes.byref(nb), dims,
                                          strides) == 0
    assert dt.value == capi.DATA_BFLOAT16 and nb.value == 4
    assert list(dims)[:4] == [5, 4, 3, 2] and list(strides)[:4] == [24, 6, 2, 1]
    # requested fewer dims -> only that many copied
    dims2 = (ctypes.c_int * 8)(*([-7] * 8))
    assert L.tecoopsGetTensorNdDescriptor(d.d, 2, None, ctypes.byref(nb), dims2, None) == 0
    assert list(dims2)[:3] == [5, 4, -7]
    assert L.tecoopsGetTensorNdDescriptor(d.d, 0, None, None, None, None) == capi.BAD_PARAM
    assert L.tecoopsSetTensorNdDescriptor(d.d, capi.DATA_HALF, 0, dims, None) == capi.BAD_PARAM
    explicit = (ctypes.c_int * 3)(100, 10, 1)
    d3 = (ctypes.c_int * 3)(2, 3, 4)
    assert L.tecoopsSetTensorNdDescriptor(d.d, capi.DATA_HALF, 3, d3, explicit) == 0
    assert L.tecoopsGetTensorNdDescriptor(d.d, 3, None, None, None, strides) == 0
    assert list(strides)[:3] == [100, 10, 1]


@pytest.mark.parametrize("fmt,expect", [
    (capi.TENSOR_NCHW, [60, 20, 5, 1]), (capi.TENSOR_NHWC, [60, 1, 15, 3]),
    (capi.TENSOR_CHWN, [1, 40, 10, 2]), (capi.TENSOR_NWHC, [60, 1, 3, 12])])
def test_4d_descriptor_formats(fmt, expect):
    L = capi.lib()
    d = ctypes.c_void_p()
    assert L.tecoopsCreateTensorDescriptor(ctypes.byref(d)) == 0
    assert L.tecoopsSetTensor4dDescriptor(d, fmt, capi.DATA_HALF, 2, 3, 4, 5) == 0
    out = [ctypes.c_int() for _ in range(9)]
    assert L.tecoopsGetTensor4dDescriptor(d, *[ctypes.byref(o) for o in out]) == 0
    assert [o.value for o in out[1:5]] == [2, 3, 4, 5]
    assert [o.value for o in out[5:]] == expect
    assert L.tecoopsDestroyTensorDescriptor(d) == 0


def test_reshape_argument_checks():
    """reference interface/ops/reshape_and_cache.cpp:39-62 (no kernel is launched)."""
    h = capi.Handle()
    p = 0x1000
    args = (p, p, p, p, p, 4, 2, 8, 4, 16)
    assert capi.lib().tecoopsReshapeAndCache(None, *[ctypes.c_void_p(a) for a in args[:5]],
                                             *args[5:]) == capi.NOT_INITIALIZED
    for i in range(5):
        a = list(args)
        a[i] = 0
        assert capi.reshape_and_cache(h, *a) == capi.BAD_PARAM
    for i in range(5, 10):
        a = list(args)
        a[i] = 0
        assert capi.reshape_and_cache(h, *a) == capi.BAD_PARAM


def _fa_descs(dt=capi.DATA_HALF, kdt=None, q=(10, 8, 128), k=(16, 2, 16, 128), bt=(2, 4)):
    kdt = dt if kdt is None else kdt
    return (capi.Desc(capi.DATA_INT32, bt), capi.Desc(dt, q), capi.Desc(kdt, k),
            capi.Desc(kdt, k), capi.Desc(dt, q))


def test_flash_attention_argument_checks():
    """reference interface/ops/flash_attention.cpp:44-69 plus the B200 extensions."""
    h = capi.Handle()
    p = 0x1000
    bt, q, k, v, o = _fa_descs()

    def call(handle=h, bt=bt, q=q, k=k, v=v, o=o, lens=p):
        return capi.flash_attention(handle, 4, 8, 16, lens, lens, bt, p, q, p, k, p, v, p, o, p)

    class NullHandle:
        h = None
    assert call(handle=NullHandle()) == capi.NOT_INITIALIZED
    # k/v dtype mismatch
    assert call(v=capi.Desc(capi.DATA_BFLOAT16, (16, 2, 16, 128))) == capi.BAD_PARAM
    # unsupported cache dtype
    f32 = _fa_descs(dt=capi.DATA_FLOAT)
    assert call(bt=f32[0], q=f32[1], k=f32[2], v=f32[3], o=f32[4]) == capi.BAD_PARAM
    # k/v shape mismatch
    assert call(v=capi.Desc(capi.DATA_HALF, (16, 2, 16, 64))) == capi.BAD_PARAM
    # Hq not a multiple of Hkv
    assert call(q=capi.Desc(capi.DATA_HALF, (10, 7, 128)),
                o=capi.Desc(capi.DATA_HALF, (10, 7, 128))) == capi.BAD_PARAM
    # q / cache dtype differ
    assert call(q=capi.Desc(capi.DATA_BFLOAT16, (10, 8, 128))) == capi.BAD_PARAM
    # null length pointers
    assert call(lens=0) == capi.BAD_PARAM
    # block table must be int32
    assert call(bt=capi.Desc(capi.DATA_INT64, (2, 4))) == capi.BAD_PARAM
    # head_dim beyond 256 -> not supported
    big = _fa_descs(q=(10, 8, 320), k=(16, 2, 16, 320))
    assert call(bt=big[0], q=big[1], k=big[2], v=big[3], o=big[4]) == capi.NOT_SUPPORTED


def test_workspace_query():
    h = capi.Handle()
    bt, q, k, _, _ = _fa_descs(q=(64, 32, 128), k=(40000, 8, 16, 128), bt=(64, 512))
    # decode with long contexts needs split partials; prefill needs none
    assert capi.workspace_size(h, 1, 8192, bt, q, k) > 0
    assert capi.workspace_size(h, 128, 8192, bt, q, k) == 0


def test_rms_norm_host_checks():
    """reference teco/interface/ops/rms_norm.cpp checkRmsNormInput."""
    L = capi.lib()
    h = capi.Handle()
    p = ctypes.c_void_p(16)
    assert L.tecoopsRmsNorm(None, p, p, None, p, None, 1, 1, 1e-6) == capi.NOT_INITIALIZED
    assert L.tecoopsRmsNorm(h.h, None, p, None, p, None, 1, 1, 1e-6) == capi.BAD_PARAM
    assert L.tecoopsRmsNorm(h.h, p, p, None, None, None, 1, 1, 1e-6) == capi.BAD_PARAM
    assert L.tecoopsRmsNorm(h.h, p, p, p, p, None, 1, 1, 1e-6) == capi.BAD_PARAM   # no residual_out
    assert L.tecoopsRmsNorm(h.h, p, p, None, p, None, 0, 8, 1e-6) == capi.BAD_PARAM
    assert L.tecoopsRmsNorm(h.h, p, p, None, p, None, 4, 0, 1e-6) == capi.BAD_PARAM
    assert L.tecoopsRmsNormEx(h.h, p, p, None, p, None, 4, 8, 1e-6, capi.DATA_FLOAT) == \
        capi.BAD_PARAM


def test_off_path_ops_not_supported():
    L = capi.lib()
    h = capi.Handle()
    assert L.tecoopsMemset(None, None, 0, 0) == capi.NOT_INITIALIZED
    assert L.tecoopsMemset(h.h, None, 0, 16) == capi.BAD_PARAM
