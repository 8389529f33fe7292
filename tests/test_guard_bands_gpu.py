"""Out-of-bounds write detection without compute-sanitizer (closed on this pool):
every buffer a kernel writes is placed inside a larger allocation whose head and
tail are filled with a sentinel byte pattern; after the kernel the sentinels must be
intact, and the result must equal the same call on an ordinary allocation."""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

GUARD = 1 << 16   # bytes of sentinel before and after each guarded buffer


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


class Guarded:
    """A tensor of `like`'s shape and dtype inside a sentinel-filled allocation."""

    def __init__(self, like: torch.Tensor):
        nbytes = like.numel() * like.element_size()
        self.raw = torch.full((GUARD + nbytes + GUARD,), 0xA5, dtype=torch.uint8,
                              device=like.device)
        self.t = self.raw[GUARD:GUARD + nbytes].view(like.dtype).view(like.shape)
        self.t.copy_(like)

    def intact(self) -> bool:
        head = self.raw[:GUARD]
        tail = self.raw[-GUARD:]
        return bool((head == 0xA5).all()) and bool((tail == 0xA5).all())


@pytest.mark.parametrize("name", ["bf16_bs16_varlen", "bf16_bs16_decode", "f16_generic_d96",
                                  "edge_empty_seqs_prefill", "opt_lse_decode_bf16"])
def test_attention_writes_stay_in_bounds(name):
    from gpu_util import attention_capi, attention_ex_capi, attn_case_to_dev, handle
    from tecoops import capi
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    out = Guarded(torch.zeros_like(d["q"]))
    kc, vc = Guarded(d["kc"]), Guarded(d["vc"])
    dt = capi.DATA_HALF if c["dtype"] == "f16" else capi.DATA_BFLOAT16
    descs = (capi.Desc(capi.DATA_INT32, d["bt"].shape), capi.Desc(dt, d["q"].shape),
             capi.Desc(dt, d["kc"].shape))
    lse = Guarded(torch.zeros(d["q"].shape[1], d["q"].shape[0], device="cuda"))
    st = capi.flash_attention_ex(handle(), int(inp["q_lens"].max()), int(inp["kv_lens"].max()),
                                 d["kc"].shape[0], d["q_lens"].data_ptr(), d["kv_lens"].data_ptr(),
                                 descs[0], d["bt"].data_ptr(), descs[1], d["q"].data_ptr(),
                                 descs[2], kc.t.data_ptr(), descs[2], vc.t.data_ptr(), descs[1],
                                 out.t.data_ptr(), 0, softmax_lse=lse.t.data_ptr())
    capi.check(st, "tecoopsFlashAttentionEx")
    torch.cuda.synchronize()
    assert out.intact() and kc.intact() and vc.intact() and lse.intact()
    assert torch.equal(out.t, ref)


@pytest.mark.parametrize("name", ["cfg1_bf16", "d72_unaligned", "all_padding"])
def test_reshape_writes_stay_in_bounds(name):
    from gpu_util import reshape_capi, words_to_dev
    c = cases.RESHAPE_CASES[name]
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    dk, dv = words_to_dev(key, c["dtype"]), words_to_dev(value, c["dtype"])
    ds = torch.from_numpy(slot).cuda()
    gk, gv = Guarded(words_to_dev(kc, c["dtype"])), Guarded(words_to_dev(vc, c["dtype"]))
    reshape_capi(dk, dv, ds, gk.t, gv.t)
    rk, rv = words_to_dev(kc, c["dtype"]), words_to_dev(vc, c["dtype"])
    reshape_capi(dk, dv, ds, rk, rv)
    torch.cuda.synchronize()
    assert gk.intact() and gv.intact()
    assert torch.equal(gk.t, rk) and torch.equal(gv.t, rv)


@pytest.mark.parametrize("name", ["api_add_4096", "f16_ragged_100", "bf16_norm_16384"])
def test_rms_norm_writes_stay_in_bounds(name):
    from gpu_util import handle, words_to_dev
    from tecoops import capi
    c = cases.RMS_CASES[name]
    x, w, r = cases.rms_inputs(c)
    dx, dw = words_to_dev(x, c["dtype"]), words_to_dev(w, c["dtype"])
    dr = words_to_dev(r, c["dtype"]) if r is not None else None
    dt = None if c["dtype"] == "f16" else capi.DATA_BFLOAT16
    out, ro = Guarded(torch.zeros_like(dx)), Guarded(torch.zeros_like(dx))
    capi.check(capi.rms_norm(handle(), dx.data_ptr(), dw.data_ptr(),
                             dr.data_ptr() if dr is not None else 0, out.t.data_ptr(),
                             ro.t.data_ptr() if dr is not None else 0, c["N"], c["D"], c["eps"],
                             dtype=dt), "tecoopsRmsNorm")
    torch.cuda.synchronize()
    assert out.intact() and ro.intact()
    assert np.isfinite(out.t.float().cpu().numpy()).all()
