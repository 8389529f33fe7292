"""tecoopsFlashAttentionDecodeNoAlloc — decode for callers that cannot allocate.

Some callers of this library cannot allocate device memory when they run
attention: an engine plugin that is handed only its input and output buffers,
or a server whose memory planner forbids cudaMalloc after start-up.  For them the
library offers a decode entry point whose split scratch is a static 16 MiB
device array inside the library.  This test calls it through the C ABI twice in
a row (two different batches) and checks each result against the regular
tecoopsFlashAttention entry point on the same inputs, within the attention
tolerances the other parity tests use; it also checks that shapes needing more
scratch than the static array holds are refused.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _decode_batch(seed, B, max_ctx, Hq=32, Hkv=8, D=128, bs=16, pool=20000):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, max_ctx + 1, (B,), generator=g)
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    pages = ((ctx + bs - 1) // bs).tolist()
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    gd = torch.Generator(device="cuda").manual_seed(seed + 1)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    return dict(q=q, kc=kc, vc=vc, q_lens=torch.ones(B, dtype=torch.int32, device="cuda"),
                kv_lens=ctx.to(torch.int32).cuda(), bt=bt.cuda(), max_k=int(ctx.max()))


def _no_alloc(d, h):
    from tecoops import capi
    dt = capi.DATA_BFLOAT16
    out = torch.full_like(d["q"], float("nan"))
    descs = (capi.Desc(capi.DATA_INT32, d["bt"].shape), capi.Desc(dt, d["q"].shape),
             capi.Desc(dt, d["kc"].shape), capi.Desc(dt, d["vc"].shape), capi.Desc(dt, out.shape))
    st = capi.flash_attention_decode_noalloc(
        h, d["max_k"], d["q_lens"].data_ptr(), d["kv_lens"].data_ptr(), descs[0],
        d["bt"].data_ptr(), descs[1], d["q"].data_ptr(), descs[2], d["kc"].data_ptr(), descs[3],
        d["vc"].data_ptr(), descs[4], out.data_ptr())
    return st, out


def test_decode_no_alloc_matches_regular_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpu_util import attention_capi, attn_case_to_dev
    from tecoops import capi
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    # two calls in a row on different batches: a long-context batch that needs
    # many splits, then a small ragged one (the array keeps the first call's data)
    batches = [_decode_batch(5, 64, 8192),
               dict(attn_case_to_dev(cases.attn_inputs(cases.ATTN_CASES["bf16_bs16_decode"]),
                                     "bf16"))]
    batches[1]["max_k"] = int(batches[1]["kv_lens"].max())
    for d in batches:
        st, out = _no_alloc(d, h)
        assert st == capi.SUCCESS, capi.error_string(st)
        ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                             max_q=1, max_k=d["max_k"])
        torch.cuda.synchronize()
        diff = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert diff.max().item() <= MAX_ABS and diff.mean().item() <= MEAN_ABS
    # shapes whose split plan needs more than the static 16 MiB are refused before
    # anything is launched (64 sequences x 128 q heads, contexts up to 32k tokens)
    d = batches[0]
    dt = capi.DATA_BFLOAT16
    big = (capi.Desc(capi.DATA_INT32, (64, 2048)), capi.Desc(dt, (64, 128, 128)),
           capi.Desc(dt, (20000, 8, 16, 128)))
    p = d["q"].data_ptr()
    st = capi.flash_attention_decode_noalloc(h, 32768, p, p, big[0], p, big[1], p, big[2], p,
                                             big[2], p, big[1], p)
    assert st == capi.NOT_SUPPORTED
    h.close()
