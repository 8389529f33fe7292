"""tecoopsFlashAttentionDecodeNoAlloc — decode for callers that cannot allocate.

Some callers of this library cannot allocate device memory when they run
attention: an engine plugin that is handed only its input and output buffers,
or a server whose memory planner forbids cudaMalloc after start-up.  For them the
library offers a decode entry point whose split scratch is a static 16 MiB
device array inside the library.  This test calls it through the C ABI several
times in a row (batches of different shapes) and checks each result against the
regular tecoopsFlashAttention entry point on the same inputs and, for the ragged
batch, against the CPU oracle of the reference golden, within the attention
tolerances the other parity tests use.  After a warm-up call (which reserves the
static array on the device) the free device memory must not change across the
following calls: the entry point allocates nothing.  It also checks that shapes
needing more scratch than the static array holds, and q tensors with more rows
than sequences, are refused, and that a q_len above 1 is reported through the
entry point's own error word.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""
import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import seeded

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


def _no_alloc(d, h, out):
    from tecoops import capi
    dt = capi.DATA_BFLOAT16
    descs = (capi.Desc(capi.DATA_INT32, d["bt"].shape), capi.Desc(dt, d["q"].shape),
             capi.Desc(dt, d["kc"].shape), capi.Desc(dt, d["vc"].shape), capi.Desc(dt, out.shape))
    st = capi.flash_attention_decode_noalloc(
        h, d["max_k"], d["q_lens"].data_ptr(), d["kv_lens"].data_ptr(), descs[0],
        d["bt"].data_ptr(), descs[1], d["q"].data_ptr(), descs[2], d["kc"].data_ptr(), descs[3],
        d["vc"].data_ptr(), descs[4], out.data_ptr())
    return st, out


def _check(out, ref):
    diff = (out.float() - ref.float()).abs()
    assert torch.isfinite(out.float()).all()
    assert diff.max().item() <= MAX_ABS and diff.mean().item() <= MEAN_ABS


def test_decode_no_alloc_matches_regular_entry_point_and_oracle():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpu_util import attention_capi, attn_case_to_dev, errors
    from tecoops import capi
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    c = cases.ATTN_CASES["bf16_bs16_decode"]
    inp = cases.attn_inputs(c)
    small = dict(attn_case_to_dev(inp, "bf16"))
    small["max_k"] = int(small["kv_lens"].max())
    big = _decode_batch(5, 64, 8192)
    ref_small = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], "bf16"), seeded.words_to_f32(inp["k_cache"], "bf16"),
        seeded.words_to_f32(inp["v_cache"], "bf16"), inp["q_lens"], inp["kv_lens"],
        inp["block_table"])
    # regular-entry-point results first (they may grow the handle's own scratch)
    regular = [attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                              max_q=1, max_k=d["max_k"], h=h) for d in (small, big)]
    outs = [torch.full_like(d["q"], float("nan")) for d in (small, big, small)]
    # warm-up call: loads the library's device code on this GPU (reserving the
    # static array) and looks up its address
    st, _ = _no_alloc(small, h, outs[0])
    assert st == capi.SUCCESS, capi.error_string(st)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    # two more calls in a row: a long-context batch that needs many splits, then the
    # small ragged batch again (the array still holds the long batch's partials)
    for d, out in ((big, outs[1]), (small, outs[2])):
        st, _ = _no_alloc(d, h, out)
        assert st == capi.SUCCESS, capi.error_string(st)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "the no-allocation entry point allocated"
    assert capi.device_error(h) == (capi.SUCCESS, 0)
    for out, ref in ((outs[0], regular[0]), (outs[1], regular[1]), (outs[2], regular[0])):
        _check(out, ref)
    for out in (outs[0], outs[2]):
        mx, mean, _ = errors(out.float().cpu().numpy(), ref_small)
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
    h.close()


def test_decode_no_alloc_refusals_and_error_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tecoops import capi
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    d = _decode_batch(7, 8, 600)
    # shapes whose split plan needs more than the static 16 MiB are refused before
    # anything is launched (64 sequences x 128 q heads, contexts up to 32k tokens)
    dt = capi.DATA_BFLOAT16
    big = (capi.Desc(capi.DATA_INT32, (64, 2048)), capi.Desc(dt, (64, 128, 128)),
           capi.Desc(dt, (20000, 8, 16, 128)))
    p = d["q"].data_ptr()
    st = capi.flash_attention_decode_noalloc(h, 32768, p, p, big[0], p, big[1], p, big[2], p,
                                             big[2], p, big[1], p)
    assert st == capi.NOT_SUPPORTED
    # more query rows than sequences: not a decode call
    q9 = torch.zeros(9, 32, 128, device="cuda", dtype=torch.bfloat16)
    d9 = dict(d, q=q9)
    st, _ = _no_alloc(d9, h, torch.empty_like(q9))
    assert st == capi.BAD_PARAM
    # a q_len above 1 reaches the kernel, which reports it through the entry point's
    # own error word (read by tecoopsGetDeviceErrorStatus on the handle's device)
    d2 = dict(d, q_lens=torch.tensor([1, 2, 1, 1, 1, 1, 0, 1], dtype=torch.int32,
                                     device="cuda"))
    st, _ = _no_alloc(d2, h, torch.empty_like(d["q"]))
    assert st == capi.SUCCESS
    assert capi.device_error(h) == (capi.INTERNAL_ERROR, 0x1400)
    assert capi.device_error(h) == (capi.SUCCESS, 0)   # cleared once read
    h.close()
