"""tecoopsReshapeAndCacheFlashAttentionDecode (one launch for a decode step's
reshape_and_cache and attention) against the two operators run back to back:
outputs and caches bit-identical, and attention within the north-star tolerance
of the oracle on the updated cache."""
import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _run(c, pad_first=False, seed=7, kv_offset=0):
    from gpu_util import TORCH_DT, attention_capi, attn_case_to_dev, handle, reshape_capi
    from tecoops import capi
    inp = cases.attn_inputs(c)
    assert all(int(x) == 1 for x in inp["q_lens"])
    d = attn_case_to_dev(inp, c["dtype"])
    B, Hkv, D, bs = len(inp["q_lens"]), c["Hkv"], c["D"], c["bs"]
    g = torch.Generator(device="cuda").manual_seed(seed)
    knew = torch.randn(B, Hkv, D, device="cuda", generator=g).to(TORCH_DT[c["dtype"]])
    vnew = torch.randn(B, Hkv, D, device="cuda", generator=g).to(TORCH_DT[c["dtype"]])
    if kv_offset:   # the same values in views that start kv_offset elements into a buffer
        kb = torch.empty(knew.numel() + kv_offset, device="cuda", dtype=knew.dtype)
        vb = torch.empty_like(kb)
        kb[kv_offset:].copy_(knew.flatten())
        vb[kv_offset:].copy_(vnew.flatten())
        knew = kb[kv_offset:].view(knew.shape)
        vnew = vb[kv_offset:].view(vnew.shape)
    kl = inp["kv_lens"]
    slot = [int(inp["block_table"][b, (int(kl[b]) - 1) // bs]) * bs + (int(kl[b]) - 1) % bs
            for b in range(B)]
    if pad_first:
        slot[0] = -1
    slot = torch.tensor(slot, dtype=torch.int64, device="cuda")
    # unfused: the two operators
    kc_a, vc_a = d["kc"].clone(), d["vc"].clone()
    reshape_capi(knew, vnew, slot, kc_a, vc_a)
    out_a = attention_capi(d["q"], kc_a, vc_a, d["q_lens"], d["kv_lens"], d["bt"], max_q=1)
    # fused
    kc_b, vc_b = d["kc"].clone(), d["vc"].clone()
    out_b = torch.zeros_like(d["q"])
    dt = capi.DATA_HALF if c["dtype"] == "f16" else capi.DATA_BFLOAT16
    descs = (capi.Desc(capi.DATA_INT32, d["bt"].shape), capi.Desc(dt, d["q"].shape),
             capi.Desc(dt, kc_b.shape))
    st = capi.reshape_and_cache_flash_attention_decode(
        handle(), knew.data_ptr(), vnew.data_ptr(), slot.data_ptr(), int(kl.max()),
        d["q_lens"].data_ptr(), d["kv_lens"].data_ptr(), descs[0], d["bt"].data_ptr(), descs[1],
        d["q"].data_ptr(), descs[2], kc_b.data_ptr(), descs[2], vc_b.data_ptr(), descs[1],
        out_b.data_ptr())
    capi.check(st, "tecoopsReshapeAndCacheFlashAttentionDecode")
    torch.cuda.synchronize()
    return inp, d, (kc_a, vc_a, out_a), (kc_b, vc_b, out_b)


@pytest.mark.parametrize("name", ["bf16_bs16_decode", "api_decode_2x128",
                                  "bf16_decode_gqa16_bs128", "api_gqa_2q1kv_decode_2b"])
def test_fused_decode_matches_two_operators(name):
    from gpu_util import errors
    c = cases.ATTN_CASES[name]
    inp, d, (kc_a, vc_a, out_a), (kc_b, vc_b, out_b) = _run(c)
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
    assert torch.equal(out_a, out_b)
    ref = oracle.flash_attn_varlen(d["q"].float().cpu().numpy(), kc_b.float().cpu().numpy(),
                                   vc_b.float().cpu().numpy(), inp["q_lens"], inp["kv_lens"],
                                   inp["block_table"])
    mx, mean, _ = errors(out_b.float().cpu().numpy(), ref)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


def test_fused_decode_element_aligned_new_kv():
    """New K/V views at an odd element offset cannot feed the kernel's 16-byte scatter:
    the call runs the two operators instead, with the same results."""
    c = cases.ATTN_CASES["bf16_bs16_decode"]
    inp, d, (kc_a, vc_a, out_a), (kc_b, vc_b, out_b) = _run(c, kv_offset=1)
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
    assert torch.equal(out_a, out_b)


def test_fused_decode_padding_slot_leaves_cache():
    """slot -1: nothing is stored (the attention still uses the new token)."""
    c = cases.ATTN_CASES["bf16_bs16_decode"]
    inp, d, (kc_a, vc_a, _), (kc_b, vc_b, _) = _run(c, pad_first=True)
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)


def test_fused_decode_config3_full_size():
    """Llama-3-8B paged decode step (64 new tokens, 40,000-page pool): fused == unfused."""
    from gpu_util import attention_capi, handle, reshape_capi
    from tecoops import capi
    B, Hq, Hkv, D, bs, pool = 64, 32, 8, 128, 16, 40000
    ctx = torch.randint(512, 8193, (B,), generator=torch.Generator().manual_seed(20))
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(21)).to(torch.int32)
    pages = ((ctx + 1 + bs - 1) // bs).tolist()
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    g = torch.Generator(device="cuda").manual_seed(22)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=g)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=g)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16, generator=g)
    knew = torch.randn(B, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    vnew = torch.randn(B, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    slot = torch.tensor([int(bt[b, int(ctx[b]) // bs]) * bs + int(ctx[b]) % bs for b in range(B)],
                        dtype=torch.int64, device="cuda")
    kv = (ctx + 1).to(torch.int32).cuda()
    ones = torch.ones(B, dtype=torch.int32, device="cuda")
    btd = bt.cuda()
    kc_b, vc_b = kc.clone(), vc.clone()
    reshape_capi(knew, vnew, slot, kc, vc)
    out_a = attention_capi(q, kc, vc, ones, kv, btd, max_q=1, max_k=int(ctx.max()) + 1)
    out_b = torch.zeros_like(q)
    descs = (capi.Desc(capi.DATA_INT32, bt.shape), capi.Desc(capi.DATA_BFLOAT16, q.shape),
             capi.Desc(capi.DATA_BFLOAT16, kc.shape))
    capi.check(capi.reshape_and_cache_flash_attention_decode(
        handle(), knew.data_ptr(), vnew.data_ptr(), slot.data_ptr(), int(ctx.max()) + 1,
        ones.data_ptr(), kv.data_ptr(), descs[0], btd.data_ptr(), descs[1], q.data_ptr(),
        descs[2], kc_b.data_ptr(), descs[2], vc_b.data_ptr(), descs[1], out_b.data_ptr()),
        "fused decode")
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)
    assert torch.equal(kc, kc_b) and torch.equal(vc, vc_b)
