"""KV-head sharding on the GPU, emulated on one device.

The multi-GPU path gives rank r of G its own tensors for KV heads
[r*Hkv/G, (r+1)*Hkv/G) and their Q heads (tecoops.sharding) and runs the unchanged C
API on them, with no collective.  Here every shard of G = 2, 4 and 8 runs on one GPU,
one after another, on separately allocated shard tensors; the outputs, concatenated in
head order (what gather_heads does across ranks), must be bit-identical to the
unsharded call, for the Llama-3-70B head shapes (Hq 64, Hkv 8) in prefill and decode.
The unsharded result itself is checked against the CPU oracle on sampled heads.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

HQ, HKV, D, BS = 64, 8, 128, 16


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _run_shards(G, q, kc, vc, q_lens, kv_lens, bt, max_q, max_k):
    from gpu_util import attention_capi
    from tecoops import sharding
    outs = []
    for r in range(G):
        s = sharding.head_shard(HQ, HKV, G, r)
        outs.append(attention_capi(sharding.shard_tokens(q, s, kv=False),
                                   sharding.shard_cache(kc, s), sharding.shard_cache(vc, s),
                                   q_lens, kv_lens, bt, max_q=max_q, max_k=max_k))
    return torch.cat(outs, dim=1)


def test_prefill_head_shards_reassemble_bit_exactly():
    from gpu_util import attention_capi, errors, reshape_capi
    L = 1536
    g = torch.Generator(device="cuda").manual_seed(60)
    q = torch.randn(2 * L, HQ, D, device="cuda", dtype=torch.bfloat16, generator=g)
    k = torch.randn(2 * L, HKV, D, device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn(2 * L, HKV, D, device="cuda", dtype=torch.bfloat16, generator=g)
    nb = 2 * L // BS
    kc = torch.zeros(nb, HKV, BS, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    reshape_capi(k, v, torch.arange(2 * L, device="cuda"), kc, vc)
    bt = torch.arange(nb, dtype=torch.int32).view(2, -1).cuda()
    lens = torch.tensor([L, L], dtype=torch.int32, device="cuda")
    full = attention_capi(q, kc, vc, lens, lens, bt)
    for G in (2, 4, 8):
        assert torch.equal(_run_shards(G, q, kc, vc, lens, lens, bt, L, L), full), G
    # the unsharded result against the oracle on the Q heads of KV heads 0 and 7
    for kvh in (0, 7):
        hs = slice(kvh * 8, kvh * 8 + 8)
        ref = oracle.flash_attn_varlen(q[:, hs].float().cpu().numpy(),
                                       kc[:, kvh:kvh + 1].float().cpu().numpy(),
                                       vc[:, kvh:kvh + 1].float().cpu().numpy(), [L, L], [L, L],
                                       bt.cpu().numpy())
        mx, mean, _ = errors(full[:, hs].float().cpu().numpy(), ref)
        assert mx <= 2e-2 and mean <= 2e-3, (kvh, mx, mean)


def test_decode_head_shards_reassemble_bit_exactly():
    from gpu_util import attention_capi, errors
    B, pool = 16, 6000
    ctx = torch.randint(1024, 5000, (B,), generator=torch.Generator().manual_seed(61))
    pages = ((ctx + BS - 1) // BS).tolist()
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(62)).to(torch.int32)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    g = torch.Generator(device="cuda").manual_seed(63)
    kc = torch.randn(pool, HKV, BS, D, device="cuda", dtype=torch.bfloat16, generator=g)
    vc = torch.randn(pool, HKV, BS, D, device="cuda", dtype=torch.bfloat16, generator=g)
    q = torch.randn(B, HQ, D, device="cuda", dtype=torch.bfloat16, generator=g)
    ones = torch.ones(B, dtype=torch.int32, device="cuda")
    kv = ctx.to(torch.int32).cuda()
    btd = bt.cuda()
    full = attention_capi(q, kc, vc, ones, kv, btd, max_q=1, max_k=int(ctx.max()))
    for G in (2, 4, 8):
        got = _run_shards(G, q, kc, vc, ones, kv, btd, 1, int(ctx.max()))
        assert torch.equal(got, full), G
    for b in (0, B - 1):
        ids = bt[b, :pages[b]].long()
        ref = oracle.flash_attn_varlen(q[b:b + 1].float().cpu().numpy(),
                                       kc[ids.cuda()].float().cpu().numpy(),
                                       vc[ids.cuda()].float().cpu().numpy(), [1], [int(ctx[b])],
                                       np.arange(pages[b], dtype=np.int32)[None])
        mx, mean, _ = errors(full[b:b + 1].float().cpu().numpy(), ref)
        assert mx <= 2e-2 and mean <= 2e-3, (b, mx, mean)
