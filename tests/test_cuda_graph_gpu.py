"""A serving loop captures its decode (and prefill) step in a CUDA graph: the torch binding's
reshape_and_cache + flash_attn_varlen_func, captured on a stream that has run the step once
(so that the stream's handle and its lazily allocated scratch exist before capture; the
split-KV partials and the prefill scheduler's counters live there), replays with new inputs
copied into the captured tensors and gives exactly the eager results."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _paged(B, ctx, Hq, Hkv, D, bs, seed):
    g = torch.Generator().manual_seed(seed)
    pages = [(c + bs - 1) // bs for c in ctx]
    pool = sum(pages) + 4
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    gd = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", generator=gd).to(torch.bfloat16)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", generator=gd).to(torch.bfloat16)
    return bt.cuda(), kc, vc


def _capture(step):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()   # warm-up on the capture stream: its handle and scratch are made here
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step()
    return g


def test_decode_step_replays_like_eager():
    import tecoops
    B, Hq, Hkv, D, bs = 8, 32, 8, 128, 16
    ctx = [int(x) for x in np.random.default_rng(5).integers(100, 3000, B)]
    bt, kc, vc = _paged(B, ctx, Hq, Hkv, D, bs, seed=11)
    kv = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    btc = bt.cpu()
    slot = torch.tensor([int(btc[b, (ctx[b] - 1) // bs]) * bs + (ctx[b] - 1) % bs
                         for b in range(B)], device="cuda")
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    q = torch.empty(B, Hq, D, device="cuda", dtype=torch.bfloat16)
    kn = torch.empty(B, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vn = torch.empty_like(kn)
    out = torch.empty_like(q)
    empty = torch.Tensor()

    def step(q=q, kn=kn, vn=vn, kc=kc, vc=vc, out=out):
        tecoops.reshape_and_cache(kn, vn, slot, kc, vc)
        tecoops.flash_attn_varlen_func(q, kc, vc, 1, cu, max(ctx), empty, kv, 0.0, True, empty,
                                       bt, False, out)

    gen = torch.Generator(device="cuda").manual_seed(12)
    for t in (q, kn, vn):
        t.copy_(torch.randn(t.shape, device="cuda", generator=gen))
    g = _capture(step)
    for it in range(3):
        for t in (q, kn, vn):
            t.copy_(torch.randn(t.shape, device="cuda", generator=gen))
        kc_e, vc_e, out_e = kc.clone(), vc.clone(), torch.empty_like(out)
        step(kc=kc_e, vc=vc_e, out=out_e)     # eager, on copies of the caches
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, out_e) and torch.equal(kc, kc_e) and torch.equal(vc, vc_e), it


def test_prefill_step_replays_like_eager():
    import tecoops
    lens = [300, 129, 77]
    B, Hq, Hkv, D, bs = len(lens), 8, 2, 128, 16
    bt, kc, vc = _paged(B, lens, Hq, Hkv, D, bs, seed=21)
    btc = bt.cpu()
    T = sum(lens)
    slot = torch.tensor([int(btc[b, i // bs]) * bs + i % bs for b in range(B)
                         for i in range(lens[b])], device="cuda")
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    kv = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.empty(T, Hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.empty(T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.empty_like(k)
    out = torch.empty_like(q)
    empty = torch.Tensor()

    def step(kc=kc, vc=vc, out=out):
        tecoops.reshape_and_cache(k, v, slot, kc, vc)
        tecoops.flash_attn_varlen_func(q, kc, vc, max(lens), cu, max(lens), empty, kv, 0.0,
                                       True, empty, bt, False, out)

    gen = torch.Generator(device="cuda").manual_seed(22)
    for t in (q, k, v):
        t.copy_(torch.randn(t.shape, device="cuda", generator=gen))
    g = _capture(step)
    for it in range(3):
        for t in (q, k, v):
            t.copy_(torch.randn(t.shape, device="cuda", generator=gen))
        kc_e, vc_e, out_e = kc.clone(), vc.clone(), torch.empty_like(out)
        step(kc=kc_e, vc=vc_e, out=out_e)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, out_e) and torch.equal(kc, kc_e), it
