"""Seeded random sweep of the attention entry point against the CPU oracle.

The hand-picked parity cases follow the reference's tests; this sweep adds shapes
nobody picked: 1-6 sequences, query lengths 0..300 with kv lengths >= them (chunked
prefill, empty sequences, kv lengths that end anywhere in a page or tile), GQA groups 1,
2, 3, 4, 8, head_dim 64 / 128, block sizes 8..256, fp16 / bf16, shuffled page pools
with spare pages, and decode calls (every q_len 0 or 1) through the split-KV branch; then
the same shapes with random tecoopsFlashAttentionEx options and random cache formats;
random reshape_and_cache cases, bit-exact; random rms_norm cases; and random fused decode
steps against the two operators.
Every case must meet the north-star tolerance (max-abs <= 2e-2, mean-abs <= 2e-3)."""
import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import seeded

pytestmark = pytest.mark.gpu


def _case(i):
    rng = np.random.default_rng(9000 + i)
    decode = i % 4 == 3
    B = int(rng.integers(1, 7))
    Hkv = int(rng.choice([1, 2, 4]))
    group = int(rng.choice([1, 2, 3, 4, 8]))
    D = int(rng.choice([64, 128]))
    bs = int(rng.choice([8, 16, 32, 64, 128, 256]))
    kv = [int(rng.integers(1, 600)) for _ in range(B)]
    if decode:
        q = [int(rng.integers(0, 2)) for _ in range(B)]
        q[0] = 1
    else:
        q = [int(min(k, rng.integers(0, 301))) for k in kv]
        q[0] = max(q[0], 1)
    pages = sum((k + bs - 1) // bs for k in kv)
    return cases._fa(q, kv, Hkv * group, Hkv, D, bs, pages + int(rng.integers(0, 9)),
                     str(rng.choice(["f16", "bf16"])), "normal", 500 + i, golden=False)


@pytest.mark.parametrize("i", range(40))
def test_random_shapes_match_the_oracle(i):
    from gpu_util import attention_capi, attn_case_to_dev, errors
    c = _case(i)
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    out = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                         out=torch.full_like(d["q"], 3.0))
    torch.cuda.synchronize()
    ref = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"])
    got = out.float().cpu().numpy()
    mx, mean, _ = errors(got, ref)
    assert mx <= 2e-2 and mean <= 2e-3, (c, mx, mean)


LSE_ABS = 2e-3   # log-sum-exp (natural log), as in the hand-picked options cases


def _opts(rng):
    o = {"lse": True}
    if rng.random() < 0.3:
        o["causal"] = False
    if rng.random() < 0.4:
        o["scale"] = float(rng.uniform(0.02, 0.4))
    if rng.random() < 0.6:
        left = int(rng.choice([-1, 0, int(rng.integers(1, 400))]))
        right = int(rng.choice([-1, 0, int(rng.integers(1, 200))]))
        o["window"] = (left, right)
    return o


@pytest.mark.parametrize("i", range(24))
def test_random_options_match_the_oracle(i):
    """tecoopsFlashAttentionEx (causal or not, sliding windows, custom scale, the
    log-sum-exp output) on random shapes of the sweep above.  Rows whose window admits
    no key have output 0 and log-sum-exp -inf in both."""
    from gpu_util import attention_ex_capi, attn_case_to_dev, errors
    c = _case(100 + i)
    opts = _opts(np.random.default_rng(7000 + i))
    c["opts"] = opts
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    out, lse = attention_ex_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                                 opts)
    torch.cuda.synchronize()
    ref, rlse = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"], return_lse=True, **cases.attn_opts(c))
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), c
    mx, mean, _ = errors(got, ref)
    assert mx <= 2e-2 and mean <= 2e-3, (c, mx, mean)
    lse = lse.cpu().numpy()
    fin = np.isfinite(rlse)
    assert np.array_equal(np.isfinite(lse), fin) and not np.isnan(lse).any(), c
    if fin.any():
        err = np.abs(lse[fin] - rlse[fin]).max()
        assert err <= LSE_ABS, (c, err)


@pytest.mark.parametrize("i", range(24))
def test_random_cache_formats_match_the_oracle(i):
    """The sweep's shapes on the cache formats beyond the reference: the vLLM page layout
    [NB, bs, Hkv, D] and e4m3 caches with per-tensor scales (tecoopsFlashAttentionEx),
    against the oracle on the dequantised cache (16-bit vLLM layout: bit-identical to the
    reference layout instead)."""
    from gpu_util import attention_capi, attn_case_to_dev, errors, handle, words_to_dev
    from oracle import fp8
    from tecoops import capi
    c = _case(200 + i)
    rng = np.random.default_rng(8000 + i)
    layout = int(rng.integers(0, 2))
    e4m3 = bool(rng.integers(0, 2)) or layout == 0
    inp = cases.attn_inputs(c)
    dt = capi.DATA_HALF if c["dtype"] == "f16" else capi.DATA_BFLOAT16
    q = words_to_dev(inp["q"], c["dtype"])
    ql = torch.from_numpy(inp["q_lens"]).cuda()
    kl = torch.from_numpy(inp["kv_lens"]).cuda()
    bt = torch.from_numpy(inp["block_table"]).cuda()
    perm = (lambda a: np.ascontiguousarray(a.transpose(0, 2, 1, 3))) if layout else (lambda a: a)
    if e4m3:
        ks, vs = float(rng.choice([1 / 64, 1 / 16, 0.5])), float(rng.choice([1 / 32, 0.25]))
        kq = fp8.quantize(seeded.words_to_f32(inp["k_cache"], c["dtype"]), ks)
        vq = fp8.quantize(seeded.words_to_f32(inp["v_cache"], c["dtype"]), vs)
        kd, vd = torch.from_numpy(perm(kq)).cuda(), torch.from_numpy(perm(vq)).cuda()
        cdt = capi.DATA_FLOAT8_E4M3
    else:
        ks = vs = 1.0
        kd = words_to_dev(perm(inp["k_cache"]), c["dtype"])
        vd = words_to_dev(perm(inp["v_cache"]), c["dtype"])
        cdt = dt
    out = torch.full_like(q, 3.0)
    dq, dc = capi.Desc(dt, q.shape), capi.Desc(cdt, kd.shape)
    st = capi.flash_attention_ex(handle(), int(inp["q_lens"].max()), int(inp["kv_lens"].max()),
                                 kd.shape[0], ql.data_ptr(), kl.data_ptr(),
                                 capi.Desc(capi.DATA_INT32, bt.shape), bt.data_ptr(), dq,
                                 q.data_ptr(), dc, kd.data_ptr(), dc, vd.data_ptr(), dq,
                                 out.data_ptr(), 0, kv_layout=layout, k_scale=ks, v_scale=vs)
    capi.check(st, "tecoopsFlashAttentionEx")
    torch.cuda.synchronize()
    if not e4m3:
        d = attn_case_to_dev(inp, c["dtype"])
        ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                             out=torch.full_like(d["q"], 3.0))
        torch.cuda.synchronize()
        assert torch.equal(out, ref), c
        return
    ref = oracle.flash_attn_varlen(seeded.words_to_f32(inp["q"], c["dtype"]),
                                   fp8.dequantize(kq, ks), fp8.dequantize(vq, vs),
                                   inp["q_lens"], inp["kv_lens"], inp["block_table"])
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), c
    mx, mean, _ = errors(got, ref)
    assert mx <= 2e-2 and mean <= 2e-3, (c, layout, ks, vs, mx, mean)


def _reshape_case(i):
    rng = np.random.default_rng(9500 + i)
    bs = int(rng.choice([8, 16, 32, 128]))
    NB = int(rng.integers(4, 200))
    T = int(rng.integers(1, min(NB * bs, 5000) + 1))
    return dict(T=T, H=int(rng.choice([1, 2, 4, 8])), D=int(rng.choice([64, 72, 128, 256])),
                NB=NB, bs=bs, dtype=str(rng.choice(["f16", "bf16"])),
                slots=str(rng.choice(["perm", "arange"])),
                pad=float(rng.choice([0.0, 0.1, 0.5])), init="random", seed=900 + i)


@pytest.mark.parametrize("i", range(24))
def test_random_reshape_is_bit_exact(i):
    """tecoopsReshapeAndCache on random token counts, head counts, head sizes (including a
    non-multiple of 8: the scalar path), block sizes, padding fractions and distinct slots,
    into caches holding earlier data: every word equal to the oracle's, untouched slots
    kept."""
    from gpu_util import dev_to_words, reshape_capi, words_to_dev
    c = _reshape_case(i)
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    ek, ev = oracle.reshape_and_cache(key, value, slot, kc.copy(), vc.copy())
    dk, dv = words_to_dev(kc, c["dtype"]), words_to_dev(vc, c["dtype"])
    reshape_capi(words_to_dev(key, c["dtype"]), words_to_dev(value, c["dtype"]),
                 torch.from_numpy(slot).cuda(), dk, dv)
    torch.cuda.synchronize()
    assert np.array_equal(dev_to_words(dk), ek), c
    assert np.array_equal(dev_to_words(dv), ev), c


@pytest.mark.parametrize("i", range(16))
def test_random_rms_norm_matches_the_oracle(i):
    """rms_norm (with and without the residual add) on random token counts and hidden sizes
    (warp-per-row, CTA-per-row and scalar paths), fp16 / bf16: residual_out bit-exact, the
    output within one step of the 16-bit type of the oracle."""
    from gpu_util import handle, words_to_dev, dev_to_words
    from tecoops import capi
    rng = np.random.default_rng(9700 + i)
    hidden = int(rng.choice([64, 100, 128, 1000, 2048, 2056, 4096, 5120, 8192, 16384]))
    c = cases._rn(int(rng.integers(1, 700)), hidden, float(rng.choice([1e-6, 1e-5])),
                  bool(rng.integers(0, 2)), seed=700 + i, dtype=str(rng.choice(["f16", "bf16"])),
                  dist=str(rng.choice(["uniform", "normal"])))
    x, w, r = cases.rms_inputs(c)
    dx, dw = words_to_dev(x, c["dtype"]), words_to_dev(w, c["dtype"])
    dr = words_to_dev(r, c["dtype"]) if r is not None else None
    out = torch.empty_like(dx)
    ro = torch.empty_like(dx) if r is not None else None
    capi.check(capi.rms_norm(handle(), dx.data_ptr(), dw.data_ptr(),
                             dr.data_ptr() if dr is not None else 0, out.data_ptr(),
                             ro.data_ptr() if ro is not None else 0, c["N"], c["D"], c["eps"],
                             dtype=None if c["dtype"] == "f16" else capi.DATA_BFLOAT16),
               "tecoopsRmsNorm")
    torch.cuda.synchronize()
    ey, ero = oracle.rms_norm(x, w, r, c["eps"], c["dtype"])
    yo = seeded.words_to_f32(dev_to_words(out), c["dtype"])
    ye = seeded.words_to_f32(ey, c["dtype"])
    mant = 10 if c["dtype"] == "f16" else 7
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ye), np.float32(2.0 ** -14)))) - mant)
    assert np.isfinite(yo).all(), c
    assert np.all(np.abs(yo - ye) <= ulp + 1e-7), (c, np.abs(yo - ye).max())
    if r is not None:
        assert np.array_equal(dev_to_words(ro), ero), c


@pytest.mark.parametrize("i", range(16))
def test_random_fused_decode_step_equals_two_operators(i):
    """tecoopsReshapeAndCacheFlashAttentionDecode on random decode shapes (GQA groups
    1-16, head_dim 64 / 128, block sizes 16-128, contexts 1-3,000, padding sequences with
    slot -1): output and caches bit-identical to tecoopsReshapeAndCache followed by
    tecoopsFlashAttention."""
    from gpu_util import attention_capi, handle, reshape_capi
    from tecoops import capi
    rng = np.random.default_rng(9900 + i)
    B = int(rng.integers(1, 40))
    Hkv = int(rng.choice([1, 2, 8]))
    group = int(rng.choice([1, 2, 4, 8, 16]))
    D = int(rng.choice([64, 128]))
    bs = int(rng.choice([16, 32, 64, 128]))
    dt = torch.float16 if rng.integers(0, 2) else torch.bfloat16
    ctx = [int(x) for x in rng.integers(1, 3001, B)]   # kv_len including the new token
    pages = [(c + bs - 1) // bs for c in ctx]
    pool = sum(pages) + int(rng.integers(0, 9))
    perm = torch.from_numpy(rng.permutation(pool).astype(np.int32))
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    g = torch.Generator(device="cuda").manual_seed(9900 + i)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", generator=g).to(dt)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", generator=g).to(dt)
    q = torch.randn(B, Hkv * group, D, device="cuda", generator=g).to(dt)
    kn = torch.randn(B, Hkv, D, device="cuda", generator=g).to(dt)
    vn = torch.randn(B, Hkv, D, device="cuda", generator=g).to(dt)
    slot = [int(bt[b, (ctx[b] - 1) // bs]) * bs + (ctx[b] - 1) % bs for b in range(B)]
    for b in range(B):
        if rng.random() < 0.1:
            slot[b] = -1
    slot = torch.tensor(slot, dtype=torch.int64, device="cuda")
    ones = torch.ones(B, dtype=torch.int32, device="cuda")
    kv = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    btd = bt.cuda()
    kc_a, vc_a = kc.clone(), vc.clone()
    reshape_capi(kn, vn, slot, kc_a, vc_a)
    ref = attention_capi(q, kc_a, vc_a, ones, kv, btd, max_q=1, max_k=max(ctx))
    kc_b, vc_b = kc.clone(), vc.clone()
    out = torch.zeros_like(q)
    cdt = capi.DATA_HALF if dt == torch.float16 else capi.DATA_BFLOAT16
    dq, dc = capi.Desc(cdt, q.shape), capi.Desc(cdt, kc.shape)
    capi.check(capi.reshape_and_cache_flash_attention_decode(
        handle(), kn.data_ptr(), vn.data_ptr(), slot.data_ptr(), max(ctx), ones.data_ptr(),
        kv.data_ptr(), capi.Desc(capi.DATA_INT32, bt.shape), btd.data_ptr(), dq, q.data_ptr(),
        dc, kc_b.data_ptr(), dc, vc_b.data_ptr(), dq, out.data_ptr()), "fused decode")
    torch.cuda.synchronize()
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b), (B, Hkv, group, D, bs)
    # a padding sequence (slot -1) attends its stale cached row in the two-operator form and
    # the new row in the fused one (which takes the new token from the inputs)
    keep = (slot >= 0).cpu()
    assert torch.equal(out[keep], ref[keep]), (B, Hkv, group, D, bs)
