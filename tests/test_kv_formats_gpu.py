"""KV-cache formats beyond the reference (hot-path scope table, next row 3): the vLLM
page layout [NB, bs, H, D] and e4m3 (FP8) caches with per-tensor scales, through
tecoopsReshapeAndCacheEx and tecoopsFlashAttentionEx.

* reshape: bit-exact against the oracle (layout permutation of the reshape oracle;
  oracle.fp8 quantisation for e4m3).
* attention, vLLM layout: bit-identical to the same call on the reference layout
  (same kernels, only the tensor-map strides differ).
* attention, e4m3: north-star tolerance against the fp32 oracle run on the
  dequantised cache."""
import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import fp8, seeded

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _capi_dt(dtype):
    from tecoops import capi
    return capi.DATA_HALF if dtype == "f16" else capi.DATA_BFLOAT16


@pytest.mark.parametrize("name", ["cfg1_bf16", "d64_bs32_pad10", "one_token"])
def test_reshape_vllm_layout_bit_exact(name):
    from gpu_util import dev_to_words, handle, words_to_dev
    from tecoops import capi
    c = cases.RESHAPE_CASES[name]
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    ek, ev = oracle.reshape_and_cache(key, value, slot, kc.copy(), vc.copy())   # [NB,H,bs,D]
    kn = np.ascontiguousarray(kc.transpose(0, 2, 1, 3))                   # [NB, bs, H, D]
    vn = np.ascontiguousarray(vc.transpose(0, 2, 1, 3))
    dk, dv = words_to_dev(kn, c["dtype"]), words_to_dev(vn, c["dtype"])
    T, H, D, NB, bs = c["T"], c["H"], c["D"], c["NB"], c["bs"]
    # keep the device inputs referenced until the kernel has run
    tk, tv = words_to_dev(key, c["dtype"]), words_to_dev(value, c["dtype"])
    ts = torch.from_numpy(slot).cuda()
    capi.check(capi.reshape_and_cache_ex(
        handle(), tk.data_ptr(), tv.data_ptr(), ts.data_ptr(), dk.data_ptr(), dv.data_ptr(), T, H,
        D, NB, bs, _capi_dt(c["dtype"]), kv_layout=capi.KV_LAYOUT_NHD), "reshape_and_cache_ex")
    torch.cuda.synchronize()
    assert np.array_equal(dev_to_words(dk), ek.transpose(0, 2, 1, 3))
    assert np.array_equal(dev_to_words(dv), ev.transpose(0, 2, 1, 3))


def _fp8_expected(key, value, slot, NB, H, bs, D, dtype, ks, vs, layout, init):
    """Reshape oracle for an e4m3 cache: cache[slot] = e4m3(x / scale)."""
    kf = seeded.words_to_f32(key, dtype)
    vf = seeded.words_to_f32(value, dtype)
    ek, ev = init.copy(), init.copy()                                     # [NB, H, bs, D] bytes
    for t, s in enumerate(slot.tolist()):
        if s < 0 or s >= NB * bs:
            continue
        ek[s // bs, :, s % bs, :] = fp8.quantize(kf[t], ks)
        ev[s // bs, :, s % bs, :] = fp8.quantize(vf[t], vs)
    if layout == 1:
        ek, ev = ek.transpose(0, 2, 1, 3), ev.transpose(0, 2, 1, 3)
    return np.ascontiguousarray(ek), np.ascontiguousarray(ev)


@pytest.mark.parametrize("name,layout,ks,vs", [("cfg1_bf16", 0, 0.05, 0.02),
                                                ("cfg1_fp16", 1, 1.0, 0.5),
                                                ("d72_unaligned", 0, 0.01, 0.03),
                                                ("d64_bs32_pad10", 1, 0.004, 0.25)])
def test_reshape_fp8_bit_exact(name, layout, ks, vs):
    """Includes saturation (7 / 0.004 > 448) and the scalar path (head_size 72)."""
    from gpu_util import handle, words_to_dev
    from tecoops import capi
    c = cases.RESHAPE_CASES[name]
    key, value, slot, _, _ = cases.reshape_inputs(c)
    T, H, D, NB, bs = c["T"], c["H"], c["D"], c["NB"], c["bs"]
    init = (np.arange(NB * H * bs * D, dtype=np.int64) * 37 % 251).astype(np.uint8).reshape(
        NB, H, bs, D)
    start = init if layout == 0 else np.ascontiguousarray(init.transpose(0, 2, 1, 3))
    dk = torch.from_numpy(start.copy()).cuda()
    dv = torch.from_numpy(start.copy()).cuda()
    tk, tv = words_to_dev(key, c["dtype"]), words_to_dev(value, c["dtype"])
    ts = torch.from_numpy(slot).cuda()
    capi.check(capi.reshape_and_cache_ex(
        handle(), tk.data_ptr(), tv.data_ptr(), ts.data_ptr(), dk.data_ptr(), dv.data_ptr(), T, H,
        D, NB, bs, _capi_dt(c["dtype"]), kv_layout=layout, cache_dtype=capi.DATA_FLOAT8_E4M3,
        k_scale=ks, v_scale=vs), "reshape_and_cache_ex fp8")
    torch.cuda.synchronize()
    ek, ev = _fp8_expected(key, value, slot, NB, H, bs, D, c["dtype"], ks, vs, layout, init)
    assert np.array_equal(dk.cpu().numpy(), ek)
    assert np.array_equal(dv.cpu().numpy(), ev)


def _attn_ex(q, kc, vc, ql, kl, bt, cache_dt, kv_layout=0, k_scale=1.0, v_scale=1.0, max_q=None,
             **opts):
    from gpu_util import handle
    from tecoops import capi
    dt = capi.DATA_HALF if q.dtype == torch.float16 else capi.DATA_BFLOAT16
    out = torch.zeros_like(q)
    d_bt, d_q, d_c = (capi.Desc(capi.DATA_INT32, bt.shape), capi.Desc(dt, q.shape),
                      capi.Desc(cache_dt, kc.shape))
    mq = int(ql.max().item()) if max_q is None else max_q
    st = capi.flash_attention_ex(handle(), mq, int(kl.max().item()), kc.shape[0], ql.data_ptr(),
                                 kl.data_ptr(), d_bt, bt.data_ptr(), d_q, q.data_ptr(), d_c,
                                 kc.data_ptr(), d_c, vc.data_ptr(), d_q, out.data_ptr(), 0,
                                 kv_layout=kv_layout, k_scale=k_scale, v_scale=v_scale, **opts)
    capi.check(st, "tecoopsFlashAttentionEx")
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("name", ["bf16_bs16_varlen", "bf16_bs16_decode", "f16_generic_d96",
                                  "bf16_d64_bs64", "api_mix_decode_prefill"])
def test_attention_vllm_layout_matches_reference_layout(name):
    from gpu_util import attention_capi, attn_case_to_dev
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    kn = d["kc"].permute(0, 2, 1, 3).contiguous()
    vn = d["vc"].permute(0, 2, 1, 3).contiguous()
    out = _attn_ex(d["q"], kn, vn, d["q_lens"], d["kv_lens"], d["bt"], _capi_dt(c["dtype"]),
                   kv_layout=1)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("name,layout", [("bf16_bs16_decode", 0), ("api_decode_2x128", 1),
                                         ("bf16_decode_gqa16_bs128", 0), ("f16_generic_d96", 0),
                                         ("bf16_bs16_varlen", 1), ("bf16_d64_bs64", 0),
                                         ("bf16_decode_d64_bs32", 0), ("bf16_decode_d64_bs32", 1),
                                         ("opt_window_decode_bf16", 1),
                                         ("opt_window700_decode_f16", 0)])
def test_attention_fp8_cache_vs_oracle(name, layout):
    """e4m3 caches: decode on the split-KV kernel (f16 MMAs on converted tiles),
    prefill on the tcgen05 kernel over a dequantised compact copy, odd shapes on the
    generic kernel."""
    from gpu_util import errors, words_to_dev
    from tecoops import capi
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    ks, vs = 1.0 / 64, 1.0 / 32
    kq = fp8.quantize(seeded.words_to_f32(inp["k_cache"], c["dtype"]), ks)   # [NB, H, bs, D]
    vq = fp8.quantize(seeded.words_to_f32(inp["v_cache"], c["dtype"]), vs)
    if layout == 1:
        kd = torch.from_numpy(np.ascontiguousarray(kq.transpose(0, 2, 1, 3))).cuda()
        vd = torch.from_numpy(np.ascontiguousarray(vq.transpose(0, 2, 1, 3))).cuda()
    else:
        kd, vd = torch.from_numpy(kq).cuda(), torch.from_numpy(vq).cuda()
    q = words_to_dev(inp["q"], c["dtype"])
    oo = cases.attn_opts(c)
    out = _attn_ex(q, kd, vd, torch.from_numpy(inp["q_lens"]).cuda(),
                   torch.from_numpy(inp["kv_lens"]).cuda(),
                   torch.from_numpy(inp["block_table"]).cuda(), capi.DATA_FLOAT8_E4M3,
                   kv_layout=layout, k_scale=ks, v_scale=vs,
                   softmax_scale=oo["softmax_scale"] or 0.0, causal=oo["causal"],
                   window=oo["window"])
    ref = oracle.flash_attn_varlen(seeded.words_to_f32(inp["q"], c["dtype"]),
                                   fp8.dequantize(kq, ks), fp8.dequantize(vq, vs),
                                   inp["q_lens"], inp["kv_lens"], inp["block_table"], **oo)
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    mx, mean, diff1 = errors(o, ref)
    assert mx <= 2e-2 and mean <= 2e-3 and diff1 <= 1e-2, (mx, mean, diff1)


def test_fp8_vllm_decode_step_round_trip():
    """A config-3-shaped step on an e4m3 vLLM-layout cache: reshape_ex of the new
    tokens, then decode, against the oracle on the dequantised cache."""
    from gpu_util import errors, handle
    from tecoops import capi
    B, Hq, Hkv, D, bs, pool = 16, 32, 8, 128, 16, 4096
    ks, vs = 1.0 / 64, 1.0 / 32
    ctx = torch.randint(100, 3000, (B,), generator=torch.Generator().manual_seed(5))
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(6)).to(torch.int32)
    pages = ((ctx + 1 + bs - 1) // bs).tolist()
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    g = torch.Generator(device="cuda").manual_seed(7)
    base = torch.randn(pool, bs, Hkv, D, device="cuda", generator=g)
    kc = (base / ks).to(torch.float8_e4m3fn).view(torch.uint8)
    vc = (torch.randn(pool, bs, Hkv, D, device="cuda", generator=g) / vs).to(
        torch.float8_e4m3fn).view(torch.uint8)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16, generator=g)
    kn = torch.randn(B, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    vn = torch.randn(B, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    slot = torch.tensor([int(bt[b, int(ctx[b]) // bs]) * bs + int(ctx[b]) % bs for b in range(B)],
                        dtype=torch.int64, device="cuda")
    capi.check(capi.reshape_and_cache_ex(
        handle(), kn.data_ptr(), vn.data_ptr(), slot.data_ptr(), kc.data_ptr(), vc.data_ptr(), B,
        Hkv, D, pool, bs, capi.DATA_BFLOAT16, kv_layout=1, cache_dtype=capi.DATA_FLOAT8_E4M3,
        k_scale=ks, v_scale=vs), "reshape fp8")
    kv = (ctx + 1).to(torch.int32).cuda()
    out = _attn_ex(q, kc, vc, torch.ones(B, dtype=torch.int32, device="cuda"), kv, bt.cuda(),
                   capi.DATA_FLOAT8_E4M3, kv_layout=1, k_scale=ks, v_scale=vs, max_q=1)
    khnd = fp8.dequantize(kc.cpu().numpy(), ks).transpose(0, 2, 1, 3)
    vhnd = fp8.dequantize(vc.cpu().numpy(), vs).transpose(0, 2, 1, 3)
    ref = oracle.flash_attn_varlen(q.float().cpu().numpy(), khnd, vhnd, [1] * B,
                                   (ctx + 1).tolist(), bt.numpy())
    mx, mean, diff1 = errors(out.float().cpu().numpy(), ref)
    assert mx <= 2e-2 and mean <= 2e-3 and diff1 <= 1e-2, (mx, mean, diff1)


def test_fp8_prefill_config2_full_size():
    """Llama-3-8B varlen prefill shapes on an e4m3 cache (scale 1/64) through the tcgen05
    prefill: tolerance against the oracle on the dequantised cache."""
    from gpu_util import errors
    from tecoops import capi
    lens = torch.randint(512, 2049, (4,), generator=torch.Generator().manual_seed(10)).tolist()
    Hq, Hkv, D, bs, ks, vs = 32, 8, 128, 16, 1.0 / 64, 1.0 / 64
    pages = [(l + bs - 1) // bs for l in lens]
    NB = sum(pages)
    bt = torch.zeros(4, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(4):
        bt[b, :pages[b]] = torch.arange(p0, p0 + pages[b], dtype=torch.int32)
        p0 += pages[b]
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn(sum(lens), Hq, D, device="cuda", dtype=torch.bfloat16, generator=g)
    kc = (torch.randn(NB, Hkv, bs, D, device="cuda", generator=g) / ks).to(
        torch.float8_e4m3fn).view(torch.uint8)
    vc = (torch.randn(NB, Hkv, bs, D, device="cuda", generator=g) / vs).to(
        torch.float8_e4m3fn).view(torch.uint8)
    ql = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = _attn_ex(q, kc, vc, ql, ql, bt.cuda(), capi.DATA_FLOAT8_E4M3, k_scale=ks, v_scale=vs)
    ref = oracle.flash_attn_varlen(q.float().cpu().numpy(), fp8.dequantize(kc.cpu().numpy(), ks),
                                   fp8.dequantize(vc.cpu().numpy(), vs), lens, lens, bt.numpy())
    mx, mean, diff1 = errors(out.float().cpu().numpy(), ref)
    assert mx <= 2e-2 and mean <= 2e-3 and diff1 <= 1e-2, (mx, mean, diff1)


def test_fp8_decode_lse_vs_oracle():
    """The split-KV decode on an e4m3 cache writes the natural-log log-sum-exp of
    every row (split partials merged) next to the output."""
    from gpu_util import errors, words_to_dev
    from tecoops import capi
    c = cases.ATTN_CASES["opt_lse_decode_bf16"]
    inp = cases.attn_inputs(c)
    ks, vs = 1.0 / 64, 1.0 / 32
    kq = fp8.quantize(seeded.words_to_f32(inp["k_cache"], c["dtype"]), ks)
    vq = fp8.quantize(seeded.words_to_f32(inp["v_cache"], c["dtype"]), vs)
    q = words_to_dev(inp["q"], c["dtype"])
    lse = torch.full((c["Hq"], q.shape[0]), float("nan"), device="cuda")
    out = _attn_ex(q, torch.from_numpy(kq).cuda(), torch.from_numpy(vq).cuda(),
                   torch.from_numpy(inp["q_lens"]).cuda(), torch.from_numpy(inp["kv_lens"]).cuda(),
                   torch.from_numpy(inp["block_table"]).cuda(), capi.DATA_FLOAT8_E4M3,
                   k_scale=ks, v_scale=vs, softmax_lse=lse.data_ptr(),
                   softmax_scale=cases.attn_opts(c)["softmax_scale"] or 0.0)
    ref, ref_lse = oracle.flash_attn_varlen(seeded.words_to_f32(inp["q"], c["dtype"]),
                                            fp8.dequantize(kq, ks), fp8.dequantize(vq, vs),
                                            inp["q_lens"], inp["kv_lens"], inp["block_table"],
                                            softmax_scale=cases.attn_opts(c)["softmax_scale"],
                                            return_lse=True)
    mx, mean, _ = errors(out.float().cpu().numpy(), ref)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)
    assert np.allclose(lse.cpu().numpy(), ref_lse, atol=1e-3, rtol=1e-4)
