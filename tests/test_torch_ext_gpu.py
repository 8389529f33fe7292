"""The PyTorch binding keeps the reference's Python surface
(api/torch_ext.cpp:208-215, called as in python_api_test/test_flash_attention.py:203-216
and python_api_test/test_reshape_and_cache.py:105-110) and the TORCH_LIBRARY ops."""
import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import seeded

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_reshape_and_cache_binding_matches_golden(golden):
    import hashlib

    import tecoops
    from gpu_util import dev_to_words, words_to_dev
    c = cases.RESHAPE_CASES["cfg1_fp16"]
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    dkc, dvc = words_to_dev(kc, "f16"), words_to_dev(vc, "f16")
    tecoops.reshape_and_cache(words_to_dev(key, "f16"), words_to_dev(value, "f16"),
                              torch.from_numpy(slot).cuda(), dkc, dvc)
    torch.cuda.synchronize()
    assert hashlib.sha256(dev_to_words(dkc).tobytes()).digest() == bytes(golden["rc/cfg1_fp16/sha_k"])
    assert hashlib.sha256(dev_to_words(dvc).tobytes()).digest() == bytes(golden["rc/cfg1_fp16/sha_v"])


@pytest.mark.parametrize("name", ["api_mix_decode_prefill", "api_decode_2x128", "bf16_bs16_varlen"])
def test_flash_attn_varlen_func_reference_signature(name):
    import tecoops
    from gpu_util import attention_capi, attn_case_to_dev, errors
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    ql = inp["q_lens"]
    cu = torch.zeros(len(ql) + 1, dtype=torch.int32)
    cu[1:] = torch.from_numpy(np.cumsum(ql)).to(torch.int32)
    out = torch.empty_like(d["q"])
    tecoops.flash_attn_varlen_func(
        d["q"], d["kc"], d["vc"], int(ql.max()), cu.cuda(), int(inp["kv_lens"].max()),
        torch.Tensor(), d["kv_lens"], 1.0 / np.sqrt(c["D"]), True, torch.Tensor(), d["bt"],
        False, out)
    ref_capi = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    torch.cuda.synchronize()
    assert torch.equal(out, ref_capi)
    ref = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"])
    mx, mean, _ = errors(out.float().cpu().numpy(), ref)
    assert mx <= 2e-2 and mean <= 2e-3


@pytest.mark.parametrize("name", ["opt_window_noncausal_bf16", "opt_lse_decode_bf16",
                                  "opt_all_prefill_f16_d64", "opt_scale_prefill_bf16_d64"])
def test_flash_attn_varlen_func_honours_flags(name):
    """softmax_scale / causal / window_size / return_softmax_lse reach the kernels
    (the reference binding ignores them)."""
    import tecoops
    from gpu_util import attention_ex_capi, attn_case_to_dev, errors
    c = cases.ATTN_CASES[name]
    o = c["opts"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    ql = inp["q_lens"]
    cu = torch.zeros(len(ql) + 1, dtype=torch.int32)
    cu[1:] = torch.from_numpy(np.cumsum(ql)).to(torch.int32)
    win = torch.tensor(o["window"], dtype=torch.int32) if "window" in o else torch.Tensor()
    res = tecoops.flash_attn_varlen_func(
        d["q"], d["kc"], d["vc"], int(ql.max()), cu.cuda(), int(inp["kv_lens"].max()),
        torch.Tensor(), d["kv_lens"], float(o.get("scale") or 0.0), bool(o.get("causal", True)),
        win, d["bt"], bool(o.get("lse", False)), torch.empty_like(d["q"]))
    out, lse = res if o.get("lse") else (res, None)
    ref_out, ref_lse = attention_ex_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"],
                                         d["bt"], o)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    if lse is not None:
        assert torch.equal(lse, ref_lse)
    ref = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"], **cases.attn_opts(c))
    mx, mean, _ = errors(out.float().cpu().numpy(), ref)
    assert mx <= 2e-2 and mean <= 2e-3


def test_torch_library_ops():
    import tecoops  # noqa: F401  (registers torch.ops.tecoops)
    from gpu_util import attention_capi, attn_case_to_dev
    c = cases.ATTN_CASES["api_chunked_2b"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    out = torch.empty_like(d["q"])
    torch.ops.tecoops.flash_attention(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                                      int(inp["q_lens"].max()), int(inp["kv_lens"].max()), out)
    ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    key = torch.randn(8, 2, 64, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(4, 2, 16, 64, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slot = torch.tensor([0, 17, -1, 5, 63, 32, 1, 2], device="cuda")
    torch.ops.tecoops.reshape_and_cache(key, key, slot, kc, vc)
    torch.cuda.synchronize()
    assert torch.equal(kc[1, :, 1], key[1]) and torch.equal(vc[3, :, 15], key[4])


def test_binding_rejects_cpu_tensors():
    import tecoops
    with pytest.raises(RuntimeError):
        tecoops.reshape_and_cache(torch.zeros(1, 1, 8, dtype=torch.half),
                                  torch.zeros(1, 1, 8, dtype=torch.half),
                                  torch.zeros(1, dtype=torch.long),
                                  torch.zeros(1, 1, 16, 8, dtype=torch.half),
                                  torch.zeros(1, 1, 16, 8, dtype=torch.half))


def test_binding_two_streams_concurrently():
    """Prefill and decode launched on two PyTorch streams at once from one thread:
    each (thread, device, stream) gets its own handle, so the split-KV scratch and the
    prefill scheduler's counters are not shared; results equal the serial ones."""
    import tecoops
    from gpu_util import attn_case_to_dev
    outs = {}
    runs = []
    for name in ("bf16_bs16_varlen", "bf16_bs16_decode"):
        c = cases.ATTN_CASES[name]
        inp = cases.attn_inputs(c)
        d = attn_case_to_dev(inp, c["dtype"])
        ql = inp["q_lens"]
        cu = torch.zeros(len(ql) + 1, dtype=torch.int32)
        cu[1:] = torch.from_numpy(np.cumsum(ql)).to(torch.int32)
        args = (d["q"], d["kc"], d["vc"], int(ql.max()), cu.cuda(), int(inp["kv_lens"].max()),
                torch.Tensor(), d["kv_lens"], 0.0, True, torch.Tensor(), d["bt"], False)
        ref = tecoops.flash_attn_varlen_func(*args, torch.empty_like(d["q"]))
        torch.cuda.synchronize()
        runs.append((name, args, ref))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for it in range(5):
        for (name, args, _), st in zip(runs, streams):
            with torch.cuda.stream(st):
                outs[(name, it)] = tecoops.flash_attn_varlen_func(*args, torch.empty_like(args[0]))
    torch.cuda.synchronize()
    for name, _, ref in runs:
        for it in range(5):
            assert torch.equal(outs[(name, it)], ref), (name, it)


def test_host_offsets_and_lengths_are_accepted():
    """cu_seqlens_q / seqused_k given as CPU tensors (the reference binding copies them to
    the host itself): moved to q's device, same result as device tensors."""
    import tecoops
    from gpu_util import attn_case_to_dev
    c = cases.ATTN_CASES["bf16_bs16_varlen"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    ql = inp["q_lens"]
    cu = torch.zeros(len(ql) + 1, dtype=torch.int32)
    cu[1:] = torch.from_numpy(np.cumsum(ql)).to(torch.int32)
    outs = []
    for dev in ("cuda", "cpu"):
        outs.append(tecoops.flash_attn_varlen_func(
            d["q"], d["kc"], d["vc"], int(ql.max()), cu.to(dev), int(inp["kv_lens"].max()),
            torch.Tensor(), d["kv_lens"].to(dev), 0.0, True, torch.Tensor(), d["bt"], False,
            torch.empty_like(d["q"])))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_fused_decode_step_binding():
    """reshape_and_cache_flash_attn_decode (and its torch.ops form) equals
    reshape_and_cache followed by flash_attn_varlen_func, caches and output bit-identical."""
    import tecoops
    from gpu_util import attn_case_to_dev
    c = cases.ATTN_CASES["bf16_bs16_decode"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    B, Hkv, D, bs = len(inp["q_lens"]), c["Hkv"], c["D"], c["bs"]
    g = torch.Generator(device="cuda").manual_seed(77)
    knew = torch.randn(B, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    vnew = torch.randn(B, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    kl = inp["kv_lens"]
    slot = torch.tensor([int(inp["block_table"][b, (int(kl[b]) - 1) // bs]) * bs
                         + (int(kl[b]) - 1) % bs for b in range(B)], device="cuda")
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    kc_a, vc_a = d["kc"].clone(), d["vc"].clone()
    tecoops.reshape_and_cache(knew, vnew, slot, kc_a, vc_a)
    ref = tecoops.flash_attn_varlen_func(d["q"], kc_a, vc_a, 1, cu, int(kl.max()), torch.Tensor(),
                                         d["kv_lens"], 0.0, True, torch.Tensor(), d["bt"], False,
                                         torch.empty_like(d["q"]))
    kc_b, vc_b = d["kc"].clone(), d["vc"].clone()
    out_b = tecoops.reshape_and_cache_flash_attn_decode(d["q"], knew, vnew, kc_b, vc_b, slot,
                                                        d["kv_lens"], d["bt"], int(kl.max()),
                                                        torch.empty_like(d["q"]))
    kc_c, vc_c = d["kc"].clone(), d["vc"].clone()
    out_c = torch.empty_like(d["q"])
    torch.ops.tecoops.reshape_and_cache_flash_attention_decode(
        d["q"], knew, vnew, kc_c, vc_c, slot, d["kv_lens"], d["bt"], int(kl.max()), out_c)
    torch.cuda.synchronize()
    for kc, vc, out in ((kc_b, vc_b, out_b), (kc_c, vc_c, out_c)):
        assert torch.equal(kc, kc_a) and torch.equal(vc, vc_a) and torch.equal(out, ref)
