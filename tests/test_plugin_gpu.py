"""Plugin Enqueue on the GPU: outputs equal the C API's (the reference's plugin
test only checks the reshape plugin against a CPU loop and runs the attention
plugin as a smoke test, plugin_test/test_plugin_*.py)."""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_reshape_plugin_matches_c_api():
    from gpu_util import reshape_capi, stream_ptr
    from tecoops import plugin
    T, H, D, NB, bs = 300, 8, 128, 32, 16
    key = torch.randn(T, H, D, device="cuda", dtype=torch.float16)
    value = torch.randn(T, H, D, device="cuda", dtype=torch.float16)
    slot = torch.randperm(NB * bs, device="cuda")[:T]
    slot[::7] = -1
    out = torch.full((2 * NB, H, bs, D), 3.0, device="cuda", dtype=torch.float16)
    plugin.enqueue("plugin_reshape_and_cache",
                   {"key": (key.data_ptr(), [T, H, D]), "value": (value.data_ptr(), [T, H, D]),
                    "slot_mapping": (slot.data_ptr(), [T])},
                   [out.data_ptr()], {"num_blocks": NB, "block_size": bs}, stream_ptr())
    kc = torch.zeros(NB, H, bs, D, device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    reshape_capi(key, value, slot, kc, vc)
    torch.cuda.synchronize()
    assert torch.equal(out[:NB], kc) and torch.equal(out[NB:], vc)


@pytest.mark.parametrize("name,dtype_attr", [("api_mix_decode_prefill", 1), ("bf16_bs16_varlen", 9),
                                             ("bf16_bs16_decode", 9)])
def test_flash_plugin_matches_c_api(name, dtype_attr):
    from gpu_util import attention_capi, attn_case_to_dev, stream_ptr
    from tecoops import plugin
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    ql = inp["q_lens"]
    cu = torch.zeros(len(ql) + 1, dtype=torch.int32)
    cu[1:] = torch.from_numpy(np.cumsum(ql)).to(torch.int32)
    cu = cu.cuda()
    out = torch.zeros_like(d["q"])
    attrs = {"max_seqlen_q": int(ql.max()), "max_seqlen_k": int(inp["kv_lens"].max()),
             "max_block_num": d["kc"].shape[0], "dtype": dtype_attr}
    plugin.enqueue("plugin_flash_attention",
                   {"q": (d["q"].data_ptr(), list(d["q"].shape)),
                    "k_cache": (d["kc"].data_ptr(), list(d["kc"].shape)),
                    "v_cache": (d["vc"].data_ptr(), list(d["vc"].shape)),
                    "block_table": (d["bt"].data_ptr(), list(d["bt"].shape)),
                    "cu_seqlens_q": (cu.data_ptr(), [len(ql) + 1]),
                    "seqused_k": (d["kv_lens"].data_ptr(), [len(ql)])},
                   [out.data_ptr()], attrs, stream_ptr())
    ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_flash_plugin_enqueue_does_not_wait_for_the_gpu():
    """An engine keeps one plugin instance per graph node and calls Enqueue on its
    stream every step.  Enqueue must only enqueue: with the stream still busy
    (a ~100 ms device spin queued first) it has to return at once, and two calls in
    a row on the same instance must match the C API."""
    import time

    from gpu_util import attention_capi, attn_case_to_dev, stream_ptr
    from tecoops import plugin
    c = cases.ATTN_CASES["bf16_bs16_varlen"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    ql = inp["q_lens"]
    cu = torch.zeros(len(ql) + 1, dtype=torch.int32)
    cu[1:] = torch.from_numpy(np.cumsum(ql)).to(torch.int32)
    cu = cu.cuda()
    attrs = {"max_seqlen_q": int(ql.max()), "max_seqlen_k": int(inp["kv_lens"].max()),
             "max_block_num": d["kc"].shape[0], "dtype": 9}
    inputs = {"q": (d["q"].data_ptr(), list(d["q"].shape)),
              "k_cache": (d["kc"].data_ptr(), list(d["kc"].shape)),
              "v_cache": (d["vc"].data_ptr(), list(d["vc"].shape)),
              "block_table": (d["bt"].data_ptr(), list(d["bt"].shape)),
              "cu_seqlens_q": (cu.data_ptr(), [len(ql) + 1]),
              "seqused_k": (d["kv_lens"].data_ptr(), [len(ql)])}
    ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    inst = plugin.Instance("plugin_flash_attention")
    try:
        outs = [torch.zeros_like(d["q"]) for _ in range(2)]
        inst.enqueue(inputs, [outs[0].data_ptr()], attrs, stream_ptr())   # first call sets up
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        torch.cuda._sleep(200_000_000)   # keeps the stream busy for ~0.1 s
        t0 = time.perf_counter()
        inst.enqueue(inputs, [outs[1].data_ptr()], attrs, stream_ptr())
        host_s = time.perf_counter() - t0
        busy = not stream.query()
        torch.cuda.synchronize()
        assert busy, "Enqueue returned only after the GPU finished"
        assert host_s < 0.05, host_s
        assert torch.equal(outs[0], ref) and torch.equal(outs[1], ref)
    finally:
        inst.close()
