"""The hot path inside CUDA graphs: a decode step (fused reshape_and_cache + split-KV
attention) and a prefill are captured once and replayed with new inputs written into
the captured buffers; every replay must equal the eager call bit for bit.  The
handle's scratch is allocated by the first (eager) call, before capture; the prefill
scheduler's counters reset themselves at the end of each launch, so replays need
nothing between them."""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _graph(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()   # eager warm-up on the capture stream (allocates the handle's scratch)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    torch.cuda.synchronize()
    return g


def test_decode_step_graph_replay():
    from gpu_util import attn_case_to_dev, handle
    from tecoops import capi
    c = cases.ATTN_CASES["bf16_bs16_decode"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, "bf16")
    B, Hkv, D, bs = len(inp["q_lens"]), c["Hkv"], c["D"], c["bs"]
    kl = inp["kv_lens"]
    slot = torch.tensor([int(inp["block_table"][b, (int(kl[b]) - 1) // bs]) * bs +
                         (int(kl[b]) - 1) % bs for b in range(B)], dtype=torch.int64).cuda()
    knew = torch.zeros(B, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vnew = torch.zeros_like(knew)
    out = torch.zeros_like(d["q"])
    descs = (capi.Desc(capi.DATA_INT32, d["bt"].shape), capi.Desc(capi.DATA_BFLOAT16, d["q"].shape),
             capi.Desc(capi.DATA_BFLOAT16, d["kc"].shape))
    h = capi.Handle()

    def step():
        h.set_stream(torch.cuda.current_stream().cuda_stream)
        capi.check(capi.reshape_and_cache_flash_attention_decode(
            h, knew.data_ptr(), vnew.data_ptr(), slot.data_ptr(), int(kl.max()),
            d["q_lens"].data_ptr(), d["kv_lens"].data_ptr(), descs[0], d["bt"].data_ptr(),
            descs[1], d["q"].data_ptr(), descs[2], d["kc"].data_ptr(), descs[2], d["vc"].data_ptr(),
            descs[1], out.data_ptr()), "fused decode")

    g = _graph(step)
    for it in range(3):
        gen = torch.Generator(device="cuda").manual_seed(100 + it)
        knew.copy_(torch.randn(knew.shape, device="cuda", generator=gen))
        vnew.copy_(torch.randn(vnew.shape, device="cuda", generator=gen))
        d["q"].copy_(torch.randn(d["q"].shape, device="cuda", generator=gen))
        g.replay()
        torch.cuda.synchronize()
        got = out.clone()
        step()   # eager, same inputs (the cache already holds the new tokens)
        torch.cuda.synchronize()
        assert torch.equal(got, out), it
    del h


def test_prefill_graph_replay():
    from gpu_util import attn_case_to_dev
    from tecoops import capi
    c = cases.ATTN_CASES["bf16_bs16_varlen"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, "bf16")
    out = torch.zeros_like(d["q"])
    descs = (capi.Desc(capi.DATA_INT32, d["bt"].shape), capi.Desc(capi.DATA_BFLOAT16, d["q"].shape),
             capi.Desc(capi.DATA_BFLOAT16, d["kc"].shape))
    h = capi.Handle()
    mq, mk = int(inp["q_lens"].max()), int(inp["kv_lens"].max())

    def run():
        h.set_stream(torch.cuda.current_stream().cuda_stream)
        capi.check(capi.flash_attention(h, mq, mk, d["kc"].shape[0], d["q_lens"].data_ptr(),
                                        d["kv_lens"].data_ptr(), descs[0], d["bt"].data_ptr(),
                                        descs[1], d["q"].data_ptr(), descs[2], d["kc"].data_ptr(),
                                        descs[2], d["vc"].data_ptr(), descs[1], out.data_ptr()),
                   "prefill")

    g = _graph(run)
    for it in range(4):
        gen = torch.Generator(device="cuda").manual_seed(200 + it)
        d["q"].copy_(torch.randn(d["q"].shape, device="cuda", generator=gen))
        g.replay()
        torch.cuda.synchronize()
        got = out.clone()
        run()
        torch.cuda.synchronize()
        assert torch.equal(got, out), it
    assert capi.device_error(h)[0] == capi.SUCCESS
    del h
