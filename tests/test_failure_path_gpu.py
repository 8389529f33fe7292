"""The give-up path of the bounded device waits, exercised without a GPU fault.

The reference never checks kernel errors (teco/ual/ops/base_op.hpp:41-45 launches
and returns).  Here every mbarrier wait of the split-KV decode kernel is bounded:
when a wait runs out, the kernel records the wait's site in the handle's error
word, the other warps see the CTA's abort flag, the producer waits (bounded) for
its copies still in flight, and the kernel returns.  The host reads the site with
tecoopsGetDeviceErrorStatus.

tecoopsSetDeviceWaitLimit makes the first ring wait of each consumer warp wait on
a barrier that nothing completes, with a 1 ms limit: a flag that nothing sets.
The producer's wait for the ring stage that consumer holds then runs out as well;
the first wait to give up records its site.
Nothing faults, traps or waits without a bound, and the decode kernel holds no
TMEM.  The test then checks that the next normal call on the same handle is
correct, and that caller errors the kernel detects (kv_len above max_seqlen_k,
q_len above 1) are reported through the same word.
"""
import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import seeded

pytestmark = pytest.mark.gpu

PRODUCER_WAIT_SITE = 0x1100   # 0x11nn: the producer's wait for a free ring stage
CONSUMER_WAIT_SITE = 0x1200   # 0x12nn: a consumer's wait for a loaded chunk
KV_BEYOND_PLAN = 0x1300
Q_LEN_ABOVE_ONE = 0x1400


def _decode_case():
    from gpu_util import attn_case_to_dev
    c = cases.ATTN_CASES["bf16_bs16_decode"]
    inp = cases.attn_inputs(c)
    return c, inp, attn_case_to_dev(inp, c["dtype"])


def _oracle(inp, dtype):
    return oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], dtype), seeded.words_to_f32(inp["k_cache"], dtype),
        seeded.words_to_f32(inp["v_cache"], dtype), inp["q_lens"], inp["kv_lens"],
        inp["block_table"])


def test_decode_wait_gives_up_and_reports_its_site():
    from gpu_util import attention_capi, errors
    from tecoops import capi
    c, inp, d = _decode_case()
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    try:
        capi.check(capi.set_device_wait_limit(h, 1_000_000, stall_test=True), "wait limit")
        attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"], max_q=1,
                       h=h)
        st, code = capi.device_error(h)   # synchronises: the kernel has returned
        assert st == capi.INTERNAL_ERROR
        # the stalled consumer's wait runs out, and so may the producer's wait for the
        # ring stage that consumer holds: whichever gives up first records its site
        assert code & 0xff00 in (CONSUMER_WAIT_SITE, PRODUCER_WAIT_SITE), hex(code)
        st, code = capi.device_error(h)   # reading the word cleared it
        assert st == capi.SUCCESS and code == 0
        # back to normal operation on the same handle: a correct result, no error
        capi.check(capi.set_device_wait_limit(h, 2_000_000_000, stall_test=False), "reset")
        out = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                             max_q=1, h=h)
        st, code = capi.device_error(h)
        assert st == capi.SUCCESS and code == 0
        mx, mean, _ = errors(out.float().cpu().numpy(), _oracle(inp, c["dtype"]))
        assert mx <= 2e-2 and mean <= 2e-3
    finally:
        h.close()


def test_wait_limit_rejects_zero():
    from tecoops import capi
    h = capi.Handle()
    try:
        assert capi.set_device_wait_limit(h, 0) == capi.BAD_PARAM
    finally:
        h.close()


def _long_decode(B=4, S=4000, Hq=8, Hkv=2, D=128, bs=16, seed=71):
    g = torch.Generator().manual_seed(seed)
    pages = (S + bs - 1) // bs
    pool = B * pages + 8
    perm = torch.randperm(pool, generator=g)[:B * pages].to(torch.int32).view(B, pages)
    gd = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    return dict(q=q, kc=kc, vc=vc, bt=perm.cuda(), S=S,
                q_lens=torch.ones(B, dtype=torch.int32, device="cuda"),
                kv_lens=torch.full((B,), S, dtype=torch.int32, device="cuda"))


def test_kv_len_above_max_seqlen_k_is_reported():
    """kv_len one split beyond the plan made from max_seqlen_k: the keys past the
    planned splits are not attended (the split scratch holds only the planned
    records), and the error word says so instead of a silent wrong result."""
    from gpu_util import attention_capi
    from tecoops import capi
    d = _long_decode()
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    try:
        # max_seqlen_k 1600 plans splits of >= 1536 tokens and a 2-split scratch; the
        # 4000-token sequences need 3
        out = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                             max_q=1, max_k=1600, h=h)
        st, code = capi.device_error(h)
        assert st == capi.INTERNAL_ERROR and code == KV_BEYOND_PLAN, hex(code)
        assert torch.isfinite(out.float()).all()
        # with the true maximum the same call is clean
        attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"], max_q=1,
                       max_k=d["S"], h=h)
        assert capi.device_error(h) == (capi.SUCCESS, 0)
    finally:
        h.close()


def test_q_len_above_one_on_the_decode_path_is_reported():
    from gpu_util import attention_capi
    from tecoops import capi
    d = _long_decode(B=2, S=300)
    q_lens = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
    q = torch.randn(3, 8, 128, device="cuda", dtype=torch.bfloat16)
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    try:
        # max_seqlen_q = 1 sends the call to the decode kernel although sequence 1 has
        # two query rows
        attention_capi(q, d["kc"], d["vc"], q_lens, d["kv_lens"], d["bt"], max_q=1,
                       max_k=d["S"], h=h)
        st, code = capi.device_error(h)
        assert st == capi.INTERNAL_ERROR and code == Q_LEN_ABOVE_ONE, hex(code)
    finally:
        h.close()


def test_q_len_above_max_seqlen_q_on_the_prefill_path_is_reported():
    """The prefill's work units are planned from max_seqlen_q: a sequence longer than that
    has rows past the plan, which are not computed; the scheduler reports it (0xb00)."""
    from gpu_util import attention_capi
    from tecoops import capi
    L, Hq, Hkv, D, bs = 300, 8, 2, 128, 16
    g = torch.Generator(device="cuda").manual_seed(72)
    q = torch.randn(L, Hq, D, device="cuda", dtype=torch.bfloat16, generator=g)
    pages = (L + bs - 1) // bs
    kc = torch.randn(pages, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=g)
    vc = torch.randn_like(kc)
    bt = torch.arange(pages, dtype=torch.int32, device="cuda")[None]
    lens = torch.tensor([L], dtype=torch.int32, device="cuda")
    h = capi.Handle(torch.cuda.current_stream().cuda_stream)
    try:
        attention_capi(q, kc, vc, lens, lens, bt, max_q=200, max_k=L, h=h)   # plans 256 rows
        st, code = capi.device_error(h)
        assert st == capi.INTERNAL_ERROR and code == 0xb00, hex(code)
        attention_capi(q, kc, vc, lens, lens, bt, max_q=L, max_k=L, h=h)
        assert capi.device_error(h) == (capi.SUCCESS, 0)
    finally:
        h.close()
