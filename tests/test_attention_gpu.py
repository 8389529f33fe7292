"""flash_attention on the GPU through the C ABI against the oracle and the
reference golden (fixture samples).  Tolerances (north star): max-abs <= 2e-2
and mean-abs <= 2e-3 against the fp32 golden; the zoo's DIFF1 <= 1e-2 too."""
import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import seeded

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
DIFF1 = 1e-2
LSE_ABS = 2e-3   # log-sum-exp (natural log) of the options cases


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _run_case(c, with_lse=False):
    from gpu_util import attention_capi, attention_ex_capi, attn_case_to_dev
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    lse = None
    if "opts" in c:
        out, lse = attention_ex_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                                     c["opts"])
    else:
        out = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    torch.cuda.synchronize()
    out = out.float().cpu().numpy()
    if with_lse:
        return inp, out, (lse.cpu().numpy() if lse is not None else None)
    return inp, out


@pytest.mark.parametrize("name", sorted(cases.ATTN_CASES))
def test_attention_vs_oracle_and_golden(golden, name):
    from gpu_util import errors
    c = cases.ATTN_CASES[name]
    inp, out, lse = _run_case(c, with_lse=True)
    ref, rlse = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"], return_lse=True, **cases.attn_opts(c))
    assert np.isfinite(out).all()
    mx, mean, diff1 = errors(out, ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS and diff1 <= DIFF1, (mx, mean, diff1)
    if lse is not None:
        fin = np.isfinite(rlse)
        assert np.array_equal(np.isfinite(lse), fin) and not np.isnan(lse).any()
        assert np.abs(lse[fin] - rlse[fin]).max() <= LSE_ABS, np.abs(lse[fin] - rlse[fin]).max()
    if not cases.has_reference_golden(c):
        return   # windowed: the oracle is the only reference
    idx = golden[f"attn/{name}/idx"]
    gmx, gmean, _ = errors(out.reshape(-1)[idx], golden[f"attn/{name}/val"])
    assert gmx <= MAX_ABS and gmean <= MEAN_ABS, (gmx, gmean)


def test_attention_deterministic():
    c = cases.ATTN_CASES["bf16_bs16_varlen"]
    _, a = _run_case(c)
    _, b = _run_case(c)
    assert np.array_equal(a, b)


def _config2_inputs(seed=10):
    """Llama-3-8B varlen prefill: 4 seqs, L ~ U{512..2048}, Hq 32, Hkv 8, D 128, bf16, bs 16,
    contiguous pages, K/V written by reshape_and_cache first."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    lens = torch.randint(512, 2049, (4,), generator=g).tolist()
    return lens


def test_config2_prefill_full_size():
    from gpu_util import attention_capi, errors, reshape_capi
    lens = _config2_inputs()
    Hq, Hkv, D, bs = 32, 8, 128, 16
    tot = sum(lens)
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn(tot, Hq, D, device="cuda", dtype=torch.bfloat16, generator=g)
    k = torch.randn(tot, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn(tot, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    pages = [(l + bs - 1) // bs for l in lens]
    NB = sum(pages)
    bt = torch.zeros(4, max(pages), dtype=torch.int32)
    slot = []
    p0 = 0
    for b, l in enumerate(lens):
        bt[b, :pages[b]] = torch.arange(p0, p0 + pages[b], dtype=torch.int32)
        slot.append(torch.arange(l) + p0 * bs)
        p0 += pages[b]
    slot = torch.cat(slot).cuda()
    kc = torch.zeros(NB, Hkv, bs, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    reshape_capi(k, v, slot, kc, vc)
    ql = torch.tensor(lens, dtype=torch.int32).cuda()
    out = attention_capi(q, kc, vc, ql, ql, bt.cuda())
    torch.cuda.synchronize()
    ref = oracle.flash_attn_varlen(q.float().cpu().numpy(), kc.float().cpu().numpy(),
                                   vc.float().cpu().numpy(), lens, lens, bt.numpy())
    mx, mean, diff1 = errors(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS and diff1 <= DIFF1, (mx, mean, diff1)


def test_config3_decode_full_size():
    """Llama-3-8B paged decode: 64 seqs, context U{512..8192}, 40,000-page pool with a
    random permutation, bs 16, Hq 32, Hkv 8, D 128, bf16."""
    from gpu_util import attention_capi, errors
    B, Hq, Hkv, D, bs, pool = 64, 32, 8, 128, 16, 40000
    g = torch.Generator(device="cpu").manual_seed(20)
    ctx = torch.randint(512, 8193, (B,), generator=g)
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(21)).to(torch.int32)
    pages = ((ctx + bs - 1) // bs).tolist()
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    gd = torch.Generator(device="cuda").manual_seed(22)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    ones = torch.ones(B, dtype=torch.int32, device="cuda")
    out = attention_capi(q, kc, vc, ones, ctx.to(torch.int32).cuda(), bt.cuda(), max_q=1,
                         max_k=int(ctx.max()))
    torch.cuda.synchronize()
    # oracle on a compacted pool (only the pages the block tables use)
    used = torch.unique(bt[bt >= 0]).long()
    remap = torch.full((pool,), -1, dtype=torch.int32)
    remap[used] = torch.arange(used.numel(), dtype=torch.int32)
    kcc = kc[used.cuda()].float().cpu().numpy()
    vcc = vc[used.cuda()].float().cpu().numpy()
    btc = remap[bt.long()].numpy()
    ref = oracle.flash_attn_varlen(q.float().cpu().numpy(), kcc, vcc, [1] * B, ctx.tolist(), btc)
    mx, mean, diff1 = errors(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS and mean <= MEAN_ABS and diff1 <= DIFF1, (mx, mean, diff1)


def test_decode_caller_workspace_matches_handle_scratch():
    from gpu_util import attention_capi, attn_case_to_dev, handle
    from tecoops import capi
    c = cases.ATTN_CASES["bf16_bs16_decode"]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, "bf16")
    a = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    dt = capi.DATA_BFLOAT16
    ws = capi.workspace_size(handle(), 1, int(inp["kv_lens"].max()),
                             capi.Desc(capi.DATA_INT32, d["bt"].shape), capi.Desc(dt, d["q"].shape),
                             capi.Desc(dt, d["kc"].shape))
    buf = torch.empty(max(ws, 16), dtype=torch.uint8, device="cuda")
    b = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                       workspace=buf.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_no_device_errors_recorded():
    from gpu_util import handle
    from tecoops import capi
    st, code = capi.device_error(handle())
    assert st == capi.SUCCESS and code == 0


@pytest.mark.parametrize("name,world", [("bf16_bs16_varlen", 2), ("bf16_bs16_varlen", 4),
                                        ("bf16_bs16_decode", 4)])
def test_kv_head_shards_reassemble(name, world):
    """Each KV-head shard runs the unchanged C API on its own cache tensors (what one
    rank of a multi-GPU job does); concatenated outputs match the unsharded run."""
    from gpu_util import attention_capi, attn_case_to_dev, errors
    from tecoops import sharding
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    full = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"])
    parts = []
    for r in range(world):
        s = sharding.head_shard(c["Hq"], c["Hkv"], world, r)
        parts.append(attention_capi(sharding.shard_tokens(d["q"], s, kv=False),
                                    sharding.shard_cache(d["kc"], s),
                                    sharding.shard_cache(d["vc"], s), d["q_lens"], d["kv_lens"],
                                    d["bt"]))
    torch.cuda.synchronize()
    got = torch.cat(parts, dim=1)
    mx, mean, _ = errors(got.float().cpu().numpy(), full.float().cpu().numpy())
    assert mx <= 2e-2 and mean <= 2e-3


def test_config5_prefill_sampled_rows():
    """Llama-3-70B prefill (Hq 64, Hkv 8, 2 x 8192 causal) at full size; checked on
    KV head 0's Q group for the last 256 rows of each sequence (they attend to all 8192
    keys; the oracle treats them as a chunked prefill of 256 rows over 8192 keys)."""
    from gpu_util import attention_capi, errors, reshape_capi
    Hq, Hkv, D, bs, L = 64, 8, 128, 16, 8192
    g = torch.Generator(device="cuda").manual_seed(40)
    q = torch.randn(2 * L, Hq, D, device="cuda", dtype=torch.bfloat16, generator=g)
    k = torch.randn(2 * L, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn(2 * L, Hkv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    nb = 2 * L // bs
    kc = torch.zeros(nb, Hkv, bs, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    reshape_capi(k, v, torch.arange(2 * L, device="cuda"), kc, vc)
    bt = torch.arange(nb, dtype=torch.int32).view(2, nb // 2)
    lens = torch.tensor([L, L], dtype=torch.int32, device="cuda")
    out = attention_capi(q, kc, vc, lens, lens, bt.cuda())
    torch.cuda.synchronize()
    for b in range(2):
        rows = slice(b * L + L - 256, b * L + L)
        ref = oracle.flash_attn_varlen(q[rows, 0:8].float().cpu().numpy(),
                                       kc[:, 0:1].float().cpu().numpy(),
                                       vc[:, 0:1].float().cpu().numpy(), [256], [L],
                                       bt[b:b + 1].numpy())
        mx, mean, diff1 = errors(out[rows, 0:8].float().cpu().numpy(), ref)
        assert mx <= MAX_ABS and mean <= MEAN_ABS and diff1 <= DIFF1, (b, mx, mean, diff1)


def test_config5_decode_sampled_sequences():
    """Llama-3-70B decode (B 256, ctx U{1024..32768}, Hq 64, Hkv 8) at full size on a
    270k-page pool; 16 sequences checked against the oracle on a compacted pool."""
    from gpu_util import attention_capi, errors
    B, Hq, Hkv, D, bs = 256, 64, 8, 128, 16
    ctx = torch.randint(1024, 32769, (B,), generator=torch.Generator().manual_seed(41))
    pages = ((ctx + bs - 1) // bs).tolist()
    pool = sum(pages) + 1024
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(42)).to(torch.int32)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    p0 = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[p0:p0 + pages[b]]
        p0 += pages[b]
    gd = torch.Generator(device="cuda").manual_seed(43)
    kc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    vc = torch.randn(pool, Hkv, bs, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16, generator=gd)
    out = attention_capi(q, kc, vc, torch.ones(B, dtype=torch.int32, device="cuda"),
                         ctx.to(torch.int32).cuda(), bt.cuda(), max_q=1, max_k=int(ctx.max()))
    torch.cuda.synchronize()
    sample = torch.randperm(B, generator=torch.Generator().manual_seed(44))[:16].tolist()
    for b in sample:
        ids = bt[b, :pages[b]].long()
        ref = oracle.flash_attn_varlen(q[b:b + 1].float().cpu().numpy(),
                                       kc[ids.cuda()].float().cpu().numpy(),
                                       vc[ids.cuda()].float().cpu().numpy(), [1], [int(ctx[b])],
                                       np.arange(pages[b], dtype=np.int32)[None])
        mx, mean, diff1 = errors(out[b:b + 1].float().cpu().numpy(), ref)
        assert mx <= MAX_ABS and mean <= MEAN_ABS and diff1 <= DIFF1, (b, mx, mean, diff1)


@pytest.mark.parametrize("name", ["bf16_bs16_varlen", "bf16_bs16_decode"])
@pytest.mark.parametrize("offset_elems", [0, 8, 16, 1])
def test_output_alignment_paths(name, offset_elems):
    """The prefill epilogue writes whole 32-row warp tiles by TMA store when `out` is
    16-byte aligned and falls back to row stores otherwise (and for partial warp tiles);
    a q or out that is only element-aligned (a view at an odd element offset) takes the
    generic kernel, whose accesses are scalar.  Every alignment must match the aligned
    call (bit-exactly where the same kernel runs, within the attention tolerance on the
    generic kernel), and nothing outside `out` may change.  Offsets in elements: 8 = 16
    bytes (TMA stores, 16-byte row stores), 16 = 32 bytes, 1 = 2 bytes (generic)."""
    from gpu_util import attention_capi, attn_case_to_dev
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    d = attn_case_to_dev(inp, c["dtype"])
    max_q = 1 if "decode" in name else None
    ref = attention_capi(d["q"], d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"],
                         max_q=max_q)
    n = d["q"].numel()
    buf = torch.full((n + offset_elems + 64,), 7.0, device="cuda", dtype=d["q"].dtype)
    out = buf[offset_elems:offset_elems + n].view(d["q"].shape)
    qbuf = torch.empty(n + offset_elems, device="cuda", dtype=d["q"].dtype)
    q = qbuf[offset_elems:].view(d["q"].shape)
    q.copy_(d["q"])
    got = attention_capi(q, d["kc"], d["vc"], d["q_lens"], d["kv_lens"], d["bt"], out=out,
                         max_q=max_q)
    torch.cuda.synchronize()
    if offset_elems % 8 == 0:
        assert torch.equal(got, ref)
    else:
        diff = (got.float() - ref.float()).abs()
        assert diff.max().item() <= MAX_ABS and diff.mean().item() <= MEAN_ABS
    assert (buf[:offset_elems] == 7.0).all() and (buf[offset_elems + n:] == 7.0).all()
