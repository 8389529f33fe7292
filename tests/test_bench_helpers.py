"""Host-side arithmetic of bench.py (no GPU): the algorithmic FLOP and byte counts the
roofline uses agree with the oracle's, the trimmed mean drops 10 % at each end as the
reference harness does (test/src/suite/executor.cpp:270-276), the headline's head split
covers every head exactly once at N = 1, 2, 4, 8, and the per-head seeding gives the
same values for a head whichever rank holds it (so every N computes the same numbers);
the torch fp32 check used by the bench's verify key matches the oracle."""
import numpy as np
import pytest
import torch

import bench
import oracle


def test_flops_and_bytes_match_the_oracle():
    for q_lens, kv_lens in (([1444, 856, 1888, 1878], [1444, 856, 1888, 1878]),
                            ([1] * 5, [17, 300, 1000, 64, 2047]),
                            ([8192, 8192], [8192, 8192]), ([100, 7], [300, 7])):
        assert bench.causal_pairs(q_lens, kv_lens) == oracle.attention.causal_pairs(q_lens,
                                                                                     kv_lens)
        assert bench.attn_flops(q_lens, kv_lens, hq=64) == oracle.attention_flops(
            q_lens, kv_lens, 64, 128)
        assert bench.attn_bytes(q_lens, kv_lens, hq=32, hkv=8) == oracle.attention_bytes(
            q_lens, kv_lens, 32, 8, 128, 16)
    # the Llama-3-70B headline: 2 x 8192 causal, 64 heads
    assert bench.attn_flops([8192] * 2, [8192] * 2, hq=64) == 2199291691008


def test_trimmed_mean_drops_ten_percent_each_end():
    xs = list(range(1, 21))          # 20 samples: 2 dropped at each end
    assert bench.trimmed_mean(xs) == pytest.approx(sum(range(3, 19)) / 16)
    assert bench.trimmed_mean([5.0, 1.0, 9.0]) == pytest.approx(5.0)   # too few to trim
    assert bench.step_ms([[1.0, 2.0, 30.0] + [2.0] * 7, [1.0] * 10]) == pytest.approx(3.0)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_headline_head_split_covers_every_head_once(world):
    from tecoops import sharding
    q, kv = [], []
    for r in range(world):
        s = sharding.head_shard(64, 8, world, r)
        q += list(range(s.q_begin, s.q_end))
        kv += list(range(s.kv_begin, s.kv_end))
        assert s.q_heads == 64 // world and s.kv_heads == 8 // world
        # a rank's Q heads are exactly its KV heads' GQA groups
        assert s.q_begin == s.kv_begin * 8 and s.q_end == s.kv_end * 8
    assert q == list(range(64)) and kv == list(range(8))


def test_per_head_seeding_is_independent_of_the_split():
    full = bench.per_head_randn(torch, (6, 4), list(range(8)), 123, "cpu", torch.float32)
    for world in (2, 4):
        per = 8 // world
        parts = [bench.per_head_randn(torch, (6, 4), list(range(r * per, (r + 1) * per)), 123,
                                      "cpu", torch.float32) for r in range(world)]
        assert torch.equal(torch.cat(parts, dim=1), full)


def test_verify_reference_matches_the_oracle():
    g = torch.Generator().manual_seed(5)
    S, Hq, Hkv, D = 96, 8, 2, 32
    q = torch.randn(S, Hq, D, generator=g)
    k = torch.randn(S, Hkv, D, generator=g)
    v = torch.randn(S, Hkv, D, generator=g)
    pos = torch.tensor([0, 5, 47, 95])
    got = bench.torch_attention_rows(torch, q[pos], pos, k, v, Hq // Hkv, D ** -0.5)
    # the oracle over the whole sequence (paged with one 96-token page), rows at pos
    ref = oracle.flash_attn_varlen(q.numpy(), k.permute(1, 0, 2).numpy()[None],
                                   v.permute(1, 0, 2).numpy()[None], [S], [S],
                                   np.zeros((1, 1), dtype=np.int32))
    np.testing.assert_allclose(got.numpy(), ref[pos.numpy()], atol=2e-5, rtol=1e-5)


def _fake_prefill_workload(lens, hq, hkv, seed=3):
    """A CPU stand-in for bench.Llama8B with the attributes the CPU baseline reads."""
    import types
    g = torch.Generator().manual_seed(seed)
    W = types.SimpleNamespace(lens=list(lens), tot=sum(lens), HKV=hkv, HQ=hq)
    W.nb = sum(bench.cdiv(n, bench.BS) for n in lens)
    W.q = torch.randn(W.tot, hq, bench.D, generator=g).to(torch.bfloat16)
    W.k = torch.randn(W.tot, hkv, bench.D, generator=g).to(torch.bfloat16)
    W.v = torch.randn(W.tot, hkv, bench.D, generator=g).to(torch.bfloat16)
    bt = torch.zeros(len(lens), max(bench.cdiv(n, bench.BS) for n in lens), dtype=torch.int32)
    slots, p0 = [], 0
    for b, n in enumerate(lens):
        pg = bench.cdiv(n, bench.BS)
        bt[b, :pg] = torch.arange(p0, p0 + pg, dtype=torch.int32)
        slots.append(torch.arange(n) + p0 * bench.BS)
        p0 += pg
    W.bt, W.slot = bt, torch.cat(slots)
    W.flops = bench.attn_flops(lens, lens, hq=hq)
    return W


def test_cpu_baseline_of_the_prefill_runs_the_golden_on_the_same_inputs():
    """bench's in-full CPU baseline (C reshape + the reference golden) on a small batch:
    the GPU output it is compared with is here the oracle's, so the reported difference
    is the golden-vs-oracle one, within the north-star tolerance."""
    golden = bench._golden_or_none()
    if golden is None:
        pytest.skip("reference golden not installed (oracle/install_ref.py)")
    W = _fake_prefill_workload([70, 33], hq=4, hkv=2)
    kc = np.zeros((W.nb, 2, bench.BS, bench.D), np.uint16)
    vc = np.zeros_like(kc)
    oracle.reshape_and_cache(bench._words(W.k), bench._words(W.v), W.slot.numpy(), kc, vc)
    f32 = lambda w: w.view(np.int16).astype(np.int32) << 16   # bf16 words -> fp32 bits
    ref = oracle.flash_attn_varlen(W.q.float().numpy(), f32(kc).view(np.float32),
                                   f32(vc).view(np.float32), W.lens, W.lens, W.bt.numpy())
    W.out = torch.from_numpy(ref).to(torch.bfloat16)
    r = bench.cpu_llama8b_prefill(W, golden)
    assert r["kind"] == "reference" and r["unit"] == "TFLOP/s" and r["value"] > 0
    assert r["gpu_vs_golden"]["max_abs"] <= 2e-2 and r["gpu_vs_golden"]["mean_abs"] <= 2e-3


def test_median_of_runs():
    calls = []
    assert bench._median_s(lambda: calls.append(1), runs=3, warmup=2) >= 0
    assert len(calls) == 5
