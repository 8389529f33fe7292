"""Pin the oracle against the reference's own goldens (fixtures made by
tests/golden/make_golden.py from the reference's python goldens)."""
import hashlib
import json

import numpy as np
import pytest

import cases
import oracle
from oracle import seeded


def test_fixture_meta_matches_cases(golden):
    meta = json.loads(bytes(golden["meta"]).decode())
    assert meta["attn"] == json.loads(json.dumps(cases.ATTN_CASES))
    assert meta["rc"] == json.loads(json.dumps(cases.RESHAPE_CASES))
    assert meta["rms"] == json.loads(json.dumps(cases.RMS_CASES))


@pytest.mark.parametrize("name", sorted(cases.ATTN_CASES))
def test_attention_oracle_vs_reference_golden(golden, name):
    c = cases.ATTN_CASES[name]
    if not cases.has_reference_golden(c):
        pytest.skip("no reference golden for this case (window / empty sequence)")
    inp = cases.attn_inputs(c)
    out = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"], **cases.attn_opts(c))
    flat = out.reshape(-1)
    idx = golden[f"attn/{name}/idx"]
    # numpy vs torch fp32 BLAS: only accumulation-order differences
    np.testing.assert_allclose(flat[idx], golden[f"attn/{name}/val"], rtol=0, atol=2e-5)
    s, a = golden[f"attn/{name}/sum"]
    assert abs(flat.astype(np.float64).sum() - s) <= 1e-5 * max(1.0, a)
    assert abs(np.abs(flat.astype(np.float64)).sum() - a) <= 1e-5 * max(1.0, a)


@pytest.mark.parametrize("name", sorted(cases.RESHAPE_CASES))
@pytest.mark.parametrize("impl", ["c", "numpy"])
def test_reshape_oracle_vs_reference_golden(golden, name, impl):
    c = cases.RESHAPE_CASES[name]
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    if impl == "c":
        assert oracle.reshape._lib() is not None, "oracle C library not built"
        oracle.reshape_and_cache(key, value, slot, kc, vc)
    else:
        oracle.reshape_and_cache_np(key, value, slot, kc, vc)
    assert hashlib.sha256(kc.tobytes()).digest() == bytes(golden[f"rc/{name}/sha_k"])
    assert hashlib.sha256(vc.tobytes()).digest() == bytes(golden[f"rc/{name}/sha_v"])


def test_reshape_oracle_threads_agree():
    c = cases.RESHAPE_CASES["cfg1_bf16"]
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    kc2, vc2 = kc.copy(), vc.copy()
    oracle.reshape_and_cache(key, value, slot, kc, vc, threads=1)
    oracle.reshape_and_cache(key, value, slot, kc2, vc2, threads=4)
    assert np.array_equal(kc, kc2) and np.array_equal(vc, vc2)


def test_flop_and_byte_counts():
    # L == S causal: L(L+1)/2 pairs; decode: S pairs
    assert oracle.attention.causal_pairs([4], [4]) == 10
    assert oracle.attention.causal_pairs([1], [100]) == 100
    assert oracle.attention.causal_pairs([2], [5]) == 4 + 5
    assert oracle.attention_flops([256], [256], 8, 128) == 4 * 128 * 8 * 256 * 257 // 2
    assert oracle.reshape_bytes(np.array([0, -1, 3]), 8, 128) == 8 * 3 + 4 * 2 * 8 * 128 * 2


def _small_case(seed=5, L=(40, 9), S=(70, 9), Hq=4, Hkv=2, D=16, bs=8):
    rng = np.random.default_rng(seed)
    NB = sum((s + bs - 1) // bs for s in S)
    q = rng.standard_normal((sum(L), Hq, D)).astype(np.float32)
    kc = rng.standard_normal((NB, Hkv, bs, D)).astype(np.float32)
    vc = rng.standard_normal((NB, Hkv, bs, D)).astype(np.float32)
    bt = np.zeros((len(L), max((s + bs - 1) // bs for s in S)), np.int32)
    p = 0
    for b, s in enumerate(S):
        n = (s + bs - 1) // bs
        bt[b, :n] = np.arange(p, p + n)
        p += n
    return q, kc, vc, list(L), list(S), bt


def _brute(q, kc, vc, L, S, bt, scale, causal, window):
    """Per (row, head) loop: explicit admissible key set, softmax, log-sum-exp."""
    Hq, D = q.shape[1], q.shape[2]
    Hkv, bs = kc.shape[1], kc.shape[2]
    out = np.zeros_like(q, dtype=np.float64)
    lse = np.full((Hq, q.shape[0]), -np.inf)
    r0 = 0
    for b in range(len(L)):
        off = S[b] - L[b]
        for i in range(L[b]):
            for h in range(Hq):
                kv = h // (Hq // Hkv)
                keys = []
                for j in range(S[b]):
                    hi = off + i if causal else (off + i + window[1] if window[1] >= 0 else 1 << 30)
                    lo = off + i - window[0] if window[0] >= 0 else -(1 << 30)
                    if lo <= j <= hi:
                        keys.append(j)
                if not keys:
                    continue
                ks = np.array([kc[bt[b, j // bs], kv, j % bs] for j in keys], np.float64)
                vs = np.array([vc[bt[b, j // bs], kv, j % bs] for j in keys], np.float64)
                x = ks @ q[r0 + i, h].astype(np.float64) * scale
                m = x.max()
                w = np.exp(x - m)
                out[r0 + i, h] = w @ vs / w.sum()
                lse[h, r0 + i] = m + np.log(w.sum())
        r0 += L[b]
    return out, lse


@pytest.mark.parametrize("causal,window", [(True, (-1, -1)), (False, (-1, -1)), (True, (7, -1)),
                                           (False, (5, 3)), (False, (-1, 0)), (True, (0, -1))])
def test_oracle_options_vs_brute_force(causal, window):
    """Window and log-sum-exp (no reference implementation) against a direct
    per-row restatement of their definitions."""
    q, kc, vc, L, S, bt = _small_case()
    out, lse = oracle.flash_attn_varlen(q, kc, vc, L, S, bt, softmax_scale=0.3, causal=causal,
                                        window=window, return_lse=True)
    ref, rlse = _brute(q, kc, vc, L, S, bt, 0.3, causal, window)
    np.testing.assert_allclose(out, ref, atol=2e-5)
    fin = np.isfinite(rlse)
    assert np.array_equal(fin, np.isfinite(lse))
    np.testing.assert_allclose(lse[fin], rlse[fin], atol=2e-5)


def test_oracle_window_properties():
    q, kc, vc, L, S, bt = _small_case(seed=6)
    base = oracle.flash_attn_varlen(q, kc, vc, L, S, bt)
    # a window wider than every sequence changes nothing; non-causal with right 0 is causal
    np.testing.assert_array_equal(
        oracle.flash_attn_varlen(q, kc, vc, L, S, bt, window=(10_000, -1)), base)
    np.testing.assert_array_equal(
        oracle.flash_attn_varlen(q, kc, vc, L, S, bt, causal=False, window=(-1, 0)), base)


def test_fp8_oracle_matches_torch_e4m3():
    """oracle.fp8 (restated OCP E4M3, round-to-nearest-even) against torch's
    float8_e4m3fn conversion on random values, every code point and every tie."""
    import torch
    from oracle import fp8
    rng = np.random.default_rng(0)
    vals = fp8.E4M3_VALUES[:127].astype(np.float32)
    ties = ((fp8.E4M3_VALUES[:126] + fp8.E4M3_VALUES[1:127]) / 2).astype(np.float32)
    x = np.concatenate([rng.standard_normal(100_000).astype(np.float32) * 60, vals, -vals, ties,
                        -ties])
    x = x[np.abs(x) <= 448]
    t = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(fp8.encode(x), t)
    # finite saturation and NaN
    assert fp8.encode(np.array([1e6, -1e6, 449.0], np.float32)).tolist() == [0x7E, 0xFE, 0x7E]
    assert fp8.encode(np.array([np.nan], np.float32))[0] == 0x7F
    codes = np.arange(256, dtype=np.uint8)
    ok = ~np.isnan(fp8.decode(codes))
    assert np.array_equal(fp8.encode(fp8.decode(codes))[ok], codes[ok] & np.where(
        codes[ok] == 0x80, 0xFF, 0xFF).astype(np.uint8))


def _half_ulp(v):
    """Spacing of fp16 at |v| (normal range; 2^-24 in the subnormal range)."""
    a = np.maximum(np.abs(v.astype(np.float32)), np.float32(2.0 ** -14))
    return np.exp2(np.floor(np.log2(a)) - 10)


@pytest.mark.parametrize("name", sorted(cases.RMS_CASES))
def test_rms_norm_oracle_vs_reference_golden(golden, name):
    """The numpy restatement of the zoo golden against the reference's python
    golden: residual_out bit-exact, output within one fp16 step (the python golden
    multiplies the unrounded residual sum; the zoo golden, the kernel and the
    oracle the rounded one; reduction order also differs)."""
    c = cases.RMS_CASES[name]
    if c["dtype"] != "f16":
        pytest.skip("the reference golden is fp16 only")
    x, w, r = cases.rms_inputs(c)
    y, ro = oracle.rms_norm(x, w, r, c["eps"], "f16")
    yf = seeded.words_to_f32(y, "f16").reshape(-1)
    idx = golden[f"rms/{name}/out/idx"]
    g = golden[f"rms/{name}/out/val"]
    assert np.all(np.abs(yf[idx] - g) <= _half_ulp(g) * (2 if r is not None else 1) + 1e-7)
    if r is not None:
        rf = seeded.words_to_f32(ro, "f16").reshape(-1)
        ridx = golden[f"rms/{name}/res_out/idx"]
        assert np.array_equal(rf[ridx], golden[f"rms/{name}/res_out/val"])
