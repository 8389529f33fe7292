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


@pytest.mark.parametrize("name", sorted(cases.ATTN_CASES))
def test_attention_oracle_vs_reference_golden(golden, name):
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    out = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"])
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
