"""Parity cases and their deterministic inputs.

Shapes follow the reference's own test cases:
* reshape: test/zoo/teco/reshape_and_cache/test_case/case_{0,1,2}.prototxt
  (512 tokens, H 8/4/2, D 128, 64 pages x 16, slot_mapping overwritten with
  0..T-1 as reshape_and_cache.cpp:77-84 does, caches zeroed) and
  python_api_test/test_reshape_and_cache.py:70-75 (same shapes), plus
  the CPU-runnable fp16 pair (random permutation slots with ~5% -1 padding, caches
  pre-filled with a sentinel so untouched slots are checked too) and edge cases.
* attention: test/zoo/teco/flash_attention/test_case/{0..5}.prototxt (block_size
  32, U(-1, 1) inputs, block tables drawn uniformly from [0, 255] — duplicates
  allowed), python_api_test/test_flash_attention.py:265-358 (prefill, decode,
  chunked, GQA, mixed; N(0, 1) inputs, 64-page pool, shuffled block tables),
  that pair's prefill and block_size-16 / bf16 / head_dim-64 variants.

Inputs are regenerated bit-identically from (seed, shape) by oracle.seeded.
"""
from __future__ import annotations

import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from oracle import seeded  # noqa: E402


def _cdiv(a, b):
    return (a + b - 1) // b


# ---------------------------------------------------------------- reshape_and_cache
RESHAPE_CASES = {
    # zoo case_0..2 / python_api_test CONFIGS
    "zoo_case0": dict(T=512, H=8, D=128, NB=64, bs=16, dtype="f16", slots="arange", pad=0.0,
                      init="zeros", seed=101),
    "zoo_case1": dict(T=512, H=4, D=128, NB=64, bs=16, dtype="f16", slots="arange", pad=0.0,
                      init="zeros", seed=102),
    "zoo_case2": dict(T=512, H=2, D=128, NB=64, bs=16, dtype="f16", slots="arange", pad=0.0,
                      init="zeros", seed=103),
    # CPU-runnable fp16 pair: randperm(1024)[:256] slots, ~5% -1
    "cfg1_fp16": dict(T=256, H=8, D=128, NB=64, bs=16, dtype="f16", slots="perm", pad=0.05,
                      init="sentinel", seed=1),
    "cfg1_bf16": dict(T=256, H=8, D=128, NB=64, bs=16, dtype="bf16", slots="perm", pad=0.05,
                      init="sentinel", seed=2),
    # edges: a single token, ragged head_dim, heavy padding, block_size 32
    "one_token": dict(T=1, H=8, D=128, NB=4, bs=16, dtype="bf16", slots="perm", pad=0.0,
                      init="sentinel", seed=3),
    "d64_bs32_pad10": dict(T=300, H=4, D=64, NB=32, bs=32, dtype="f16", slots="perm", pad=0.10,
                           init="sentinel", seed=4),
    "d72_unaligned": dict(T=77, H=3, D=72, NB=16, bs=8, dtype="bf16", slots="perm", pad=0.10,
                          init="sentinel", seed=5),
    "all_padding": dict(T=64, H=2, D=128, NB=8, bs=16, dtype="f16", slots="perm", pad=1.0,
                        init="sentinel", seed=6),
}


def reshape_inputs(c):
    """Returns (key, value, slot_mapping, key_cache, value_cache) as uint16 words / int64."""
    T, H, D, NB, bs = c["T"], c["H"], c["D"], c["NB"], c["bs"]
    s = c["seed"]
    key = seeded.to_words(seeded.normal(s * 10 + 1, (T, H, D)), c["dtype"])
    value = seeded.to_words(seeded.normal(s * 10 + 2, (T, H, D)), c["dtype"])
    if c["slots"] == "arange":
        slot = np.arange(T, dtype=np.int64)
    else:
        slot = seeded.permutation(s * 10 + 3, NB * bs)[:T].astype(np.int64)
    if c["pad"] > 0:
        drop = seeded.uniform(s * 10 + 4, (T,), 0.0, 1.0) < c["pad"]
        if c["pad"] >= 1.0:
            drop[:] = True
        slot[drop] = -1
    if c["init"] == "zeros":
        kc = np.zeros((NB, H, bs, D), dtype=np.uint16)
        vc = np.zeros((NB, H, bs, D), dtype=np.uint16)
    else:
        kc = seeded.to_words(seeded.uniform(s * 10 + 5, (NB, H, bs, D), -7.0, 7.0), c["dtype"])
        vc = seeded.to_words(seeded.uniform(s * 10 + 6, (NB, H, bs, D), -7.0, 7.0), c["dtype"])
    return key, value, slot, kc, vc


# ---------------------------------------------------------------- flash_attention
def _fa(q_lens, kv_lens, Hq, Hkv, D, bs, NB, dtype, dist, seed, bt="perm", opts=None,
        golden=True):
    c = dict(q_lens=list(q_lens), kv_lens=list(kv_lens), Hq=Hq, Hkv=Hkv, D=D, bs=bs, NB=NB,
             dtype=dtype, dist=dist, seed=seed, bt=bt)
    if opts:
        c["opts"] = dict(opts)
    if not golden:
        c["golden"] = False
    return c


ATTN_CASES = {
    # zoo flash_attention test_case 0..5 (bs 32, U(-1,1), bt ~ U[0,255])
    "zoo0": _fa([256], [256], 32, 8, 128, 32, 8, "f16", "uniform", 10, bt="zoo"),
    "zoo1": _fa([1, 256, 128], [511, 257, 511], 32, 8, 128, 32, 256, "f16", "uniform", 11, "zoo"),
    "zoo2": _fa([1, 256, 128], [512, 256, 512], 16, 2, 128, 32, 256, "f16", "uniform", 12, "zoo"),
    "zoo3": _fa([1, 256, 128], [512, 256, 512], 16, 4, 128, 32, 256, "f16", "uniform", 13, "zoo"),
    "zoo4": _fa([1, 256, 128], [512, 256, 512], 16, 8, 64, 32, 256, "f16", "uniform", 14, "zoo"),
    # zoo case 5 uses a 35,845-page pool; the pool here is 2,048 pages (same sequence shape)
    "zoo5": _fa([22], [22], 2, 1, 128, 32, 2048, "f16", "uniform", 15, "zoo"),
    # python_api_test cases (bs 32, N(0,1), 64-page pool)
    "api_prefill_1x64": _fa([64], [64], 8, 4, 128, 32, 64, "f16", "normal", 20),
    "api_prefill_1x128": _fa([128], [128], 8, 4, 128, 32, 64, "f16", "normal", 21),
    "api_prefill_2x64_128": _fa([64, 128], [64, 128], 8, 4, 128, 32, 64, "f16", "normal", 22),
    "api_decode_1x128": _fa([1], [128], 8, 4, 128, 32, 64, "f16", "normal", 23),
    "api_decode_1x256": _fa([1], [256], 8, 4, 128, 32, 64, "f16", "normal", 24),
    "api_decode_2x128": _fa([1, 1], [128, 64], 8, 4, 128, 32, 64, "f16", "normal", 25),
    "api_chunked_32x64": _fa([32], [64], 8, 4, 128, 32, 64, "f16", "normal", 26),
    "api_chunked_64x128": _fa([64], [128], 8, 4, 128, 32, 64, "f16", "normal", 27),
    "api_chunked_2b": _fa([32, 16], [64, 32], 8, 4, 128, 32, 64, "f16", "normal", 28),
    "api_gqa_32q8kv_prefill": _fa([64], [64], 32, 8, 128, 32, 64, "f16", "normal", 29),
    "api_gqa_16q4kv_decode": _fa([1], [128], 16, 4, 128, 32, 64, "f16", "normal", 30),
    "api_gqa_8q2kv_chunked": _fa([32], [64], 8, 2, 128, 32, 64, "f16", "normal", 31),
    "api_gqa_2q1kv_decode_2b": _fa([1, 1], [64, 128], 2, 1, 128, 32, 64, "f16", "normal", 32),
    "api_mix_decode_prefill": _fa([1, 32], [128, 64], 8, 4, 128, 32, 64, "f16", "normal", 33),
    # CPU-runnable fp16 pair: causal prefill B 1, L 256, 8/8 heads, bs 16
    "cfg1_prefill": _fa([256], [256], 8, 8, 128, 16, 64, "f16", "normal", 4),
    # block_size 16 / bf16 / ragged variants on the B200 paths
    "bf16_bs16_varlen": _fa([200, 37, 513], [200, 300, 513], 32, 8, 128, 16, 160, "bf16", "normal", 40),
    "bf16_bs16_decode": _fa([1] * 7, [1, 17, 300, 1000, 64, 5, 2047], 32, 8, 128, 16, 400, "bf16",
                            "normal", 41),
    "bf16_d64_bs64": _fa([130, 7], [130, 300], 16, 4, 64, 64, 16, "bf16", "normal", 42),
    "f16_bs8_gqa8": _fa([65], [90], 16, 2, 128, 8, 40, "f16", "normal", 43),
    # decode at head_dim 64 (no reference golden: checked against the oracle only)
    "bf16_decode_d64_bs32": _fa([1] * 5, [1, 33, 300, 1000, 2047], 16, 4, 64, 32, 200, "bf16",
                                "normal", 71, golden=False),
    "bf16_decode_gqa16_bs128": _fa([1, 1, 1], [700, 129, 2000], 16, 1, 128, 128, 40, "bf16",
                                   "normal", 44),
    "f16_generic_d96": _fa([33, 1], [40, 77], 6, 3, 96, 16, 16, "f16", "normal", 45),
    "bf16_generic_bs4": _fa([9], [23], 4, 2, 128, 4, 16, "bf16", "normal", 46),
    # pages larger than a 128-token tile (prefill boxes of 128 rows at a row offset) and
    # head_dim 256 (generic kernel)
    "bf16_bs256_prefill": _fa([300, 77], [700, 77], 16, 4, 128, 256, 12, "bf16", "normal", 49),
    "f16_d256_generic": _fa([20, 1], [45, 90], 4, 2, 256, 16, 16, "f16", "normal", 63),
    # empty sequences inside a batch (q_len 0, and q_len = kv_len = 0); the reference
    # golden raises on q_len 0 < kv_len (its mask shape), so these have no fixture
    "edge_empty_seqs_prefill": _fa([0, 100, 0, 37], [10, 300, 0, 37], 32, 8, 128, 16, 64, "bf16",
                                   "normal", 47, golden=False),
    "edge_empty_seqs_decode": _fa([1, 0, 1, 0], [50, 20, 700, 0], 16, 2, 128, 16, 64, "f16",
                                  "normal", 48, golden=False),
    # options of tecoopsFlashAttentionEx (the binding's softmax_scale / causal /
    # window_size / return_softmax_lse).  "scale" and "causal" are pinned by the
    # reference golden's own arguments; "window" and "lse" have no reference
    # implementation (restated in the oracle, no golden fixture).
    "opt_noncausal_prefill_bf16": _fa([200, 37, 513], [200, 300, 513], 32, 8, 128, 16, 160,
                                      "bf16", "normal", 50, opts=dict(causal=False)),
    "opt_noncausal_generic_f16": _fa([65], [90], 16, 2, 128, 8, 40, "f16", "normal", 51,
                                     opts=dict(causal=False)),
    "opt_scale_prefill_bf16_d64": _fa([130, 7], [130, 300], 16, 4, 64, 64, 16, "bf16", "normal",
                                      52, opts=dict(scale=0.05)),
    "opt_scale_decode_bf16": _fa([1] * 4, [17, 300, 1000, 2047], 32, 8, 128, 16, 400, "bf16",
                                 "normal", 53, opts=dict(scale=0.3)),
    "opt_window_prefill_bf16": _fa([300, 129, 520], [300, 400, 520], 32, 8, 128, 16, 160, "bf16",
                                   "normal", 54, opts=dict(window=(100, 0))),
    "opt_window_rowpairs_f16": _fa([700], [900], 6, 2, 128, 16, 64, "f16", "normal", 55,
                                   opts=dict(window=(250, -1))),
    "opt_window_noncausal_bf16": _fa([256, 64], [256, 200], 8, 2, 128, 16, 64, "bf16", "normal",
                                     56, opts=dict(causal=False, window=(40, 24))),
    "opt_window_decode_bf16": _fa([1] * 5, [1, 17, 300, 1000, 2047], 32, 8, 128, 16, 400, "bf16",
                                  "normal", 57, opts=dict(window=(100, -1))),
    "opt_window700_decode_f16": _fa([1] * 3, [2047, 701, 1500], 8, 1, 128, 32, 200, "f16",
                                    "normal", 58, opts=dict(window=(700, -1))),
    "opt_lse_prefill_bf16": _fa([200, 37, 513], [200, 300, 513], 32, 8, 128, 16, 160, "bf16",
                                "normal", 59, opts=dict(lse=True)),
    "opt_lse_decode_bf16": _fa([1] * 7, [1, 17, 300, 1000, 64, 5, 2047], 32, 8, 128, 16, 400,
                               "bf16", "normal", 60, opts=dict(lse=True)),
    "opt_lse_window_generic_f16": _fa([33, 1], [40, 77], 6, 3, 96, 16, 16, "f16", "normal", 61,
                                      opts=dict(lse=True, window=(10, -1))),
    "opt_all_prefill_f16_d64": _fa([130, 7], [130, 300], 16, 4, 64, 64, 16, "f16", "normal", 62,
                                   opts=dict(scale=0.1, causal=False, window=(50, 20), lse=True)),
}


def attn_opts(c):
    """Oracle keyword arguments of a case's options."""
    o = c.get("opts", {})
    return dict(softmax_scale=o.get("scale"), causal=o.get("causal", True),
                window=tuple(o.get("window", (-1, -1))))


def has_reference_golden(c):
    """The reference golden covers scale and causal but no window, and fails on a
    sequence with q_len 0 < kv_len."""
    return "window" not in c.get("opts", {}) and c.get("golden", True)


def attn_inputs(c):
    """Returns dict with q/k_cache/v_cache (uint16 words), q_lens, kv_lens (int32),
    block_table (int32) for a case spec."""
    ql = np.asarray(c["q_lens"], dtype=np.int32)
    kl = np.asarray(c["kv_lens"], dtype=np.int32)
    B = len(ql)
    Hq, Hkv, D, bs, NB = c["Hq"], c["Hkv"], c["D"], c["bs"], c["NB"]
    s = c["seed"]
    gen = (lambda sd, shp: seeded.uniform(sd, shp, -1.0, 1.0)) if c["dist"] == "uniform" \
        else seeded.normal
    q = seeded.to_words(gen(s * 10 + 1, (int(ql.sum()), Hq, D)), c["dtype"])
    kc = seeded.to_words(gen(s * 10 + 2, (NB, Hkv, bs, D)), c["dtype"])
    vc = seeded.to_words(gen(s * 10 + 3, (NB, Hkv, bs, D)), c["dtype"])
    pages = [_cdiv(int(k), bs) for k in kl]
    width = max(max(pages), 1)
    if c["bt"] == "zoo":
        bt = seeded.randint(s * 10 + 4, (B, width), 0, NB).astype(np.int32)
    else:
        perm = seeded.permutation(s * 10 + 4, NB)
        bt = np.zeros((B, width), dtype=np.int32)
        idx = 0
        for b in range(B):
            for j in range(pages[b]):
                bt[b, j] = perm[idx % NB]
                idx += 1
    return dict(q=q, k_cache=kc, v_cache=vc, q_lens=ql, kv_lens=kl, block_table=bt)


def sample_index(n: int, k: int = 4096, seed: int = 7) -> np.ndarray:
    """Deterministic subset of flat output positions stored in the fixtures."""
    if n <= k:
        return np.arange(n, dtype=np.int64)
    return np.sort(seeded.permutation(seed + n, n)[:k])


# ---------------------------------------------------------------- rms_norm
# zoo test_case 0..7 (64 tokens, U(-1, 1) input / weight / residual) and
# python_api_test/test_rms_norm.py (64 tokens, N(0, 1)), plus the B200 kernel
# variants: bf16, ragged hidden sizes (scalar path), CTA-per-row sizes.
def _rn(N, D, eps, res, dtype="f16", dist="uniform", seed=0):
    return dict(N=N, D=D, eps=eps, res=res, dtype=dtype, dist=dist, seed=seed)


RMS_CASES = {
    "zoo0": _rn(64, 4096, 1e-6, False, seed=200), "zoo1": _rn(64, 4096, 1e-6, True, seed=201),
    "zoo2": _rn(64, 2048, 1e-5, False, seed=202), "zoo3": _rn(64, 2048, 1e-5, True, seed=203),
    "zoo4": _rn(64, 1536, 1e-6, False, seed=204), "zoo5": _rn(64, 1536, 1e-6, True, seed=205),
    "zoo6": _rn(64, 128, 1e-6, False, seed=206), "zoo7": _rn(64, 128, 1e-5, False, seed=207),
    "api_norm_128": _rn(64, 128, 1e-6, False, dist="normal", seed=210),
    "api_add_4096": _rn(64, 4096, 1e-6, True, dist="normal", seed=211),
    "bf16_add_8192": _rn(37, 8192, 1e-5, True, dtype="bf16", dist="normal", seed=212),
    "bf16_norm_16384": _rn(5, 16384, 1e-6, False, dtype="bf16", dist="normal", seed=213),
    "f16_ragged_100": _rn(9, 100, 1e-6, True, dist="normal", seed=214),
    "f16_scalar_20000": _rn(3, 20000, 1e-5, False, dist="normal", seed=215),
    "f16_one_token": _rn(1, 4096, 1e-6, True, dist="normal", seed=216),
}


def rms_inputs(c):
    """(x, w, r or None) as 16-bit words."""
    s = c["seed"]
    gen = (lambda sd, shp: seeded.uniform(sd, shp, -1.0, 1.0)) if c["dist"] == "uniform" \
        else seeded.normal
    x = seeded.to_words(gen(s * 10 + 1, (c["N"], c["D"])), c["dtype"])
    w = seeded.to_words(gen(s * 10 + 2, (c["D"],)), c["dtype"])
    r = seeded.to_words(gen(s * 10 + 3, (c["N"], c["D"])), c["dtype"]) if c["res"] else None
    return x, w, r
