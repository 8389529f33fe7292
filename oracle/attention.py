"""ORACLE — test infrastructure only (see oracle/__init__.py).

numpy fp32 restatement of the reference golden ``flash_attn_varlen_func``,
test/zoo/teco/flash_attention/flash_attention.py:79-140 (identical to
python_api_test/test_flash_attention.py:49-110):

* caches arrive in the SDAA layout ``[num_blocks, num_kv_heads, block_size, D]``;
  the golden first permutes them to ``[num_blocks, block_size, Hkv, D]``
  (flash_attention.py:171-173) — done here per gathered page;
* per sequence ``b``: keys/values are gathered through
  ``block_table[b, :cdiv(S, block_size)]`` and truncated to ``S`` (py:101-103);
* bottom-right causal mask ``tril(ones(S, S))[-L:]`` (py:114-116), i.e. row ``i``
  attends keys ``j <= S - L + i``;
* GQA: q head ``h`` uses kv head ``h // (Hq // Hkv)`` (``repeat_interleave``,
  py:125,134);
* ``softmax(Q K^T * scale + bias) V`` in fp32 with scale ``1/sqrt(D)`` (py:127-137).

Options beyond the reference (the flags its Python binding accepts and ignores,
api/torch_ext.cpp:99-113): ``causal=False`` follows the golden's own ``causal``
argument (no mask, py:112-116); ``window=(left, right)`` and the log-sum-exp
output follow flash-attn's published definitions (key j admissible for row i when
``S-L+i-left <= j <= S-L+i+right``, negative sides unbounded; lse = natural-log
log-sum-exp of the scaled, masked scores, ``[Hq, total_q]``).  The reference has
no window or lse, so those two are restated, not pinned to reference outputs.
Rows with no admissible key give zeros (lse -inf).

The golden's softmax is torch's (subtract the row max, exp, divide by the sum);
numpy does the same in fp32.  The work is done one KV-head group at a time to
bound memory (the math is unchanged).
"""
from __future__ import annotations

import math

import numpy as np


def _cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def flash_attn_varlen(q, k_cache, v_cache, q_lens, kv_lens, block_table, softmax_scale=None,
                      causal=True, window=(-1, -1), return_lse=False):
    """Paged varlen causal GQA attention, fp32.

    q: float32 [total_q, Hq, D]; k_cache/v_cache: float32 [NB, Hkv, bs, D];
    q_lens/kv_lens: int sequences; block_table: int [B, bt_dim].
    Returns float32 [total_q, Hq, D] (rows outside every sequence stay 0, as the
    golden's ``torch.zeros_like(q)``), and with ``return_lse`` also float32
    [Hq, total_q] log-sum-exp values (-inf where a row has no admissible key).
    """
    q = np.asarray(q, dtype=np.float32)
    k_cache = np.asarray(k_cache, dtype=np.float32)
    v_cache = np.asarray(v_cache, dtype=np.float32)
    block_table = np.asarray(block_table)
    _, hq, d = q.shape
    _, hkv, bs, _ = k_cache.shape
    g = hq // hkv
    scale = 1.0 / math.sqrt(float(d)) if softmax_scale is None else float(softmax_scale)
    out = np.zeros_like(q)
    lse = np.full((hq, q.shape[0]), -np.inf, dtype=np.float32)
    wl, wr = int(window[0]), int(window[1])
    start = 0
    for b in range(len(q_lens)):
        L, S = int(q_lens[b]), int(kv_lens[b])
        qs = q[start:start + L]
        start += L
        if L == 0:
            continue
        ids = block_table[b, :_cdiv(S, bs)].astype(np.int64)
        # [n, Hkv, bs, D] -> [n, bs, Hkv, D] -> [n*bs, Hkv, D][:S]
        k = k_cache[ids].transpose(0, 2, 1, 3).reshape(-1, hkv, d)[:S]
        v = v_cache[ids].transpose(0, 2, 1, 3).reshape(-1, hkv, d)[:S]
        i = np.arange(L)[:, None]
        j = np.arange(S)[None, :]
        if causal:
            masked = j > (S - L + i)
        elif wr >= 0:
            masked = j > (S - L + i + wr)
        else:
            masked = np.zeros((L, S), dtype=bool)
        if wl >= 0:
            masked = masked | (j < (S - L + i - wl))
        empty = masked.all(axis=1)                                         # [L]
        o = np.empty((L, hq, d), dtype=np.float32)
        for kv in range(hkv):
            qh = qs[:, kv * g:(kv + 1) * g, :].transpose(1, 0, 2)        # [g, L, D]
            s = np.matmul(qh, k[:, kv, :].T) * np.float32(scale)          # [g, L, S]
            s = np.where(masked[None], np.float32(-np.inf), s)
            mx = s.max(axis=-1, keepdims=True) if S > 0 else np.zeros((g, L, 1), np.float32)
            mx = np.where(np.isfinite(mx), mx, np.float32(0))
            s = s - mx
            np.exp(s, out=s)
            tot = s.sum(axis=-1, keepdims=True)
            with np.errstate(divide="ignore"):
                lse[kv * g:(kv + 1) * g, start - L:start] = np.where(
                    tot[..., 0] > 0, np.log(tot[..., 0]) + mx[..., 0], -np.inf)
            s /= np.where(tot > 0, tot, np.float32(1))
            o[:, kv * g:(kv + 1) * g, :] = np.matmul(s, v[:, kv, :]).transpose(1, 0, 2)
        o[empty] = 0.0
        out[start - L:start] = o
    return (out, lse) if return_lse else out


def causal_pairs(q_lens, kv_lens) -> int:
    """Number of admissible (query, key) pairs under bottom-right causal masking."""
    tot = 0
    for L, S in zip(q_lens, kv_lens):
        L, S = int(L), int(S)
        if L <= 0:
            continue
        # row i attends min(S, S - L + i + 1) keys (clamped at 0)
        first = S - L + 1
        # sum_{i=0}^{L-1} clamp(first + i, 0, S)
        i = np.arange(L, dtype=np.int64)
        tot += int(np.clip(first + i, 0, S).sum())
    return tot


def attention_flops(q_lens, kv_lens, num_heads: int, head_dim: int) -> int:
    """Algorithmic FLOPs: 4 * D * Hq * admissible pairs (QK^T and PV)."""
    return 4 * head_dim * num_heads * causal_pairs(q_lens, kv_lens)


def attention_bytes(q_lens, kv_lens, num_heads: int, num_kv_heads: int, head_dim: int,
                    block_size: int, elem: int = 2) -> int:
    """Algorithmic HBM bytes: K and V once per kv head, Q and O once, block
    tables and lengths."""
    kv = sum(int(s) for s in kv_lens) * num_kv_heads * head_dim * elem * 2
    qo = 2 * sum(int(l) for l in q_lens) * num_heads * head_dim * elem
    tables = 4 * sum(_cdiv(int(s), block_size) for s in kv_lens) + 8 * len(q_lens)
    return kv + qo + tables
