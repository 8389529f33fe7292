"""Helpers for the GPU parity tests: move oracle.seeded words to CUDA tensors
and call the kernels through the C ABI (tecoops.capi)."""
import numpy as np
import torch

from tecoops import capi

TORCH_DT = {"f16": torch.float16, "bf16": torch.bfloat16}
CAPI_DT = {"f16": capi.DATA_HALF, "bf16": capi.DATA_BFLOAT16}


def words_to_dev(w: np.ndarray, dtype: str) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(w).view(np.int16))
    return t.view(TORCH_DT[dtype]).cuda()


def dev_to_words(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


_HANDLE = None


def handle() -> capi.Handle:
    global _HANDLE
    if _HANDLE is None:
        _HANDLE = capi.Handle()
    _HANDLE.set_stream(stream_ptr())
    return _HANDLE


def reshape_capi(key, value, slot, kc, vc):
    """All arguments CUDA tensors; caches updated in place."""
    T, H, D = key.shape
    NB, _, BS, _ = kc.shape
    st = capi.reshape_and_cache(handle(), key.data_ptr(), value.data_ptr(), slot.data_ptr(),
                                kc.data_ptr(), vc.data_ptr(), T, H, D, NB, BS)
    capi.check(st, "tecoopsReshapeAndCache")


def attention_capi(q, kc, vc, q_lens, kv_lens, bt, max_q=None, max_k=None, out=None,
                   workspace=0, h=None):
    """CUDA tensors in the C-API layout; returns the output tensor."""
    dt = capi.DATA_HALF if q.dtype == torch.float16 else capi.DATA_BFLOAT16
    if out is None:
        out = torch.zeros_like(q)
    ql = q_lens.cpu() if max_q is None else None
    max_q = int(ql.max()) if max_q is None else max_q
    max_k = int(kv_lens.max().item()) if max_k is None else max_k
    descs = (capi.Desc(capi.DATA_INT32, bt.shape), capi.Desc(dt, q.shape),
             capi.Desc(dt, kc.shape), capi.Desc(dt, vc.shape), capi.Desc(dt, out.shape))
    st = capi.flash_attention(h or handle(), max_q, max_k, kc.shape[0], q_lens.data_ptr(),
                              kv_lens.data_ptr(), descs[0], bt.data_ptr(), descs[1],
                              q.data_ptr(), descs[2], kc.data_ptr(), descs[3], vc.data_ptr(),
                              descs[4], out.data_ptr(), workspace)
    capi.check(st, "tecoopsFlashAttention")
    return out


def attention_ex_capi(q, kc, vc, q_lens, kv_lens, bt, opts, max_q=None, max_k=None):
    """tecoopsFlashAttentionEx with a case's options dict (scale, causal, window, lse);
    returns (out, lse or None)."""
    dt = capi.DATA_HALF if q.dtype == torch.float16 else capi.DATA_BFLOAT16
    out = torch.zeros_like(q)
    lse = torch.full((q.shape[1], q.shape[0]), float("nan"), device=q.device) \
        if opts.get("lse") else None
    max_q = int(q_lens.max().item()) if max_q is None else max_q
    max_k = int(kv_lens.max().item()) if max_k is None else max_k
    descs = (capi.Desc(capi.DATA_INT32, bt.shape), capi.Desc(dt, q.shape),
             capi.Desc(dt, kc.shape), capi.Desc(dt, vc.shape), capi.Desc(dt, out.shape))
    st = capi.flash_attention_ex(handle(), max_q, max_k, kc.shape[0], q_lens.data_ptr(),
                                 kv_lens.data_ptr(), descs[0], bt.data_ptr(), descs[1],
                                 q.data_ptr(), descs[2], kc.data_ptr(), descs[3], vc.data_ptr(),
                                 descs[4], out.data_ptr(), 0,
                                 softmax_scale=opts.get("scale") or 0.0,
                                 causal=opts.get("causal", True),
                                 window=tuple(opts.get("window", (-1, -1))),
                                 softmax_lse=lse.data_ptr() if lse is not None else 0)
    capi.check(st, "tecoopsFlashAttentionEx")
    return out, lse


def attn_case_to_dev(inp, dtype):
    return dict(q=words_to_dev(inp["q"], dtype), kc=words_to_dev(inp["k_cache"], dtype),
                vc=words_to_dev(inp["v_cache"], dtype),
                q_lens=torch.from_numpy(inp["q_lens"]).cuda(),
                kv_lens=torch.from_numpy(inp["kv_lens"]).cuda(),
                bt=torch.from_numpy(inp["block_table"]).cuda())


def errors(out: np.ndarray, ref: np.ndarray):
    d = np.abs(out.astype(np.float64) - ref.astype(np.float64))
    diff1 = d.sum() / max(np.abs(ref).sum(), 1e-30)
    return float(d.max()), float(d.mean()), float(diff1)
