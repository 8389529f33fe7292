"""tecoops — B200 (sm_100a) implementation of the Teco-Ops paged-KV attention path.

Drop-in for the reference package api/tecoops/__init__.py: exports
``reshape_and_cache(key, value, slot_mapping, key_cache, value_cache)`` and
``flash_attn_varlen_func(q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k,
cu_seqlens_k, seqused_k, softmax_scale, causal, window_size, block_table,
return_softmax_lse, out)`` (the flags honoured; ``(out, lse)`` is returned with
``return_softmax_lse``), ``rms_norm(input, weight, residual, output, residual_out,
eps)``, and registers ``torch.ops.tecoops.reshape_and_cache`` /
``torch.ops.tecoops.flash_attention`` / ``torch.ops.tecoops.rms_norm``; and, as an
extension, ``reshape_and_cache_flash_attn_decode(q, key, value, k_cache, v_cache,
slot_mapping, seqused_k, block_table, max_seqlen_k, out)`` (one launch per decode step;
``torch.ops.tecoops.reshape_and_cache_flash_attention_decode``).  The other
reference ops (flatten_rays, morton3D_invert, causal_conv1d_fn_torch) are not on
this path and are not provided.

There is no CPU or eager fallback: importing fails loudly when the compiled
extension (built by ``teco-ops_b200/build.py``) is missing.
"""
import os as _os

import torch  # noqa: F401  (loads libtorch before the extension)

_HERE = _os.path.dirname(_os.path.abspath(__file__))

try:
    from ._torch_ext import (flash_attn_varlen_func, reshape_and_cache,  # noqa: F401
                             reshape_and_cache_flash_attn_decode, rms_norm)
except ImportError as _e:  # pragma: no cover - exercised only on a broken install
    raise ImportError(
        "tecoops: the compiled extension is missing; run `python teco-ops_b200/build.py` "
        f"(looked in {_HERE}): {_e}") from _e

LIBRARY_PATH = _os.path.join(_HERE, "libteco_ops.so")

__all__ = ["reshape_and_cache", "flash_attn_varlen_func", "rms_norm",
           "reshape_and_cache_flash_attn_decode", "LIBRARY_PATH"]
