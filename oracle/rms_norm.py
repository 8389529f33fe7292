"""ORACLE — test infrastructure only (see oracle/__init__.py).

numpy restatement of the reference's rms_norm CPU golden,
test/zoo/teco/rms_norm/rms_norm.cpp (RmsNormExecutor::cpuCompute), which the
reference kernel teco/ual/kernel/rms_norm/rms_norm_fp16.scpp follows:

* without residual: ``rstd = 1 / sqrt(sum(x^2) / D + eps)``, ``y = x * rstd * w``;
* with residual: ``h = x + r`` in fp32, ``residual_out = half(h)``, the sum of
  squares uses the unrounded ``h`` and the output ``half(h) * rstd * w``;
* fp32 arithmetic, products evaluated left to right, one rounding (nearest
  even) to the 16-bit type per stored value.

The python golden (python_api_test/test_rms_norm.py:33-45) differs only in using
the unrounded ``h`` for the output of the residual form; both are within its
5e-3 tolerance.  bf16 tensors (an extension) follow the same formulas.
"""
from __future__ import annotations

import numpy as np

from . import seeded


def rms_norm(x_words, w_words, r_words=None, eps=1e-6, dtype="f16"):
    """Words in, words out: returns (output, residual_out or None) as uint16 arrays."""
    x = seeded.words_to_f32(x_words, dtype)
    w = seeded.words_to_f32(w_words, dtype)
    D = x.shape[-1]
    if r_words is not None:
        h = (x + seeded.words_to_f32(r_words, dtype)).astype(np.float32)
        ss = np.einsum("nd,nd->n", h, h, dtype=np.float32)
        ho = seeded.to_words(h, dtype)
        base = seeded.words_to_f32(ho, dtype)
    else:
        ss = np.einsum("nd,nd->n", x, x, dtype=np.float32)
        ho, base = None, x
    rstd = np.float32(1.0) / np.sqrt(ss / np.float32(D) + np.float32(eps)).astype(np.float32)
    y = (base * rstd[:, None]).astype(np.float32) * w[None, :]
    return seeded.to_words(y.astype(np.float32), dtype), ho


def rms_norm_bytes(num_tokens: int, hidden: int, residual: bool, elem: int = 2) -> int:
    """Algorithmic HBM bytes (the zoo's getTheoryIoSize, rms_norm.cpp:101-115)."""
    rows = 4 if residual else 2
    return num_tokens * hidden * elem * rows + hidden * elem
