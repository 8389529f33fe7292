"""ORACLE — test infrastructure only.

CPU restatements of the reference's own goldens for the paged-KV attention path,
used as the checker by tests/, by ``__graft_entry__.smoke()`` and as the timed
CPU baseline of ``bench.py --impl reference``.  The product (the ``tecoops``
package and ``libteco_ops.so``) never imports, links or calls anything here.

* ``reshape_and_cache.c`` / :func:`reshape_and_cache`: the zoo C++ golden loop,
  test/zoo/teco/reshape_and_cache/reshape_and_cache.cpp:136-147.
* :func:`flash_attn_varlen`: the torch golden
  test/zoo/teco/flash_attention/flash_attention.py:79-140 restated in numpy fp32.
* :func:`rms_norm`: the zoo rms_norm golden, test/zoo/teco/rms_norm/rms_norm.cpp
  (cpuCompute), restated in numpy fp32.
* :mod:`oracle.fp8`: e4m3 encode / decode of the FP8 KV-cache extension (OCP E4M3
  definition; no reference counterpart).
* :mod:`oracle.seeded`: deterministic counter-based input generator shared by
  the golden-fixture script and the parity tests.

Parity pin: both restatements are checked against fixtures produced by the
reference's own golden functions (tests/golden/make_golden.py) in
tests/test_oracle.py.
"""
from .attention import flash_attn_varlen, attention_flops, attention_bytes  # noqa: F401
from .reshape import reshape_and_cache, reshape_and_cache_np, reshape_bytes  # noqa: F401
from .rms_norm import rms_norm, rms_norm_bytes  # noqa: F401
