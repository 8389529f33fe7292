"""Generate the golden fixtures in this directory from the REFERENCE's own CPU
goldens.  Runs only where the reference source tree is available (it is not on
the GPU box); the fixtures it writes are committed.

    python tests/golden/make_golden.py /path/to/reference

Goldens imported (three unavailable modules are stubbed in sys.modules):
* attention: ``flash_attn_varlen_func`` from
  test/zoo/teco/flash_attention/flash_attention.py (needs ``prototxt_parser``),
  cross-checked against ``flash_attn_varlen_func_ref`` from
  python_api_test/test_flash_attention.py (needs ``torch_sdaa``, ``tecoops``);
  inputs are converted exactly as test_flash_attention.py:167-181 does
  (16-bit -> fp32, cache permute [NB,H,bs,D] -> [NB,bs,H,D]).
* rms_norm: ``rms_norm_ref`` / ``rms_norm_add_ref`` from
  python_api_test/test_rms_norm.py (fp16 cases).
* reshape_and_cache: ``reshape_and_cache_flash`` from
  python_api_test/test_reshape_and_cache.py on the vLLM-layout view, as that
  test does (sdaa_to_cpu permute).

Cases with options pass their softmax_scale / causal to both goldens; cases
with a window are skipped (the reference has no windowed attention).

Each fixture stores the case name, a deterministic sample of golden output
values (float32) with their flat indices, float64 sum / abs-sum checksums, and
for reshape the SHA-256 of the resulting caches in the SDAA layout.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import cases  # noqa: E402
from oracle import seeded  # noqa: E402


def _stub(name, **attrs):
    m = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(m, k, v)
    sys.modules[name] = m
    return m


def load_goldens(ref):
    pp = _stub("prototxt_parser")
    pp.prototxt_parser_main = _stub("prototxt_parser.prototxt_parser_main", parse=lambda *a, **k: {})
    _stub("torch_sdaa")
    _stub("tecoops")
    sys.path.insert(0, os.path.join(ref, "test", "zoo", "teco"))
    sys.path.insert(0, os.path.join(ref, "test", "zoo", "teco", "flash_attention"))
    sys.path.insert(0, os.path.join(ref, "python_api_test"))
    import flash_attention as zoo_fa  # noqa: E402
    import test_flash_attention as api_fa  # noqa: E402
    import test_reshape_and_cache as api_rc  # noqa: E402
    import test_rms_norm as api_rn  # noqa: E402
    return zoo_fa.flash_attn_varlen_func, api_fa.flash_attn_varlen_func_ref, \
        api_rc.reshape_and_cache_flash, (api_rn.rms_norm_ref, api_rn.rms_norm_add_ref)


def words_to_torch_f32(w, dtype):
    return torch.from_numpy(seeded.words_to_f32(w, dtype))


def words_to_torch16(w, dtype):
    t = torch.from_numpy(np.ascontiguousarray(w).view(np.int16))
    return t.view(torch.float16 if dtype == "f16" else torch.bfloat16)


def main(ref):
    zoo_golden, api_golden, rc_golden, rn_golden = load_goldens(ref)
    torch.set_num_threads(os.cpu_count() or 1)
    out = {}
    for name, c in cases.ATTN_CASES.items():
        inp = cases.attn_inputs(c)
        q = words_to_torch_f32(inp["q"], c["dtype"])
        k = words_to_torch_f32(inp["k_cache"], c["dtype"]).permute(0, 2, 1, 3).contiguous()
        v = words_to_torch_f32(inp["v_cache"], c["dtype"]).permute(0, 2, 1, 3).contiguous()
        bt = torch.from_numpy(inp["block_table"])
        ql = inp["q_lens"].tolist()
        kl = inp["kv_lens"].tolist()
        if not cases.has_reference_golden(c):
            continue   # windowed attention: no reference implementation
        opts = cases.attn_opts(c)
        scale = opts["softmax_scale"] or 1.0 / np.sqrt(float(c["D"]))
        g = zoo_golden(q, k, v, ql, kl, bt, causal=opts["causal"], softmax_scale=scale).numpy()
        g2 = api_golden(q, k, v, torch.tensor(ql), torch.tensor(kl), bt, causal=opts["causal"],
                        softmax_scale=scale).numpy()
        assert np.array_equal(g, g2), f"reference goldens disagree on {name}"
        flat = g.reshape(-1).astype(np.float32)
        idx = cases.sample_index(flat.size)
        out[f"attn/{name}/idx"] = idx
        out[f"attn/{name}/val"] = flat[idx]
        out[f"attn/{name}/sum"] = np.array([flat.astype(np.float64).sum(),
                                            np.abs(flat.astype(np.float64)).sum()])
        print(f"attn {name}: shape {g.shape} sum {flat.sum():.6f}")
    for name, c in cases.RESHAPE_CASES.items():
        key, value, slot, kc, vc = cases.reshape_inputs(c)
        kt = words_to_torch16(key, c["dtype"])
        vt = words_to_torch16(value, c["dtype"])
        # the golden works on the vLLM layout view [NB, bs, H, D] (test_reshape_and_cache.py:35-46)
        kct = words_to_torch16(kc, c["dtype"]).permute(0, 2, 1, 3).contiguous()
        vct = words_to_torch16(vc, c["dtype"]).permute(0, 2, 1, 3).contiguous()
        rc_golden(kt, vt, kct, vct, torch.from_numpy(slot))
        kres = kct.permute(0, 2, 1, 3).contiguous().view(torch.int16).numpy().view(np.uint16)
        vres = vct.permute(0, 2, 1, 3).contiguous().view(torch.int16).numpy().view(np.uint16)
        out[f"rc/{name}/sha_k"] = np.frombuffer(hashlib.sha256(kres.tobytes()).digest(), np.uint8)
        out[f"rc/{name}/sha_v"] = np.frombuffer(hashlib.sha256(vres.tobytes()).digest(), np.uint8)
        print(f"reshape {name}: {int((slot >= 0).sum())} valid slots")
    for name, c in cases.RMS_CASES.items():
        if c["dtype"] != "f16":
            continue   # the reference golden is fp16 only
        x, w, r = cases.rms_inputs(c)
        xt, wt = words_to_torch16(x, "f16"), words_to_torch16(w, "f16")
        if r is None:
            outs = {"out": rn_golden[0](xt, wt, c["eps"])}
        else:
            o, ro = rn_golden[1](xt, words_to_torch16(r, "f16"), wt, c["eps"])
            outs = {"out": o, "res_out": ro}
        for key, t in outs.items():
            flat = t.float().numpy().reshape(-1)
            idx = cases.sample_index(flat.size)
            out[f"rms/{name}/{key}/idx"] = idx
            out[f"rms/{name}/{key}/val"] = flat[idx]
        print(f"rms_norm {name}: {tuple(xt.shape)} residual={r is not None}")
    meta = {"attn": cases.ATTN_CASES, "rc": cases.RESHAPE_CASES, "rms": cases.RMS_CASES,
            "generator": "tests/golden/make_golden.py", "torch": torch.__version__}
    out["meta"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), np.uint8)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the reference source tree>")
    main(sys.argv[1])
