"""reshape_and_cache on the GPU through the C ABI: bit-exact against the
reference golden (fixture hashes) and the oracle; full-size property checks."""
import hashlib

import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("name", sorted(cases.RESHAPE_CASES))
def test_reshape_bit_exact_vs_golden(golden, name):
    from gpu_util import dev_to_words, reshape_capi, words_to_dev
    c = cases.RESHAPE_CASES[name]
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    dk, dv = words_to_dev(key, c["dtype"]), words_to_dev(value, c["dtype"])
    dkc, dvc = words_to_dev(kc, c["dtype"]), words_to_dev(vc, c["dtype"])
    reshape_capi(dk, dv, torch.from_numpy(slot).cuda(), dkc, dvc)
    torch.cuda.synchronize()
    gk, gv = dev_to_words(dkc), dev_to_words(dvc)
    assert hashlib.sha256(gk.tobytes()).digest() == bytes(golden[f"rc/{name}/sha_k"])
    assert hashlib.sha256(gv.tobytes()).digest() == bytes(golden[f"rc/{name}/sha_v"])
    oracle.reshape_and_cache(key, value, slot, kc, vc)
    assert np.array_equal(gk, kc) and np.array_equal(gv, vc)


@pytest.mark.parametrize("T,layout,pad", [(1, "scattered", 0.0), (16, "sequential", 0.1),
                                           (4096, "scattered", 0.1), (65536, "scattered", 0.0),
                                           (65536, "sequential", 0.1)])
def test_reshape_full_size_properties(T, layout, pad):
    """Reshape-sweep sizes (65,536-page cache, 2 GiB per cache): every valid
    token's rows land bit-exactly at their slot and nothing else changes."""
    from gpu_util import reshape_capi
    H, D, NB, BS = 8, 128, 65536, 16
    g = torch.Generator(device="cuda").manual_seed(30 + T)
    key = torch.randn(T, H, D, device="cuda", dtype=torch.bfloat16, generator=g)
    value = torch.randn(T, H, D, device="cuda", dtype=torch.bfloat16, generator=g)
    if layout == "scattered":
        slot = torch.randperm(NB * BS, device="cuda", generator=g)[:T]
    else:
        slot = torch.arange(T, device="cuda")
    if pad > 0:
        slot = torch.where(torch.rand(T, device="cuda", generator=g) < pad,
                           torch.full_like(slot, -1), slot)
    sentinel = -12345
    kc = torch.full((NB, H, BS, D), sentinel, dtype=torch.int16, device="cuda").view(torch.bfloat16)
    vc = torch.full((NB, H, BS, D), sentinel, dtype=torch.int16, device="cuda").view(torch.bfloat16)
    reshape_capi(key, value, slot, kc, vc)
    valid = slot >= 0
    s = slot[valid]
    blk, off = s // BS, s % BS
    got_k = kc[blk, :, off, :].view(torch.int16)
    got_v = vc[blk, :, off, :].view(torch.int16)
    assert torch.equal(got_k, key[valid].view(torch.int16))
    assert torch.equal(got_v, value[valid].view(torch.int16))
    n_written = int(valid.sum()) * H * D
    untouched_k = int((kc.view(torch.int16) == sentinel).sum())
    untouched_v = int((vc.view(torch.int16) == sentinel).sum())
    total = NB * H * BS * D
    # a written element may itself equal the sentinel bit pattern: allow that
    coincide_k = int((key[valid].view(torch.int16) == sentinel).sum())
    coincide_v = int((value[valid].view(torch.int16) == sentinel).sum())
    assert untouched_k == total - n_written + coincide_k
    assert untouched_v == total - n_written + coincide_v


def test_reshape_repeatable():
    from gpu_util import dev_to_words, reshape_capi, words_to_dev
    c = cases.RESHAPE_CASES["cfg1_bf16"]
    key, value, slot, kc, vc = cases.reshape_inputs(c)
    outs = []
    for _ in range(2):
        dkc, dvc = words_to_dev(kc, "bf16"), words_to_dev(vc, "bf16")
        reshape_capi(words_to_dev(key, "bf16"), words_to_dev(value, "bf16"),
                     torch.from_numpy(slot).cuda(), dkc, dvc)
        outs.append(dev_to_words(dkc).tobytes() + dev_to_words(dvc).tobytes())
    assert outs[0] == outs[1]
