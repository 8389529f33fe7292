"""KV-head sharding across ranks (CPU, gloo, world size 2): each rank computes its
head shard of a parity case with the oracle, the shards are gathered, and the
result must equal the unsharded oracle bit for bit (heads are independent)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tecoops import sharding


def test_head_shard_ranges():
    s = [sharding.head_shard(64, 8, 4, r) for r in range(4)]
    assert [(x.kv_begin, x.kv_end) for x in s] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert [(x.q_begin, x.q_end) for x in s] == [(0, 16), (16, 32), (32, 48), (48, 64)]
    assert sharding.head_shard(32, 8, 8, 7).q_heads == 4
    with pytest.raises(ValueError):
        sharding.head_shard(32, 8, 3, 0)
    with pytest.raises(ValueError):
        sharding.head_shard(30, 8, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, name, result_file):
    import cases
    import oracle
    from oracle import seeded
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    q = torch.from_numpy(seeded.words_to_f32(inp["q"], c["dtype"]))
    kc = torch.from_numpy(seeded.words_to_f32(inp["k_cache"], c["dtype"]))
    vc = torch.from_numpy(seeded.words_to_f32(inp["v_cache"], c["dtype"]))
    s = sharding.head_shard(c["Hq"], c["Hkv"], world, rank)
    out_local = oracle.flash_attn_varlen(
        sharding.shard_tokens(q, s, kv=False).numpy(), sharding.shard_cache(kc, s).numpy(),
        sharding.shard_cache(vc, s).numpy(), inp["q_lens"], inp["kv_lens"], inp["block_table"])
    full = sharding.gather_heads(torch.from_numpy(out_local), world)
    if rank == 0:
        np.save(result_file, full.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["api_gqa_32q8kv_prefill", "bf16_bs16_decode"])
def test_two_rank_head_sharding_reassembles(tmp_path, name):
    import cases
    import oracle
    from oracle import seeded
    world = 2
    out_file = str(tmp_path / "out.npy")
    mp.spawn(_rank_main, args=(world, _free_port(), name, out_file), nprocs=world, join=True)
    c = cases.ATTN_CASES[name]
    inp = cases.attn_inputs(c)
    ref = oracle.flash_attn_varlen(
        seeded.words_to_f32(inp["q"], c["dtype"]), seeded.words_to_f32(inp["k_cache"], c["dtype"]),
        seeded.words_to_f32(inp["v_cache"], c["dtype"]), inp["q_lens"], inp["kv_lens"],
        inp["block_table"])
    got = np.load(out_file)
    assert np.array_equal(got, ref)
