"""KV-head sharding of the attention path across the GPUs of one node.

Attention for KV head k reads only that head's cache slice and writes only the
outputs of its Q heads k*g .. k*g+g-1 (g = Hq / Hkv), so the path partitions by
KV head with no data exchange.  Rank r of G owns KV heads
[r*Hkv/G, (r+1)*Hkv/G) as its own cache tensors [pages, Hkv/G, block_size, D],
its slice of the new K/V [T, Hkv/G, D] and of Q / O [T, Hq/G, D]; slot_mapping,
block tables and lengths are replicated.  Each rank runs the unchanged C API on
its shard.  Outputs are gathered only to verify (gather_heads).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_begin: int
    kv_end: int
    q_begin: int
    q_end: int

    @property
    def kv_heads(self) -> int:
        return self.kv_end - self.kv_begin

    @property
    def q_heads(self) -> int:
        return self.q_end - self.q_begin


def head_shard(num_heads: int, num_kv_heads: int, world: int, rank: int) -> HeadShard:
    """KV-head range of `rank`; requires num_kv_heads % world == 0 and
    num_heads % num_kv_heads == 0."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be a multiple of num_kv_heads")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world} ranks")
    g = num_heads // num_kv_heads
    per = num_kv_heads // world
    kb, ke = rank * per, (rank + 1) * per
    return HeadShard(rank, world, kb, ke, kb * g, ke * g)


def shard_tokens(x, s: HeadShard, kv: bool):
    """Slice [T, H, D] (K/V when kv=True, Q/O otherwise) to this shard, contiguous."""
    b, e = (s.kv_begin, s.kv_end) if kv else (s.q_begin, s.q_end)
    return x[:, b:e].contiguous()


def shard_cache(cache, s: HeadShard):
    """[pages, Hkv, block_size, D] -> this shard's own [pages, Hkv/G, block_size, D]."""
    return cache[:, s.kv_begin:s.kv_end].contiguous()


def gather_heads(out_local, world: int, group=None):
    """Verification only: all-gather [T, Hq/G, D] shards into [T, Hq, D] (head order)."""
    import torch
    import torch.distributed as dist
    parts = [torch.empty_like(out_local) for _ in range(world)]
    dist.all_gather(parts, out_local.contiguous(), group=group)
    return torch.cat(parts, dim=1)
