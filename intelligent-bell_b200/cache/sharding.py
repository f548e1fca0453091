"""KV-head sharding across the GPUs of one machine.

KV heads are independent in the dequant and in the RoPE rotation, so the restore shards
by head with no exchange: GPU ``rank`` of ``world_size`` restores heads
``[rank * H / world_size, (rank + 1) * H / world_size)`` from its own pinned slab over its
own PCIe link, and the output stays sharded (a tensor-parallel attention consumes head
shards).  There is no collective on the data path.
"""

from __future__ import annotations

import torch


def head_shard(num_kv_heads: int, world_size: int, rank: int) -> slice:
    """Heads owned by ``rank``; ``num_kv_heads`` must divide evenly."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside a world of {world_size}")
    if num_kv_heads % world_size:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world_size} GPUs")
    per = num_kv_heads // world_size
    return slice(rank * per, (rank + 1) * per)


def shard_view(x: torch.Tensor, num_kv_heads: int, world_size: int, rank: int,
               head_dim: int = -2) -> torch.Tensor:
    """View of ``rank``'s heads of a tensor whose ``head_dim`` axis holds the KV heads
    (e.g. a full-model slab ``[L, blocks, chunk, H, D]`` when filling a shard's slab)."""
    if x.shape[head_dim] != num_kv_heads:
        raise ValueError(f"axis {head_dim} has {x.shape[head_dim]} heads, expected {num_kv_heads}")
    sl = head_shard(num_kv_heads, world_size, rank)
    return x.narrow(head_dim, sl.start, sl.stop - sl.start)
