"""Tensor-parallel head sharding of the hot path.

Ranks own contiguous KV-head ranges with the remainder going to the low
ranks, and each query head follows its KV head, as ASPIRE's tensor parallelism
shards ``wqkv`` (aspire/tp.py:35-51, :66-78).  Attention, KV append, the
refresh-layer dump and page selection are all rank-local under this sharding:
no collective runs on the hot path.
"""

from __future__ import annotations


def tp_heads(num_heads: int, rank: int, world: int) -> range:
    """Contiguous range of heads owned by `rank` (remainder to the low ranks)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, rem = divmod(num_heads, world)
    start = rank * base + min(rank, rem)
    return range(start, start + base + (1 if rank < rem else 0))


def local_head_counts(num_qo_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    """(local query heads, local KV heads) of a rank; query heads follow their KV group."""
    if num_qo_heads % num_kv_heads:
        raise ValueError("num_qo_heads must be a multiple of num_kv_heads")
    kv = tp_heads(num_kv_heads, rank, world)
    group = num_qo_heads // num_kv_heads
    return len(kv) * group, len(kv)


def local_qo_heads(num_qo_heads: int, num_kv_heads: int, rank: int, world: int) -> range:
    """Query heads of a rank: the groups of its KV heads."""
    kv = tp_heads(num_kv_heads, rank, world)
    group = num_qo_heads // num_kv_heads
    return range(kv.start * group, kv.stop * group)
