"""How the sharded forms split their work across ranks (host logic shared by the bench and the tests).

Heads are independent, so the head-sharded form gives each rank a contiguous block of kv heads with their query
heads (GQA groups stay whole).  A decode query sees every key of its sequence and softmax does not depend on key
order, so the KV-sharded form gives each rank a contiguous, balanced range of each sequence's keys.
"""
from __future__ import annotations


def head_shard(heads: int, kv_heads: int, n_ranks: int, rank: int):
    """(head0, heads_local, kv_head0, kv_heads_local) of `rank`: kv heads split evenly, queries follow their kv head."""
    if kv_heads % n_ranks or heads % kv_heads:
        raise ValueError(f"{heads} heads / {kv_heads} kv heads do not split over {n_ranks} ranks")
    kv_local = kv_heads // n_ranks
    group = heads // kv_heads
    return rank * kv_local * group, kv_local * group, rank * kv_local, kv_local


def kv_shard(length: int, n_ranks: int, rank: int):
    """(start, count) of `rank`'s keys of a `length`-key sequence: contiguous ranges whose sizes differ by at most 1."""
    base, extra = divmod(length, n_ranks)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)
