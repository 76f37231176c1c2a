"""How the hot path spreads over the GPUs of one node (one process per GPU).

Decode attention: (sequence, kv-head) units are independent, so a long-context batch is
split by KV head -- rank r owns kv-heads [r*H/N, (r+1)*H/N) and the query heads of their
GQA groups, and its own slice of every page.  There is no exchange inside attention; an
all-gather of the outputs is optional (replicated outputs).

Prefill -> decode migration: the first half of the ranks are prefill ranks, the second
half decode ranks; prefill rank r pushes to decode rank r + N/2 over NVLink (peer stores
into the decode pool, mapped by CUDA IPC).  Requests go round-robin to prefill ranks.

These are plain host functions; the multi-rank tests run them under gloo on CPU.
"""
from __future__ import annotations


def kv_head_shard(num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) kv-heads owned by `rank`; heads must split evenly."""
    if world <= 0 or num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def q_head_shard(num_q_heads: int, num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Query heads that go with the rank's kv-heads (GQA groups stay whole)."""
    lo, hi = kv_head_shard(num_kv_heads, world, rank)
    g = num_q_heads // num_kv_heads
    return lo * g, hi * g


def migration_peer(world: int, rank: int) -> tuple[bool, int]:
    """(is_prefill_rank, peer rank) for the prefill -> decode push."""
    if world < 2 or world % 2:
        raise ValueError("migration needs an even number of ranks >= 2")
    half = world // 2
    return (rank < half, rank + half if rank < half else rank - half)


def assign_requests(num_requests: int, world: int) -> list[int]:
    """Prefill rank of each request (round-robin over the prefill half)."""
    half = max(1, world // 2)
    return [i % half for i in range(num_requests)]
