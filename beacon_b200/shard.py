"""Data-parallel sharding of the hot path across the GPUs of one node.

The path has no exchange step: attention shards by (batch, head) units and the
GEMM by output columns, so each rank works on its own slice with no collective
inside the step.  The only collective is the verification gather after timing,
which brings every rank's result (or a checksum of it) to rank 0 over NCCL (gloo
in the CPU tests).
"""
from __future__ import annotations


def even_shard(total: int, world: int, rank: int):
    """(start, count) of rank's contiguous block of `total` units; the first
    `total % world` ranks take one extra unit."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def head_shard(batch: int, heads: int, world: int, rank: int):
    """Flat (b*heads + h) head range [start, start+count) owned by `rank`."""
    return even_shard(batch * heads, world, rank)


def gqa_shard(batch: int, q_heads: int, kv_heads: int, world: int, rank: int):
    """Grouped-query attention: whole KV groups per rank, so K/V are never replicated.
    Returns (kv_start, kv_count) over the flat b*kv_heads KV heads; the query heads
    are that range times the group size."""
    return even_shard(batch * kv_heads, world, rank)


def column_shard(n: int, world: int, rank: int):
    """GEMM: columns [start, start+count) of B (and C) owned by `rank`."""
    return even_shard(n, world, rank)


def checksum(t):
    """Order-independent float64 sum and absolute sum of a tensor (verification)."""
    import torch
    x = t.detach().to(torch.float64)
    return torch.stack([x.sum(), x.abs().sum()])


def gather_checksums(t, world: int):
    """All-gather every rank's checksum (2 float64 values) -> [world, 2] on each rank."""
    import torch
    c = checksum(t)
    if world == 1:
        return c.unsqueeze(0)
    import torch.distributed as dist
    out = [torch.empty_like(c) for _ in range(world)]
    dist.all_gather(out, c)
    return torch.stack(out)


def gather_rows(t, world: int):
    """All-gather equally shaped per-rank tensors along dim 0 (verification of
    small cases)."""
    import torch
    if world == 1:
        return t
    import torch.distributed as dist
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t.contiguous())
    return torch.cat(out, dim=0)
