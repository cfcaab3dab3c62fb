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


def owner(unit: int, total: int, world: int) -> int:
    """The rank whose even_shard block holds `unit`."""
    for r in range(world):
        s, c = even_shard(total, world, r)
        if s <= unit < s + c:
            return r
    raise ValueError(f"unit {unit} outside [0, {total})")


def gather_units(local, start: int, total: int, wanted, world: int):
    """Bring the `wanted` units (global indices) of a sharded tensor to every rank.

    `local` is this rank's block [count, ...] of units start .. start+count-1 of `total`.
    Every rank fills one slot per wanted unit (zeros where it does not own the unit)
    and the slots are all-gathered, so all ranks take the same collective step whatever
    they own; each unit is then read from its owner's slots.  Returns [len(wanted), ...].
    Used after timing, to verify sampled heads / columns / rows on rank 0."""
    import torch
    count = local.shape[0]
    slots = torch.zeros((len(wanted),) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    for i, u in enumerate(wanted):
        if start <= u < start + count:
            slots[i] = local[u - start]
    if world == 1:
        return slots
    import torch.distributed as dist
    parts = [torch.empty_like(slots) for _ in range(world)]
    dist.all_gather(parts, slots)
    return torch.stack([parts[owner(u, total, world)][i] for i, u in enumerate(wanted)])


def unit_generator(seed: int, unit: int, device):
    """A torch generator for one unit (head, KV group, weight) of a global seeded tensor:
    the unit's values depend on (seed, unit) only, never on how many ranks share the work."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + unit)
    return g


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
