"""Batch sharding across GPUs of one node (one process per GPU).

The batched ops of the path (batch_matmul batches, SDPA batch x heads,
conv2d / group_norm images) are independent along their leading dimension,
so a job is split into contiguous leading-dim shards, each rank runs the
library's kernels on its shard, and -- when the caller wants the whole
result on every rank -- the shards are all-gathered (NCCL over NVLink on
GPUs, gloo on CPU).  The reference has no multi-GPU code; this is the
plumbing around the single-GPU ops, not a new op.
"""
from __future__ import annotations

from typing import Tuple


def batch_shard(total: int, world: int, rank: int) -> Tuple[int, int]:
    """(start, count) of rank's contiguous shard of `total` items: the first
    total % world ranks take one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def shard_counts(total: int, world: int):
    return [batch_shard(total, world, r)[1] for r in range(world)]


def all_gather_shards(local, total: int, item_elems: int, group=None):
    """All-gather uneven contiguous shards of a flat tensor into the full
    `total * item_elems` tensor on every rank (shards padded to the largest
    shard for the collective, then compacted)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    counts = shard_counts(total, world)
    cmax = max(counts) * item_elems
    send = torch.zeros(cmax, dtype=local.dtype, device=local.device)
    send[: local.numel()] = local.reshape(-1)
    recv = torch.empty(world * cmax, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    parts = [recv[r * cmax: r * cmax + counts[r] * item_elems] for r in range(world)]
    return torch.cat(parts)
