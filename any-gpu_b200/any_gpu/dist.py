"""Batch sharding across the GPUs of one node (one process per GPU).

The batched ops of the path (batch_matmul batches, SDPA batch x heads,
conv2d / group_norm images, the decoder layer's sequences) are independent
along their leading dimension.  A job of `total` items is split across the
ranks; each rank runs the library's kernels on its items and writes each
result straight into its slot of the full-size output, and the slots are
all-gathered in place (NCCL over NVLink on GPUs, gloo on CPU), so that every
rank ends with the whole result and nothing is padded, copied or
concatenated.

Rounds.  To overlap the gather with compute, the items are cut into
`rounds` consecutive spans; inside each span every rank owns one
contiguous run, in rank order.  A span's output is then one contiguous
rank-major region, which is exactly the layout an in-place all-gather
needs: rank r's run already sits at offset r * count inside it.  Round i's
gather runs on the communicator's stream while round i+1 computes.  With
one round this is the plain contiguous leading-dim shard of `batch_shard`.

The reference has no multi-GPU code (any-gpu BACKLOG.md lists multi-GPU
dispatch as planned); this is the plumbing around the single-GPU ops, not
a new op.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, List, Optional, Tuple


def batch_shard(total: int, world: int, rank: int) -> Tuple[int, int]:
    """(start, count) of rank's contiguous shard of `total` items: the first
    total % world ranks take one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def shard_counts(total: int, world: int) -> List[int]:
    return [batch_shard(total, world, r)[1] for r in range(world)]


@dataclass
class Round:
    """One span of items: ranks own contiguous runs in rank order."""
    start: int                 # first global item of the span
    count: int                 # items in the span (all ranks)
    offsets: List[int]         # first global item of each rank's run
    counts: List[int]          # items in each rank's run
    local: int                 # this rank's first item in its local (compacted) order

    @property
    def even(self) -> bool:
        return len(set(self.counts)) == 1


@dataclass
class ShardPlan:
    """`total` items over `world` ranks in `rounds` rounds (see module doc)."""
    total: int
    world: int
    rank: int
    rounds: int = 1
    spans: List[Round] = field(init=False)

    def __post_init__(self):
        if self.world <= 0 or not 0 <= self.rank < self.world:
            raise ValueError(f"bad rank {self.rank} of world {self.world}")
        # at least one item per rank per round where the total allows it
        self.rounds = max(1, min(self.rounds, self.total // self.world))
        self.spans = []
        local = 0
        for i in range(self.rounds):
            s0, n = batch_shard(self.total, self.rounds, i)
            counts = shard_counts(n, self.world)
            offsets = [s0 + batch_shard(n, self.world, r)[0] for r in range(self.world)]
            self.spans.append(Round(s0, n, offsets, counts, local))
            local += counts[self.rank]

    @property
    def my_count(self) -> int:
        return sum(r.counts[self.rank] for r in self.spans)

    def my_items(self) -> List[int]:
        """Global indices of this rank's items, in local order."""
        out = []
        for r in self.spans:
            o = r.offsets[self.rank]
            out.extend(range(o, o + r.counts[self.rank]))
        return out


def gather_round(out, item_elems: int, rd: Round, rank: int, group=None,
                 async_op: bool = False) -> list:
    """In-place all-gather of one round.  `out` is the full flat result
    (total * item_elems elements) on every rank with this rank's run of `rd`
    already in its slot; afterwards every rank holds the whole span.  Equal
    runs: one all_gather_into_tensor whose input is the rank's own slot (NCCL
    gathers in place when the send buffer is the receive buffer's rank
    slice).  Uneven runs: one in-place broadcast per rank from its slot.
    Returns the async work handles (empty when async_op is False)."""
    import torch.distributed as dist
    ie = item_elems
    world = len(rd.counts)
    if rd.even:
        span = out[rd.start * ie:(rd.start + rd.count) * ie]
        mine = out[rd.offsets[rank] * ie:(rd.offsets[rank] + rd.counts[rank]) * ie]
        w = dist.all_gather_into_tensor(span, mine, group=group, async_op=async_op)
        return [w] if async_op else []
    works = []
    for r in range(world):
        if rd.counts[r] == 0:
            continue
        part = out[rd.offsets[r] * ie:(rd.offsets[r] + rd.counts[r]) * ie]
        src = dist.get_global_rank(group, r) if group is not None else r
        w = dist.broadcast(part, src=src, group=group, async_op=async_op)
        if async_op:
            works.append(w)
    return works


def run_rounds(plan: ShardPlan, out, item_elems: int,
               launch_round: Callable[[Round], object], stream, group=None,
               gather: bool = True) -> None:
    """One sharded step on the GPU: for each round, `launch_round(rd)` enqueues
    this rank's part of the round (writing its slot of `out`) and returns
    the torch CUDA stream on which that output is complete; the round's
    in-place gather is issued from that stream, so it starts as soon as the
    round is done and runs beside the next round's compute.  On return
    `stream` waits for every launch and gather (nothing blocks the host)."""
    import torch
    works, ready_streams = [], []
    for rd in plan.spans:
        ready = launch_round(rd)
        if ready is not None and ready is not stream:
            ready_streams.append(ready)
        if gather and plan.world > 1:
            with torch.cuda.stream(ready if ready is not None else stream):
                works += gather_round(out, item_elems, rd, plan.rank, group, async_op=True)
    with torch.cuda.stream(stream):
        for s in ready_streams:
            stream.wait_stream(s)
        for w in works:
            w.wait()


def all_gather_shards(local, total: int, item_elems: int, group=None):
    """Gather uneven contiguous shards (rank r holds items batch_shard(total,
    world, r)) into the full `total * item_elems` tensor on every rank: the
    local shard is placed in its slot of the result and the slots are
    gathered in place (no padding, no concatenation)."""
    import torch
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    plan = ShardPlan(total, world, rank, 1)
    full = torch.empty(total * item_elems, dtype=local.dtype, device=local.device)
    rd = plan.spans[0]
    off = rd.offsets[rank] * item_elems
    full[off:off + local.numel()] = local.reshape(-1)
    gather_round(full, item_elems, rd, rank, group)
    return full
