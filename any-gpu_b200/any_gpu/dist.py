"""Batch sharding across the GPUs of one node (one process per GPU).

The batched ops of the path (batch_matmul batches, SDPA batch x heads,
conv2d / group_norm images, the decoder layer's sequences) are independent
along their leading dimension.  A job of `total` items is split across the
ranks; each rank runs the library's kernels on its items and writes each
result straight into its slot of the full-size output, and the slots are
all-gathered in place (NCCL over NVLink on GPUs, gloo on CPU), so that every
rank ends with the whole result and nothing is padded, copied or
concatenated.

Gathers.  PeerGather pushes each finished round into every peer's copy of
the output with the copy engines over CUDA IPC (no SMs, so it overlaps the
persistent contraction kernels); NcclGather runs the in-place NCCL
collectives instead.

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


class NcclGather:
    """Round gathers as in-place NCCL collectives (gather_round), each issued
    from the stream on which its round's output is complete, so NCCL's stream
    starts it as soon as the round is done."""
    kind = "nccl"

    def __init__(self, plan: ShardPlan, out, item_elems: int, group=None):
        self.plan, self.out, self.ie, self.group = plan, out, item_elems, group
        self._works: list = []

    def round(self, rd: Round, ready) -> None:
        import torch
        with torch.cuda.stream(ready):
            self._works += gather_round(self.out, self.ie, rd, self.plan.rank, self.group,
                                        async_op=True)

    def finish(self, stream) -> None:
        import torch
        with torch.cuda.stream(stream):
            for w in self._works:
                w.wait()
        self._works = []

    def close(self) -> None:
        pass


class PeerGather:
    """Round gathers on the copy engines: every rank pushes its run of each
    finished round straight into the same slot of every peer's output over
    NVLink (agpu_copy_async into the peer's buffer, mapped with CUDA IPC), on
    `streams` copy streams with the peers in rotated order, so the pushes use
    no SMs and run beside the next round's kernels.

    End of step (`sync="flags"`, default): after its pushes a rank stores the
    step number into its slot of every rank's flag array
    (agpu_signal_peers, a system-scope release after the copies), and its
    stream waits until all slots of its own array reach the step
    (agpu_wait_flags: one warp, a bounded spin whose expiry is reported as
    AGPU_ERR_TIMEOUT) -- no host round trip, so the host keeps queueing the
    next step.  `sync="events"`: interprocess events plus a host barrier on
    `host_group` instead.  Either way every rank then holds the whole
    output.  Uneven runs need no special case.  `out` must come from
    cudaMalloc (torch's default allocator does)."""
    kind = "ce"

    def __init__(self, dev, plan: ShardPlan, out, item_elems: int, host_group,
                 streams: int = 1, sync: str = "flags", wait_limit_us: int = 2_000_000):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _check, _lib
        if sync not in ("flags", "events"):
            raise ValueError(f"sync must be 'flags' or 'events', got {sync!r}")
        self.lib, self._check, self.C = _lib.load(), _check, C
        self.dev, self.plan, self.out, self.ie = dev, plan, out, item_elems
        self.group, self.sync, self.limit = host_group, sync, wait_limit_us
        lib, h = self.lib, dev.handle
        world, rank = plan.world, plan.rank
        self.flags = torch.zeros(world, dtype=torch.int32, device=out.device)
        self.step = 0

        def export(ptr):
            mem, off = (C.c_ubyte * 64)(), C.c_uint64()
            _check(lib.agpu_ipc_export(h, ptr, mem, C.byref(off)))
            return bytes(mem), off.value

        ev, evh = C.c_void_p(), (C.c_ubyte * 64)()
        _check(lib.agpu_ipc_event_create(h, C.byref(ev), evh))
        self.event = ev
        mine = (export(out.data_ptr()), export(self.flags.data_ptr()), bytes(evh))
        table = [None] * world
        dist.all_gather_object(table, mine, group=host_group)
        torch.cuda.synchronize()  # the zeroed flags are in place before any peer signals
        dist.barrier(group=host_group)
        self._bases = []
        imported = {}

        def import_(mb):
            if mb not in imported:  # one mapping per allocation
                base = C.c_void_p()
                _check(lib.agpu_ipc_import(h, (C.c_ubyte * 64).from_buffer_copy(mb),
                                           C.byref(base)))
                imported[mb] = base
                self._bases.append(base)
            return imported[mb].value

        self.peers = []  # (rank, dst pointer of the peer's out, its event)
        flag_slots = []  # this rank's slot in every rank's flag array
        for p in range(world):
            (mb, moff), (fb, foff), eb = table[p]
            if p == rank:
                flag_slots.append(self.flags.data_ptr() + 4 * rank)
                continue
            flag_slots.append(import_(fb) + foff + 4 * rank)
        # peers in rotated order (rank+1, rank+2, ...): at any moment every rank
        # pushes to a different peer
        for p in ((rank + i) % world for i in range(1, world)):
            (mb, moff), _, eb = table[p]
            pev = C.c_void_p()
            _check(lib.agpu_ipc_event_import(h, (C.c_ubyte * 64).from_buffer_copy(eb),
                                             C.byref(pev)))
            self.peers.append((p, import_(mb) + moff, pev))
        self.flag_slots = (C.c_void_p * world)(*flag_slots)
        # `streams` copy streams, peer i on stream i % streams: a few engines
        # each streaming one copy after another beat one copy per engine per
        # peer, which contend for the copy engines at 7 peers
        n = max(1, min(streams, len(self.peers)))
        self.streams = [torch.cuda.Stream() for _ in range(n)]

    def round(self, rd: Round, ready) -> None:
        import torch
        n = rd.counts[self.plan.rank]
        if n == 0:
            return
        ev = torch.cuda.Event()
        ev.record(ready)
        nbytes = 4 * n * self.ie
        off = 4 * rd.offsets[self.plan.rank] * self.ie
        src = self.out.data_ptr() + off
        for cs in self.streams:
            cs.wait_event(ev)
        for i, (_, dst, _) in enumerate(self.peers):
            cs = self.streams[i % len(self.streams)]
            self._check(self.lib.agpu_copy_async(self.dev.handle, dst + off, src, nbytes,
                                                 cs.cuda_stream))

    def finish(self, stream) -> None:
        h = self.dev.handle
        for cs in self.streams:
            stream.wait_stream(cs)
        if self.sync == "flags":
            self.step += 1
            # the signal follows every push of this step (stream order)
            self._check(self.lib.agpu_signal_peers(h, self.flag_slots, self.plan.world,
                                                   self.step, stream.cuda_stream))
            self._check(self.lib.agpu_wait_flags(h, self.flags.data_ptr(), self.plan.world,
                                                 self.step, self.limit, stream.cuda_stream))
            return
        import torch.distributed as dist
        self._check(self.lib.agpu_event_record(h, self.event, stream.cuda_stream))
        dist.barrier(group=self.group)  # every rank's record is issued
        for _, _, pev in self.peers:
            self._check(self.lib.agpu_stream_wait_event(h, stream.cuda_stream, pev))

    def close(self) -> None:
        """Unmap the peers' buffers (after every rank's pushes are done)."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        h = self.dev.handle
        for _, _, pev in self.peers:
            self.lib.agpu_event_destroy(h, pev)
        for base in self._bases:
            self.lib.agpu_ipc_close(h, base)
        self.lib.agpu_event_destroy(h, self.event)
        self.peers, self._bases = [], []
        dist.barrier(group=self.group)


def run_rounds(plan: ShardPlan, launch_round: Callable[[Round], object], stream,
               gatherer=None) -> None:
    """One sharded step on the GPU: for each round, `launch_round(rd)` enqueues
    this rank's part of the round (writing its slots of the output) and
    returns the torch CUDA stream on which that output is complete; the
    gatherer (NcclGather or PeerGather; None: no gather) starts that round's
    gather from there, so it runs beside the next round's compute.  On return
    `stream` waits for every launch and gather (nothing blocks the host but
    the PeerGather host barrier)."""
    ready_streams = []
    for rd in plan.spans:
        ready = launch_round(rd)
        if ready is None:
            ready = stream
        if ready is not stream:
            ready_streams.append(ready)
        if gatherer is not None and plan.world > 1:
            gatherer.round(rd, ready)
    for s in ready_streams:
        stream.wait_stream(s)
    if gatherer is not None and plan.world > 1:
        gatherer.finish(stream)


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
