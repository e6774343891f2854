"""CPU, world size 2 (gloo): the host-side sharding used to spread batched ops
over the GPUs of one node -- the round plan, and the in-place gathers that
leave the whole result on every rank -- checked against the oracle's
full-batch result (batch_matmul + softmax of the headline workload at a small
size).  Uneven runs, several rounds and a rank with no items are covered."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, rounds, m, n, k, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "any-gpu_b200"))
    sys.path.insert(0, str(root))
    import datetime

    import torch
    import torch.distributed as dist
    from any_gpu.dist import ShardPlan, all_gather_shards, batch_shard, gather_round
    from oracle import oracle as orc
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        r = np.random.default_rng(7)
        a = r.standard_normal(batch * m * k).astype(np.float32)
        b = r.standard_normal(batch * k * n).astype(np.float32)
        want = orc.softmax(orc.batch_matmul(a, b, batch, m, n, k), batch * m, n)
        plan = ShardPlan(batch, world, rank, rounds)
        # this rank's inputs, compacted in local order (what a GPU rank holds)
        items = plan.my_items()
        a_loc = np.concatenate([a[g * m * k:(g + 1) * m * k] for g in items] or [a[:0]])
        b_loc = np.concatenate([b[g * k * n:(g + 1) * k * n] for g in items] or [b[:0]])
        full = torch.full((batch * m * n,), float("nan"))
        for rd in plan.spans:
            cnt = rd.counts[rank]
            if cnt:
                c = orc.batch_matmul(a_loc[rd.local * m * k:(rd.local + cnt) * m * k],
                                     b_loc[rd.local * k * n:(rd.local + cnt) * k * n],
                                     cnt, m, n, k)
                s = orc.softmax(c, cnt * m, n)
                o = rd.offsets[rank] * m * n
                full[o:o + s.size] = torch.from_numpy(s)
            gather_round(full, m * n, rd, rank)
        ok_rounds = bool(np.array_equal(full.numpy(), want))
        # the one-round helper from contiguous shards
        start, cnt = batch_shard(batch, world, rank)
        s_loc = orc.softmax(orc.batch_matmul(a[start * m * k:(start + cnt) * m * k],
                                             b[start * k * n:(start + cnt) * k * n],
                                             cnt, m, n, k), cnt * m, n)
        g = all_gather_shards(torch.from_numpy(s_loc), batch, m * n).numpy()
        q.put((rank, ok_rounds, bool(np.array_equal(g, want)), None))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, False, repr(e)))


@pytest.mark.parametrize("batch,rounds", [(4, 1), (5, 1), (8, 2), (9, 3), (6, 3), (1, 1)])
def test_sharded_rounds_gather_in_place_gloo(batch, rounds):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, rounds, 8, 16, 12, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_rounds, ok_helper, err in results:
        assert err is None, f"rank {rank}: {err}"
        assert ok_rounds, f"rank {rank}: round-gathered result differs from the full batch"
        assert ok_helper, f"rank {rank}: all_gather_shards result differs from the full batch"


def test_batch_shard_covers_everything():
    from any_gpu.dist import batch_shard, shard_counts
    for total in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [batch_shard(total, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == total
            pos = 0
            for s, c in spans:
                assert s == pos
                pos += c
            assert shard_counts(total, world) == [c for _, c in spans]
    with pytest.raises(ValueError):
        batch_shard(4, 2, 2)


@pytest.mark.parametrize("total", [1, 5, 16, 32, 64, 65, 256])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("rounds", [1, 2, 4, 8])
def test_shard_plan_layout(total, world, rounds):
    """Every item is owned once; inside a round the ranks' runs are contiguous
    and in rank order (so the round's gather is in place); local order is
    round-major; the plan does not depend on which rank builds it."""
    from any_gpu.dist import ShardPlan
    plans = [ShardPlan(total, world, r, rounds) for r in range(world)]
    owned = sorted(g for p in plans for g in p.my_items())
    assert owned == list(range(total))
    p0 = plans[0]
    pos = 0
    for i, rd in enumerate(p0.spans):
        assert rd.start == pos and rd.count == sum(rd.counts)
        o = rd.start
        for r in range(world):
            assert rd.offsets[r] == o
            o += rd.counts[r]
        pos += rd.count
        for p in plans[1:]:
            assert (p.spans[i].start, p.spans[i].counts) == (rd.start, rd.counts)
    assert pos == total
    for p in plans:
        loc = 0
        for rd in p.spans:
            assert rd.local == loc
            loc += rd.counts[p.rank]
        assert loc == p.my_count == len(p.my_items())
    if total >= world:
        assert all(min(rd.counts) >= 1 for rd in p0.spans)
