"""CPU, world size 2 (gloo): the host-side sharding / gather logic used to
spread batched ops over the GPUs of one node, checked against the oracle's
full-batch result (batch_matmul and softmax of the headline workload at a
small size)."""
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


def _worker(rank, world, port, batch, m, n, k, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "any-gpu_b200"))
    sys.path.insert(0, str(root))
    import datetime

    import torch
    import torch.distributed as dist
    from any_gpu.dist import all_gather_shards, batch_shard
    from oracle import oracle as orc
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        r = np.random.default_rng(7)
        a = r.standard_normal(batch * m * k).astype(np.float32)
        b = r.standard_normal(batch * k * n).astype(np.float32)
        start, cnt = batch_shard(batch, world, rank)
        a_s = a[start * m * k:(start + cnt) * m * k]
        b_s = b[start * k * n:(start + cnt) * k * n]
        c_s = orc.batch_matmul(a_s, b_s, cnt, m, n, k)
        s_s = orc.softmax(c_s, cnt * m, n)
        full = all_gather_shards(torch.from_numpy(s_s), batch, m * n).numpy()
        want = orc.softmax(orc.batch_matmul(a, b, batch, m, n, k), batch * m, n)
        q.put((rank, bool(np.array_equal(full, want)), None))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("batch", [4, 5])
def test_sharded_batch_matmul_softmax_gloo(batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, 8, 16, 12, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, err in results:
        assert err is None, f"rank {rank}: {err}"
        assert ok, f"rank {rank}: gathered result differs from the full batch"


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
