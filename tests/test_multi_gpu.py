"""GPU, 2 ranks over NCCL (skipped with fewer than 2 GPUs): each rank runs
batch_matmul + softmax on its shard of the batch through the library's launch
layer, the shards are all-gathered, and every rank checks the full result
against a single-GPU run of the whole batch."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "any-gpu_b200"))
    import datetime

    import torch
    import torch.distributed as dist
    from any_gpu import GpuDevice
    from any_gpu.dist import all_gather_shards, batch_shard
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        batch, m, n, k = 6, 256, 512, 384
        r = np.random.default_rng(3)
        a = (r.standard_normal(batch * m * k) * 0.05).astype(np.float32)
        b = (r.standard_normal(batch * k * n) * 0.05).astype(np.float32)
        dev = GpuDevice.gpu(rank)
        s = torch.cuda.Stream()
        torch.cuda.set_stream(s)
        start, cnt = batch_shard(batch, world, rank)
        A = torch.from_numpy(a[start * m * k:(start + cnt) * m * k]).cuda()
        B = torch.from_numpy(b[start * k * n:(start + cnt) * k * n]).cuda()
        C = torch.empty(cnt * m * n, device="cuda")
        S = torch.empty_like(C)
        dev.launch_batch_matmul(A.data_ptr(), B.data_ptr(), C.data_ptr(), cnt, m, n, k,
                                s.cuda_stream)
        dev.launch_softmax(C.data_ptr(), S.data_ptr(), cnt * m, n, s.cuda_stream)
        full = all_gather_shards(S, batch, m * n).cpu().numpy()
        # the same batch on this one GPU, through the buffer API
        want = dev.read(dev.softmax(dev.batch_matmul(dev.upload(a), dev.upload(b), batch, m, n,
                                                     k), batch * m, n))
        q.put((rank, float(np.abs(full - want).max()), None))
        torch.cuda.synchronize()
        dist.destroy_process_group()
        dev.close()
    except Exception as e:
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_batch_matmul_softmax():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, diff, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert diff == 0.0, f"rank {rank}: max |diff| {diff}"
