"""GPU, 2 ranks over NCCL (skipped with fewer than 2 GPUs): the sharded step
the bench runs.  Each rank runs its items of each round through the library's
launch layer, writing its slots of the full-size output, and the rounds are
all-gathered in place (any_gpu.dist.run_rounds).  Checked: every rank holds
the same bytes, and the whole result matches the oracle.  Covers batch_matmul
+ softmax in two rounds (GEMMs on one stream, softmaxes on another), an
uneven split (5 items over 2 ranks: in-place broadcasts), and attention
sharded by heads -- each through both gatherers: copy-engine pushes over CUDA
IPC (PeerGather, ending each step on device flag words or on interprocess
events) and in-place NCCL collectives (NcclGather)."""
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
    sys.path.insert(0, str(root))
    import datetime

    import torch
    import torch.distributed as dist
    from any_gpu import GpuDevice
    from any_gpu.dist import NcclGather, PeerGather, ShardPlan, run_rounds
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        host = dist.new_group(backend="gloo")
        dev = GpuDevice.gpu(rank)
        stream = torch.cuda.Stream()
        aux = torch.cuda.Stream()
        torch.cuda.set_stream(stream)
        results = {}

        # batch_matmul + softmax: (batch, rounds)
        m, n, k = 256, 512, 384
        for batch, rounds in ((8, 2), (5, 1)):
            r = np.random.default_rng(3 + batch)
            a = (r.standard_normal(batch * m * k) * 0.05).astype(np.float32)
            b = (r.standard_normal(batch * k * n) * 0.05).astype(np.float32)
            plan = ShardPlan(batch, world, rank, rounds)
            items = plan.my_items()
            A = torch.from_numpy(np.concatenate([a[g * m * k:(g + 1) * m * k]
                                                 for g in items])).cuda()
            B = torch.from_numpy(np.concatenate([b[g * k * n:(g + 1) * k * n]
                                                 for g in items])).cuda()

            def launch(rd, out):
                cnt = rd.counts[rank]
                c = out.data_ptr() + 4 * rd.offsets[rank] * m * n
                dev.launch_batch_matmul(A.data_ptr() + 4 * rd.local * m * k,
                                        B.data_ptr() + 4 * rd.local * k * n, c, cnt, m, n, k,
                                        stream.cuda_stream)
                ev = torch.cuda.Event()
                ev.record(stream)
                aux.wait_event(ev)
                dev.launch_softmax(c, c, cnt * m, n, aux.cuda_stream)
                return aux
            for kind in ("nccl", "ce", "ce_events"):
                out = torch.full((batch * m * n,), float("nan"), device="cuda")
                g = NcclGather(plan, out, m * n) if kind == "nccl" else \
                    PeerGather(dev, plan, out, m * n, host,
                               sync="events" if kind == "ce_events" else "flags")
                for _ in range(2):  # twice: the second step reuses the events and mappings
                    out.fill_(float("nan"))
                    stream.synchronize()
                    dist.barrier(group=host)
                    run_rounds(plan, lambda rd: launch(rd, out), stream, g)
                stream.synchronize()
                g.close()
                results[f"bmm{batch}_{kind}"] = (out.cpu().numpy(), a, b)

        # attention, heads split over the ranks in one round
        bh, s, d = 6, 256, 128
        r = np.random.default_rng(9)
        qkv = [r.standard_normal(bh * s * d).astype(np.float32) for _ in range(3)]
        plan = ShardPlan(bh, world, rank, 1)
        st, cnt = plan.spans[0].offsets[rank], plan.spans[0].counts[rank]
        Q, K, V = (torch.from_numpy(x[st * s * d:(st + cnt) * s * d]).cuda() for x in qkv)
        for kind in ("nccl", "ce"):
            O = torch.full((bh * s * d,), float("nan"), device="cuda")

            def launch_attn(rd):
                dev.launch_sdpa(Q.data_ptr(), K.data_ptr(), V.data_ptr(),
                                O.data_ptr() + 4 * st * s * d, cnt, s, d, False,
                                stream.cuda_stream)
                return stream
            g = NcclGather(plan, O, s * d) if kind == "nccl" else \
                PeerGather(dev, plan, O, s * d, host)
            run_rounds(plan, launch_attn, stream, g)
            stream.synchronize()
            g.close()
            results[f"sdpa_{kind}"] = (O.cpu().numpy(), *qkv)
        dev.synchronize()
        q.put((rank, results, None))
        torch.cuda.synchronize()
        dist.destroy_process_group()
        dev.close()
    except Exception as e:
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_rounds_gather_in_place(orc):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in procs), key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, _, err in res:
        assert err is None, f"rank {rank}: {err}"
    r0, r1 = res[0][1], res[1][1]
    m, n, k = 256, 512, 384
    for kind in ("nccl", "ce", "ce_events"):
        for batch in (8, 5):
            got0, a, b = r0[f"bmm{batch}_{kind}"]
            got1 = r1[f"bmm{batch}_{kind}"][0]
            assert np.array_equal(got0, got1), f"bmm{batch} {kind}: ranks hold different results"
            want = orc.softmax(orc.batch_matmul(a, b, batch, m, n, k), batch * m, n)
            assert orc.rel_fro(got0, want) <= 1e-3, kind
        if kind == "ce_events":
            continue
        got0, qh, kh, vh = r0[f"sdpa_{kind}"]
        assert np.array_equal(got0, r1[f"sdpa_{kind}"][0]), kind
        assert orc.rel_fro(got0, orc.attention(qh, kh, vh, 6, 256, 128)) <= 1e-3, kind
    # the gatherers move the same bytes
    assert np.array_equal(r0["bmm8_nccl"][0], r0["bmm8_ce"][0])
    assert np.array_equal(r0["bmm8_ce"][0], r0["bmm8_ce_events"][0])
