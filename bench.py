#!/usr/bin/env python
"""Benchmark of the B200 dense-op path (one JSON line on rank 0).

Headline (the default line): fp32 batch_matmul -> row softmax.
  One step = C = batch_matmul(A, B), batch 64, M = K = N = 2048, A, B ~ N(0,1)*0.05
  (seeded), then S = softmax(C) over the last dim (131072 rows x 2048).  The GEMM
  runs on tcgen05 tensor cores in TF32 (operands rounded to nearest by TMA) with
  fp32 accumulation; softmax is the one-read-one-write warp-per-row kernel.

`workloads` (same line, same N): every other benchmark configuration under the
same clock -- square matmul 512^3 (+ 1024, 2048, 4096, 8192, and 8192^3 in
3xTF32), scaled_dot_product_attention B8 H32 S2048 D128, the UNet block (conv2d
3x3 N16 320->320 64x64 -> group_norm 32 -> swish), the LLaMA-style decoder layer
(B32 S2048 d4096 H32x128 FFN 11008) -- each with its own value, roofline,
clocks, e2e and (at N = 1) CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl agpu|reference]
                    [--workload bmm_softmax|matmul|sdpa|unet|llama] [--replicas]

Multi-GPU (one process per GPU, torchrun for N > 1): the batched configs are
split across the ranks ("scaling": "strong"; the job is the same at every N).
Each rank computes its items and writes them into its slot of the full-size
output, and every rank ends with the whole result through in-place NCCL
all-gathers over NVLink, one per round of items, each issued as soon as its
round is done so that it runs beside the next round's compute (`comm` block:
bytes received, gathers alone, compute alone, exposed gather time).  Square
matmul is one item: it runs as replicas ("scaling": "weak").  `--replicas`
runs every config as full-size replicas with no collective.

  value    whole-job TFLOPS = job FLOPs / (max over ranks of the device time per
           step); inputs resident in HBM; CUDA events on the launching stream.
           Working sets exceed the 126 MB L2 (`config.l2`); the small matmul
           sizes say so and re-read their inputs from L2.
  e2e      the same FLOPs over the wall time of the public API with host buffers
           (pinned host inputs up, the ops, this rank's outputs down, every copy
           inside the step), max over ranks.
  roofline the dominant kernel's FLOP/s (CUDA events around its launches, in a
           loop of its own) against the TF32 dense peak = half the measured bf16
           peak (a third of that for 3xTF32).
  Inputs come from one seeded generator per (config, item), so a config's data
  do not depend on N.  matmul steps are microseconds of device work, less than
  a host enqueue takes: their K steps are timed as one CUDA graph.
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "any-gpu_b200"))
sys.path.insert(0, str(ROOT))

from any_gpu.dist import NcclGather, PeerGather, ShardPlan, run_rounds  # noqa: E402

METRIC = "TFLOPS (matmul, SDPA) and GB/s (softmax/norm) at 1/2/4/8 B200, % of roofline"

# DRAM bytes (read + write) of one launch of the dominant kernel over the
# config's full batch, from one ncu capture (dram__bytes_read.sum +
# dram__bytes_write.sum); where the capture ran a smaller case, scaled by the
# items processed.  A launch over part of the batch scales it by its items.
TRAFFIC_BYTES = {
    "bmm_softmax": 3.5e9,   # pair GEMM, batch-8 capture x 8
    "sdpa": 0.99e9,         # attention_pair_kernel, 64-head capture x 4
    "unet": 1.21e8,         # conv kernel, full workload
    "llama": 2.39e10,       # gate/up GEMM, batch-2 capture x 16
    "matmul512": 2.13e6,    # split-K GEMM at 512^3, full capture (C stays in L2)
}

PRECISION_NOTE = {
    "tf32": "tf32 multiply (operands rounded to nearest), fp32 accumulate, fp32 I/O",
    "tf32x3": "3xTF32 (hi/lo split, three tcgen05 products), fp32 accumulate, fp32 I/O",
}


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ------------------------------------------------------------- clocks ----
REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
           0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
           0x2: "applications_clocks_setting", 0x10: "sync_boost"}


class ClockSampler(threading.Thread):
    """Samples SM clock and clock-event reasons every 20 ms via NVML."""

    def __init__(self, cuda_index: int):
        super().__init__(daemon=True)
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._halt = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            try:
                import torch
                p = torch.cuda.get_device_properties(cuda_index)
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self._h = h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: record nothing, say so
            self.error = str(e)

    def run(self):
        if self._h is None:
            return
        nv = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self._halt.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = get_reasons(self._h)
                for bit, name in REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._halt.wait(0.02)

    def stop(self) -> dict:
        self._halt.set()
        self.join(timeout=2)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def item_rng(seed: int, item: int) -> np.random.Generator:
    """One generator per (config seed, global item index): a config's inputs are
    the same whatever the number of ranks that share it."""
    return np.random.default_rng([seed, item])


def _normal_into(r, out, scale=1.0):
    r.standard_normal(out=out, dtype=np.float32)
    if scale != 1.0:
        out *= np.float32(scale)


def _cores(orc, threads):
    """Host threads a CPU sample uses: all of the oracle's pool, or one."""
    return max(1, orc.num_threads()) if threads else 1


# ----------------------------------------------------------- workloads ---
class Workload:
    """One benchmark configuration: `total` independent items (batch items,
    heads, images, sequences) of `item_flops` each, split across the ranks by
    a ShardPlan.  Subclasses fill the inputs of one item, launch one round of
    this rank's items on a stream (launch layer, caller memory), and define
    the dominant kernel's own loop and the public-API e2e step."""
    name = ""
    precision = "tf32"
    l2 = ""
    item = "item"
    seed = 0
    round_items = 8        # this rank's items per round of the sharded step
    shardable = True
    graph_default = False  # time the K steps as one CUDA graph (latency-bound steps)
    dom_kernel = ""
    item_elems: dict = {}  # per-item input name -> elements
    out_item = 0           # output elements per item
    item_flops = 0.0
    dom_item_flops = 0.0   # the dominant kernel's FLOPs per item (0: item_flops)

    def __init__(self, args, world, rank, replicas=False):
        self.args, self.world, self.rank = args, world, rank
        self.total = self.total_items()
        self.sharded = world > 1 and self.shardable and not replicas
        w, r = (world, rank) if self.sharded else (1, 0)
        rounds = 1
        if self.sharded:
            per_rank = self.total // world
            rounds = max(1, per_rank // self.round_items)
            if args.rounds:
                rounds = max(1, min(args.rounds, per_rank))
        self.plan = ShardPlan(self.total, w, r, rounds)
        self.local = self.plan.my_count
        self.job_items = self.total if (self.sharded or world == 1) else self.total * world
        self.flops = self.job_items * self.item_flops
        # FLOPs of the dominant kernel's launch over this rank's items
        self.dom_flops = self.local * (self.dom_item_flops or self.item_flops)

    # ---- description
    def total_items(self) -> int:
        raise NotImplementedError

    def config(self) -> dict:
        raise NotImplementedError

    @property
    def dtype(self) -> str:
        return self.precision

    def scaling(self) -> str:
        return "weak" if (self.world > 1 and not self.sharded) else "strong"

    def parallelism(self) -> str:
        if self.world == 1:
            return "single"
        return f"shard{self.world}" if self.sharded else f"replicas{self.world}"

    def full_config(self) -> dict:
        cfg = self.config()
        cfg.update({"parallelism": self.parallelism(), "l2": self.l2,
                    "items": f"{self.total} {self.item}s",
                    "rounds": len(self.plan.spans) if self.sharded else 1})
        if self.sharded:
            cfg["gather"] = self.args.comm
        return cfg

    # ---- data
    def fill_item(self, g: int, views: dict) -> None:
        raise NotImplementedError

    def shared_inputs(self) -> dict:
        return {}

    def setup(self, torch, local):
        """Pinned host inputs of this rank's items (one seeded generator per
        item), their device copies, and the full-size device output."""
        items = self.plan.my_items()
        self.host = {}
        for k, n in self.item_elems.items():
            self.host[k] = torch.empty(len(items) * n, dtype=torch.float32, pin_memory=True)
        for j, g in enumerate(items):
            self.fill_item(g, {k: self.host[k].numpy()[j * n:(j + 1) * n]
                               for k, n in self.item_elems.items()})
        for k, v in self.shared_inputs().items():
            t = torch.empty(v.size, dtype=torch.float32, pin_memory=True)
            t.numpy()[:] = v
            self.host[k] = t
        dev = f"cuda:{local}"
        self.d = {k: v.to(dev) for k, v in self.host.items()}
        self.out = torch.empty(self.total * self.out_item, dtype=torch.float32, device=dev)
        self.out_host = torch.empty(self.local * self.out_item, dtype=torch.float32,
                                    pin_memory=True)
        self.aux = torch.cuda.Stream(device=local)

    def make_gatherer(self, dev, ctx):
        """The round gatherer of a sharded step: copy-engine pushes over CUDA
        IPC (`--comm ce`, default) or in-place NCCL collectives (`--comm nccl`)."""
        self.gatherer = None
        if self.sharded:
            self.gatherer = (PeerGather(dev, self.plan, self.out, self.out_item, ctx.host_group,
                                        ctx.args.ce_streams, ctx.args.ce_sync)
                             if ctx.args.comm == "ce" else
                             NcclGather(self.plan, self.out, self.out_item))

    def teardown(self):
        if getattr(self, "gatherer", None) is not None:
            self.gatherer.close()
        for k in ("host", "d", "out", "out_host", "aux", "_pipe", "_scratch", "gatherer"):
            if hasattr(self, k):
                delattr(self, k)

    def ptr(self, name, item_off=0):
        return self.d[name].data_ptr() + 4 * item_off * self.item_elems[name]

    def out_ptr(self, global_item):
        return self.out.data_ptr() + 4 * global_item * self.out_item

    # ---- device steps
    def launch_round(self, dev, rd, stream):
        """Enqueue this rank's items of round `rd` (writing their output slots);
        return the stream on which that output is complete."""
        raise NotImplementedError

    def step(self, dev, stream, gather=True):
        run_rounds(self.plan, lambda rd: self.launch_round(dev, rd, stream), stream,
                   self.gatherer if gather else None)

    def gather_only(self, stream):
        run_rounds(self.plan, lambda rd: stream, stream, self.gatherer)

    def dom_step(self, dev, stream):
        raise NotImplementedError

    def checksum(self, torch) -> dict:
        o = self.out
        nrm = float(torch.linalg.vector_norm(o, dtype=torch.float64))
        return {"sum": float(o.sum(dtype=torch.float64)), "sum_sq": nrm * nrm,
                "elems": o.numel(),
                "note": "float64 sum and sum of squares of the whole gathered output, "
                        "taken after the timed steps"}

    # ---- end to end
    def e2e_bytes(self):
        h2d = sum(v.numel() * 4 for v in self.host.values())
        return h2d, self.local * self.out_item * 4

    def e2e_step(self, dev):
        raise NotImplementedError

    def _pipelined(self, dev, chunked, shared, chunks, launch):
        """One e2e step with its PCIe transfers pipelined over the async API:
        `shared` host inputs go up whole first; per chunk i the `chunked`
        inputs' i-th slices go up on an upload stream, `launch(i, ptrs,
        stream)` runs on a compute stream once they are there, and the
        output's i-th slice comes down on a download stream."""
        import torch
        if not hasattr(self, "_pipe"):
            bufs = {k: dev.alloc(self.host[k].numel()) for k in list(chunked) + list(shared)}
            bufs["_out"] = dev.alloc(self.local * self.out_item)
            dev.synchronize()  # the zero fills finish before other streams write
            self._pipe = (bufs, [torch.cuda.Stream() for _ in range(3)])
        bufs, (up, comp, down) = self._pipe
        ptrs = {k: b.device_ptr for k, b in bufs.items()}
        for k in shared:
            n = self.host[k].numel()
            dev.write_async(bufs[k], self.host[k].data_ptr(), n, 0, up.cuda_stream)
        per_out = self.local * self.out_item // chunks
        for i in range(chunks):
            for k in chunked:
                n = self.host[k].numel() // chunks
                dev.write_async(bufs[k], self.host[k].data_ptr() + 4 * i * n, n, i * n,
                                up.cuda_stream)
            e_up = torch.cuda.Event()
            e_up.record(up)
            comp.wait_event(e_up)
            launch(i, ptrs, comp.cuda_stream)
            e_c = torch.cuda.Event()
            e_c.record(comp)
            down.wait_event(e_c)
            dev.read_async(bufs["_out"], self.out_host.data_ptr() + 4 * i * per_out, per_out,
                           i * per_out, down.cuda_stream)
        down.synchronize()
        dev.synchronize()  # surfaces an expired device-side wait, if any

    def e2e_chunks(self, options):
        return next(c for c in options if self.local % c == 0)

    def cpu_sample(self, orc, target_s, threads=True):
        raise NotImplementedError

    def extra(self, ms_step, ms_dom, peaks, aux_ms=None) -> dict:
        return {}

    def traffic(self):
        t = TRAFFIC_BYTES.get(self.name)
        if t is None or not self.default_size():
            return None
        return t * self.local / self.total

    def default_size(self) -> bool:
        return False


class BmmSoftmax(Workload):
    name = "bmm_softmax"
    l2 = "inputs 2 GiB + output 1 GiB > 126 MB L2 (no flush needed)"
    item = "batch item"
    seed = 1235
    # 8 items per round: at N = 8 one round, whose 128 MiB copies per peer
    # reach 712 GB/s received; 4 rounds of 32 MiB copies measured 545 against
    # 655 TFLOPS (their gathers slower by more than the compute they hide)
    round_items = 8
    M = N = K = 2048
    item_elems = {"a": M * K, "b": K * N}
    out_item = M * N
    item_flops = 2.0 * M * N * K
    dom_kernel = ("umma_tf32_pair_kernel<GemmPairPolicy<K-major A, MN-major B>> "
                  "(256x256 CTA-pair tiles)")

    def total_items(self):
        return self.args.batch

    def default_size(self):
        return self.args.batch == 64

    def config(self):
        return {"workload": "batch_matmul+softmax", "batch": self.total, "m": self.M,
                "n": self.N, "k": self.K, "inputs": "N(0,1)*0.05 seeded per batch item",
                "softmax_rows": self.total * self.M, "softmax_cols": self.N}

    def fill_item(self, g, v):
        r = item_rng(self.seed, g)
        _normal_into(r, v["a"], 0.05)
        _normal_into(r, v["b"], 0.05)

    def launch_round(self, dev, rd, stream):
        import torch
        n = rd.counts[self.plan.rank]
        if n == 0:
            return stream
        M, N, K = self.M, self.N, self.K
        a, b = self.ptr("a", rd.local), self.ptr("b", rd.local)
        c = self.out_ptr(rd.offsets[self.plan.rank])
        if len(self.plan.spans) == 1:
            # one round: the fused entry point (its own pieces, each piece's
            # softmax beside the next piece's GEMM)
            dev.launch_batch_matmul_softmax(a, b, c, n, M, N, K, stream.cuda_stream)
            return stream
        # rounds: GEMMs back to back on `stream`, each round's softmax (in
        # place) on the aux stream, whose tail then starts the round's gather
        dev.launch_batch_matmul(a, b, c, n, M, N, K, stream.cuda_stream)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.aux.wait_event(ev)
        dev.launch_softmax(c, c, n * M, N, self.aux.cuda_stream)
        return self.aux

    def dom_step(self, dev, stream):
        dev.launch_batch_matmul(self.ptr("a"), self.ptr("b"), self.out.data_ptr(), self.local,
                                self.M, self.N, self.K, stream.cuda_stream)

    def aux_step(self, dev, stream):
        p = self.out.data_ptr()
        dev.launch_softmax(p, p, self.local * self.M, self.N, stream.cuda_stream)

    def e2e_step(self, dev):
        ga, gb = dev.upload(self.host["a"].numpy()), dev.upload(self.host["b"].numpy())
        gc = dev.batch_matmul(ga, gb, self.local, self.M, self.N, self.K)
        gs = dev.softmax(gc, self.local * self.M, self.N)
        dev.read(gs, out=self.out_host.numpy())
        for b in (ga, gb, gc, gs):
            b.free()

    def e2e_pipelined(self, dev):
        chunks = self.e2e_chunks((16, 8, 4, 2, 1))
        per = self.local // chunks
        M, N, K = self.M, self.N, self.K
        self.e2e_how = (f"this rank's {self.local} batch items in {chunks} chunks; per chunk "
                        "agpu_write_async of A and B on an upload stream, batch_matmul + "
                        "softmax (launch layer) on a compute stream, agpu_read_async of S on "
                        "a download stream: PCIe both ways overlapped")

        def launch(i, p, st):
            oa, ob, oc = 4 * i * per * M * K, 4 * i * per * K * N, 4 * i * per * M * N
            dev.launch_batch_matmul(p["a"] + oa, p["b"] + ob, p["_out"] + oc, per, M, N, K, st)
            dev.launch_softmax(p["_out"] + oc, p["_out"] + oc, per * M, N, st)
        self._pipelined(dev, ["a", "b"], [], chunks, launch)

    def cpu_sample(self, orc, target_s, threads=True):
        if not hasattr(self, "_cpu_in"):
            self._cpu_in = {k: np.empty(n, np.float32) for k, n in self.item_elems.items()}
            self.fill_item(0, self._cpu_in)
        a, b = self._cpu_in["a"], self._cpu_in["b"]
        M, N, K = self.M, self.N, self.K
        chunk, done, t, start = max(16, 2 * _cores(orc, threads)), 0, 0.0, 0
        while t < target_s:
            rows = min(chunk, M - start)
            t0 = time.perf_counter()
            c = orc.matmul(a[start * K:(start + rows) * K], b, rows, N, K, threads=threads)
            orc.softmax(c, rows, N, threads=threads)
            t += time.perf_counter() - t0
            done += rows
            start = (start + rows) % M
        return 2.0 * done * N * K / t / 1e12, (
            f"{done} rows of batch item 0 (each: a 1x{K} by {K}x{N} matmul row + its "
            f"softmax), {t:.1f} s, extrapolated by FLOPs")

    def extra(self, ms_step, ms_dom, peaks, aux_ms=None):
        nbytes = 2.0 * self.local * self.M * self.N * 4
        gbs = nbytes / (aux_ms * 1e-3) / 1e9
        return {"softmax": {"ms": aux_ms, "gbs": gbs, "frac_hbm": gbs / peaks["hbm_gbs"],
                            "note": f"softmax_warp_kernel alone over this rank's "
                                    f"{self.local * self.M} x {self.N} rows (8 B per element, "
                                    "of measured HBM copy bandwidth)"}}


class Matmul(Workload):
    name = "matmul"
    graph_default = True
    shardable = False
    item = "matrix"
    seed = 1234

    def __init__(self, args, world, rank, replicas=False, size=None, precision=None):
        self.n = size or args.size
        self.precision = precision or args.precision
        n = self.n
        self.item_elems = {"a": n * n, "b": n * n}
        self.out_item = n * n
        self.item_flops = 2.0 * n ** 3
        super().__init__(args, world, rank, replicas)
        self.dom_kernel = (
            "umma_tf32_kernel<GemmPolicy<128|256, 3xTF32>> (single CTA, K segments)"
            if self.precision == "tf32x3" and n < 256 else
            "umma_x3_pair_kernel<GemmPairX3Policy<256>> (CTA pairs, K segments summed in TMEM)"
            if self.precision == "tf32x3" else
            "umma_tf32_kernel<GemmPolicy<128|256>> (single CTA)" if n < 256 else
            "umma_tf32_pair_splitk_kernel<GemmPairPolicy<256|128>, 4|2> (cluster split-K)"
            if n <= 1024 else "umma_tf32_pair_kernel<GemmPairPolicy<256|512>>")
        ws = 3 * n * n * 4
        self.l2 = (f"working set {ws / 2**20:.1f} MiB "
                   + ("> 126 MB L2" if ws > 126e6 else "fits in L2: inputs re-read from L2"))

    def total_items(self):
        return 1

    def default_size(self):
        return self.n == 512 and self.precision == "tf32"

    def traffic(self):
        return TRAFFIC_BYTES["matmul512"] if self.default_size() else None

    def config(self):
        return {"workload": "matmul", "m": self.n, "n": self.n, "k": self.n,
                "inputs": "U[-1,1) seeded",
                "timing": "K steps captured in one CUDA graph" if self.args.graph is not False
                else "K steps launched from the host"}

    def fill_item(self, g, v):
        r = item_rng(self.seed, g)
        for k in ("a", "b"):
            r.random(out=v[k], dtype=np.float32)
            v[k] *= np.float32(2.0)
            v[k] -= np.float32(1.0)

    def launch_round(self, dev, rd, stream):
        dev.launch_batch_matmul(self.ptr("a"), self.ptr("b"), self.out.data_ptr(), 1, self.n,
                                self.n, self.n, stream.cuda_stream)
        return stream

    def dom_step(self, dev, stream):
        self.launch_round(dev, None, stream)

    def e2e_step(self, dev):
        ga, gb = dev.upload(self.host["a"].numpy()), dev.upload(self.host["b"].numpy())
        gc = dev.matmul(ga, gb, self.n, self.n, self.n)
        dev.read(gc, out=self.out_host.numpy())
        for b in (ga, gb, gc):
            b.free()

    def cpu_sample(self, orc, target_s, threads=True):
        if not hasattr(self, "_cpu_in"):
            self._cpu_in = {k: np.empty(e, np.float32) for k, e in self.item_elems.items()}
            self.fill_item(0, self._cpu_in)
        a, b, n = self._cpu_in["a"], self._cpu_in["b"], self.n
        chunk, done, t, start = max(8, _cores(orc, threads)), 0, 0.0, 0
        while t < target_s:
            rows = min(chunk, n - start)
            t0 = time.perf_counter()
            orc.matmul(a[start * n:(start + rows) * n], b, rows, n, n, threads=threads)
            t += time.perf_counter() - t0
            done += rows
            start = (start + rows) % n
        return 2.0 * done * n * n / t / 1e12, (f"{done} rows of the {n}^3 product "
                                               f"(cpu_matmul), {t:.1f} s")


class Sdpa(Workload):
    name = "sdpa"
    l2 = "Q, K, V, O 1 GiB > 126 MB L2"
    item = "head"
    seed = 1236
    round_items = 64
    D = 128
    dom_kernel = "attention_pair_kernel<128, non-causal> (CTA-pair flash attention)"

    def __init__(self, args, world, rank, replicas=False):
        self.s = args.seq
        hs = self.s * self.D
        self.item_elems = {"q": hs, "k": hs, "v": hs}
        self.out_item = hs
        self.item_flops = 4.0 * self.s * self.s * self.D
        super().__init__(args, world, rank, replicas)

    def total_items(self):
        return self.args.bh

    def default_size(self):
        return self.args.bh == 256 and self.args.seq == 2048

    def config(self):
        return {"workload": "scaled_dot_product_attention", "batch_heads": self.total,
                "seq_len": self.s, "d_k": self.D, "causal": False,
                "inputs": "N(0,1) seeded per head", "flops": "4*BH*S^2*D (QK^T + PV)"}

    def fill_item(self, g, v):
        r = item_rng(self.seed, g)
        for k in ("q", "k", "v"):
            _normal_into(r, v[k])

    def launch_round(self, dev, rd, stream):
        n = rd.counts[self.plan.rank]
        if n:
            dev.launch_sdpa(self.ptr("q", rd.local), self.ptr("k", rd.local),
                            self.ptr("v", rd.local), self.out_ptr(rd.offsets[self.plan.rank]),
                            n, self.s, self.D, False, stream.cuda_stream)
        return stream

    def dom_step(self, dev, stream):
        dev.launch_sdpa(self.ptr("q"), self.ptr("k"), self.ptr("v"), self.out.data_ptr(),
                        self.local, self.s, self.D, False, stream.cuda_stream)

    def e2e_step(self, dev):
        g = [dev.upload(self.host[n].numpy()) for n in "qkv"]
        go = dev.scaled_dot_product_attention(*g, self.local, self.s, self.D)
        dev.read(go, out=self.out_host.numpy())
        for b in g + [go]:
            b.free()

    def e2e_pipelined(self, dev):
        chunks = self.e2e_chunks((8, 4, 2, 1))
        per = self.local // chunks
        hsz = self.s * self.D
        self.e2e_how = (f"this rank's {self.local} heads in {chunks} chunks; per chunk "
                        "agpu_write_async of Q, K, V on an upload stream, attention (launch "
                        "layer) on a compute stream, agpu_read_async of O on a download stream")

        def launch(i, p, st):
            off = 4 * i * per * hsz
            dev.launch_sdpa(p["q"] + off, p["k"] + off, p["v"] + off, p["_out"] + off, per,
                            self.s, self.D, False, st)
        self._pipelined(dev, ["q", "k", "v"], [], chunks, launch)

    def cpu_sample(self, orc, target_s, threads=True):
        heads = _cores(orc, threads)
        hsz = self.s * self.D
        q, k, v = (np.empty(heads * hsz, np.float32) for _ in range(3))
        for h in range(heads):
            self.fill_item(h, {"q": q[h * hsz:(h + 1) * hsz], "k": k[h * hsz:(h + 1) * hsz],
                               "v": v[h * hsz:(h + 1) * hsz]})
        done, t = 0, 0.0
        while t < target_s:
            t0 = time.perf_counter()
            orc.attention(q, k, v, heads, self.s, self.D, threads=threads)
            t += time.perf_counter() - t0
            done += heads
        return (4.0 * done * self.s * self.s * self.D / t / 1e12,
                f"{done} heads of S={self.s}, D={self.D} (cpu_attention per head), {t:.1f} s")


class SdpaBwd(Workload):
    """Attention backward (agpu_launch_sdpa_backward) at the SDPA config: dQ,
    dK, dV from Q, K, V, dO; FLOPs counted as its five products
    (S = QK^T recomputed, dV = P^T dO, dP = dO V^T, dQ = dS K, dK = dS^T Q),
    5 * 2 * BH * S^2 * D.  Three outputs: runs as replicas at N > 1."""
    name = "sdpa_bwd"
    l2 = "Q, K, V, dO, dQ, dK, dV 1.75 GiB + P, dS scratch 8 GiB > 126 MB L2"
    item = "head"
    seed = 1240
    shardable = False
    D = 128
    dom_kernel = ("umma_tf32_pair_kernel<GemmPairPolicy> (the five products; timed as the "
                  "whole backward call)")

    def __init__(self, args, world, rank, replicas=False):
        self.s = args.seq
        hs = self.s * self.D
        self.item_elems = {"q": hs, "k": hs, "v": hs, "do": hs}
        self.out_item = hs
        self.item_flops = 5 * 2.0 * self.s * self.s * self.D
        super().__init__(args, world, rank, replicas)

    def total_items(self):
        return self.args.bh

    def config(self):
        return {"workload": "scaled_dot_product_attention backward", "batch_heads": self.total,
                "seq_len": self.s, "d_k": self.D, "causal": False,
                "inputs": "Q, K, V, dO N(0,1) seeded per head",
                "flops": "5 * 2*BH*S^2*D (S recomputed, dV, dP, dQ, dK)"}

    def fill_item(self, g, v):
        r = item_rng(self.seed, g)
        for k in ("q", "k", "v", "do"):
            _normal_into(r, v[k])

    def setup(self, torch, local):
        super().setup(torch, local)
        n = self.total * self.out_item
        self.dk = torch.empty(n, dtype=torch.float32, device=f"cuda:{local}")
        self.dv = torch.empty_like(self.dk)

    def teardown(self):
        super().teardown()
        for k in ("dk", "dv"):
            if hasattr(self, k):
                delattr(self, k)

    def launch_round(self, dev, rd, stream):
        dev.launch_sdpa_backward(self.ptr("q"), self.ptr("k"), self.ptr("v"), self.ptr("do"),
                                 self.out.data_ptr(), self.dk.data_ptr(), self.dv.data_ptr(),
                                 self.total, self.s, self.D, False, stream.cuda_stream)
        return stream

    def dom_step(self, dev, stream):
        self.launch_round(dev, None, stream)

    def e2e_bytes(self):
        h2d = sum(v.numel() * 4 for v in self.host.values())
        return h2d, 3 * self.total * self.out_item * 4

    def e2e_step(self, dev):
        g = [dev.upload(self.host[n].numpy()) for n in ("q", "k", "v", "do")]
        outs = dev.sdpa_backward(*g, self.total, self.s, self.D)
        for b in outs:
            dev.read(b, out=self.out_host.numpy())
        for b in g + list(outs):
            b.free()

    def cpu_sample(self, orc, target_s, threads=True):
        hs = self.s * self.D
        x = {k: np.empty(hs, np.float32) for k in ("q", "k", "v", "do")}
        self.fill_item(0, x)
        done, t = 0, 0.0
        while t < target_s:
            t0 = time.perf_counter()
            orc.attention_backward(x["q"], x["k"], x["v"], x["do"], 1, self.s, self.D)
            t += time.perf_counter() - t0
            done += 1
        return (self.item_flops * done / t / 1e12,
                f"{done} head(s) of S={self.s}, D={self.D} (the reference's SDPA composition "
                f"differentiated with its own rules, one head), {t:.1f} s")


class Unet(Workload):
    name = "unet"
    l2 = "x 80 MiB + conv out 80 MiB + y 80 MiB > 126 MB L2"
    item = "image"
    seed = 1237
    round_items = 4
    C, H, W, G = 320, 64, 64, 32
    item_elems = {"x": C * H * W}
    out_item = C * H * W
    item_flops = 2.0 * C * H * W * C * 9
    dom_kernel = ("umma_tf32_pair_kernel<ConvPairPolicy<320>> (implicit-GEMM conv2d, "
                  "staging included; timed in a separate loop of conv2d calls)")

    def total_items(self):
        return self.args.images

    def default_size(self):
        return self.args.images == 16

    def config(self):
        return {"workload": "unet_block conv2d3x3->group_norm->swish", "n": self.total,
                "cin": self.C, "cout": self.C, "h": self.H, "w": self.W, "groups": self.G,
                "eps": 1e-5, "inputs": "x N(0,1) seeded per image; W Kaiming-uniform "
                "U(+-sqrt(6/2880)); bias 0", "flops": "conv only: 2*N*Cout*H*W*Cin*9"}

    def fill_item(self, g, v):
        _normal_into(item_rng(self.seed, g), v["x"])

    def shared_inputs(self):
        r = np.random.default_rng([self.seed, 1 << 20])
        bound = np.float32(np.sqrt(6.0 / (self.C * 9)))
        return {"w": r.uniform(-bound, bound, self.C * self.C * 9).astype(np.float32),
                "gamma": np.ones(self.C, np.float32), "beta": np.zeros(self.C, np.float32)}

    def _block(self, dev, x, y, n, st):
        d = self.d
        dev.launch_conv2d_group_norm_swish(
            x, d["w"].data_ptr(), 0, y, n, self.C, self.H, self.W, self.C, 3, 3, 1, 1, 1, 1, 1,
            1, 1, d["gamma"].data_ptr(), d["beta"].data_ptr(), self.G, 1e-5, st)

    def launch_round(self, dev, rd, stream):
        n = rd.counts[self.plan.rank]
        if n:
            self._block(dev, self.ptr("x", rd.local), self.out_ptr(rd.offsets[self.plan.rank]),
                        n, stream.cuda_stream)
        return stream

    def dom_step(self, dev, stream):
        d = self.d
        dev.launch_conv2d(d["x"].data_ptr(), d["w"].data_ptr(), 0, self.out.data_ptr(),
                          self.local, self.C, self.H, self.W, self.C, 3, 3, 1, 1, 1, 1, 1, 1, 1,
                          stream.cuda_stream)

    def aux_step(self, dev, stream):
        d = self.d
        p = self.out.data_ptr()
        dev.launch_group_norm(p, d["gamma"].data_ptr(), d["beta"].data_ptr(), p, self.local,
                              self.C, self.H * self.W, self.G, 1e-5, True, stream.cuda_stream)

    def e2e_step(self, dev):
        g = {k: dev.upload(v.numpy()) for k, v in self.host.items()}
        y = dev.conv2d_group_norm_swish(g["x"], g["w"], None, self.local, self.C, self.H, self.W,
                                        self.C, 3, 3, (1, 1), (1, 1), (1, 1), 1, gamma=g["gamma"],
                                        beta=g["beta"], gn_groups=self.G, eps=1e-5)
        dev.read(y, out=self.out_host.numpy())
        for b in list(g.values()) + [y]:
            b.free()

    def e2e_pipelined(self, dev):
        chunks = self.e2e_chunks((4, 2, 1))
        per = self.local // chunks
        img = self.C * self.H * self.W
        self.e2e_how = (f"this rank's {self.local} images in {chunks} chunks; the weights, "
                        "then per chunk the images, up by agpu_write_async on an upload "
                        "stream, the fused conv2d -> group_norm -> swish (launch layer) on a "
                        "compute stream, agpu_read_async of the output on a download stream")

        def launch(i, p, st):
            off = 4 * i * per * img
            dev.launch_conv2d_group_norm_swish(
                p["x"] + off, p["w"], 0, p["_out"] + off, per, self.C, self.H, self.W, self.C,
                3, 3, 1, 1, 1, 1, 1, 1, 1, p["gamma"], p["beta"], self.G, 1e-5, st)
        self._pipelined(dev, ["x"], ["w", "gamma", "beta"], chunks, launch)

    def cpu_sample(self, orc, target_s, threads=True):
        img = self.C * self.H * self.W
        x = np.empty(img, np.float32)
        self.fill_item(0, {"x": x})
        s = self.shared_inputs()
        done, t = 0, 0.0
        while t < target_s:
            t0 = time.perf_counter()
            y = orc.conv2d(x, s["w"], None, 1, self.C, self.H, self.W, self.C, 3, 3, (1, 1),
                           (1, 1), (1, 1), 1, threads=threads)
            y = orc.group_norm(y, s["gamma"], s["beta"], 1, self.C, self.H * self.W, self.G,
                               1e-5, threads=threads)
            orc.elementwise("swish", y)
            t += time.perf_counter() - t0
            done += 1
        return (2.0 * done * img * self.C * 9 / t / 1e12,
                f"{done} image(s) of the block (cpu_conv2d + cpu_group_norm + swish), {t:.1f} s")

    def extra(self, ms_step, ms_dom, peaks, aux_ms=None):
        n = self.local * self.out_item
        nbytes, pbytes = 8.0 * n, 12.0 * n
        gbs, pgbs = nbytes / (aux_ms * 1e-3) / 1e9, pbytes / (aux_ms * 1e-3) / 1e9
        return {"group_norm_swish": {
            "ms": aux_ms, "gbs": gbs, "frac_hbm": gbs / peaks["hbm_gbs"],
            "gbs_per_pass": pgbs, "frac_hbm_per_pass": pgbs / peaks["hbm_gbs"],
            "exposed_ms": ms_step - ms_dom,
            "note": "ms: the group norm + swish alone (two kernels); gbs counts 8 B per "
                    "element (x read once, y written once), gbs_per_pass the 12 B per element "
                    "the two passes move; exposed_ms: step time minus conv time, the part the "
                    "fused step does not hide behind the conv"}}


class Llama(Workload):
    name = "llama"
    l2 = "activations ~19 GB > 126 MB L2"
    item = "sequence"
    seed = 1239
    round_items = 2
    dom_kernel = "umma_tf32_pair_kernel<GemmPairPolicy<K-major A, MN-major B>> (gate/up, SwiGLU)"

    def __init__(self, args, world, rank, replicas=False):
        from any_gpu.llama import LlamaDims
        self.LlamaDims = LlamaDims
        one = LlamaDims(batch=1, seq=2048, d_model=4096, heads=32, ffn=11008)
        self.one = one
        self.item_elems = {"x": one.seq * one.d_model}
        self.out_item = one.seq * one.d_model
        self.item_flops = one.gemm_flops() + one.attention_flops()
        self.dom_item_flops = 2.0 * one.tokens * one.d_model * 2 * one.ffn  # gate/up GEMM
        super().__init__(args, world, rank, replicas)

    def dims(self, batch):
        o = self.one
        return self.LlamaDims(batch=batch, seq=o.seq, d_model=o.d_model, heads=o.heads,
                              ffn=o.ffn)

    def total_items(self):
        return self.args.llama_batch

    def default_size(self):
        return self.args.llama_batch == 32

    def config(self):
        dm = self.one
        return {"workload": "llama_decoder_layer_forward", "batch": self.total, "seq": dm.seq,
                "d_model": dm.d_model, "heads": dm.heads, "head_dim": dm.head_dim,
                "ffn": dm.ffn, "rope_base": dm.rope_base, "causal": dm.causal,
                "inputs": "x N(0,1) seeded per sequence; W N(0,0.02); norm weights 1",
                "flops": "2*T*(4d^2+3dF) + 4*B*H*S^2*Dh"}

    def fill_item(self, g, v):
        _normal_into(item_rng(self.seed, g), v["x"])

    def shared_inputs(self):
        d, Fd = self.one.d_model, self.one.ffn
        r = np.random.default_rng([self.seed, 1 << 20])
        out = {"attn_norm": np.ones(d, np.float32), "ffn_norm": np.ones(d, np.float32)}
        for k, n in (("wqkv", d * 3 * d), ("wo", d * d), ("wgu", d * 2 * Fd), ("wd", Fd * d)):
            w = np.empty(n, np.float32)
            _normal_into(r, w, 0.02)
            out[k] = w
        return out

    def setup(self, torch, local):
        super().setup(torch, local)
        per_round = max(r.counts[self.plan.rank] for r in self.plan.spans)
        self.ws = {k: torch.empty(n, dtype=torch.float32, device=f"cuda:{local}")
                   for k, n in self.dims(max(1, per_round)).workspace_elems().items()}

    def teardown(self):
        super().teardown()
        if hasattr(self, "ws"):
            del self.ws

    def _weights(self):
        return {k: v.data_ptr() for k, v in self.d.items() if k != "x"}

    def launch_round(self, dev, rd, stream):
        from any_gpu.llama import layer_forward
        n = rd.counts[self.plan.rank]
        if n:
            ws = {k: v.data_ptr() for k, v in self.ws.items()}
            layer_forward(dev, self.dims(n), self.ptr("x", rd.local), self._weights(), ws,
                          self.out_ptr(rd.offsets[self.plan.rank]), stream.cuda_stream)
        return stream

    def dom_step(self, dev, stream):
        # the gate/up GEMM with its SwiGLU epilogue over all of this rank's
        # tokens: A = rmsnorm output [T, d], C = [T, F]
        import torch
        dm = self.dims(self.local)
        if not hasattr(self, "_scratch"):
            self._scratch = (torch.empty(dm.tokens * dm.d_model, device=self.out.device),
                             torch.empty(dm.tokens * dm.ffn, device=self.out.device))
        h, a = self._scratch
        dev.launch_gemm_ex(h.data_ptr(), self.d["wgu"].data_ptr(), a.data_ptr(), 1, dm.tokens,
                           2 * dm.ffn, dm.d_model, act=3, stream=stream.cuda_stream)

    def e2e_step(self, dev):
        from any_gpu.llama import layer_forward
        dm = self.dims(self.local)
        g = {k: dev.upload(v.numpy()) for k, v in self.host.items()}
        ws = {k: dev.alloc(n) for k, n in dm.workspace_elems().items()}
        y = dev.alloc(self.local * self.out_item)
        layer_forward(dev, dm, g["x"].device_ptr,
                      {k: b.device_ptr for k, b in g.items() if k != "x"},
                      {k: b.device_ptr for k, b in ws.items()}, y.device_ptr)
        dev.read(y, out=self.out_host.numpy())
        for b in list(g.values()) + list(ws.values()) + [y]:
            b.free()

    def cpu_sample(self, orc, target_s, threads=True):
        d = self.one.d_model
        r = np.random.default_rng([self.seed, 1])
        x = np.empty(64 * d, np.float32)
        _normal_into(r, x)
        wqkv = np.empty(d * 3 * d, np.float32)
        _normal_into(r, wqkv, 0.02)
        done, t = 0, 0.0
        rows = max(8, _cores(orc, threads))
        while t < target_s:
            t0 = time.perf_counter()
            orc.matmul(x[: rows * d], wqkv, rows, 3 * d, d, threads=threads)
            t += time.perf_counter() - t0
            done += rows
        return (2.0 * done * d * 3 * d / t / 1e12,
                f"{done} token rows of the Wqkv projection (cpu_matmul), {t:.1f} s, "
                "the layer's dominant op, extrapolated by FLOPs")


WORKLOADS = {"bmm_softmax": BmmSoftmax, "matmul": Matmul, "sdpa": Sdpa, "sdpa_bwd": SdpaBwd,
             "unet": Unet, "llama": Llama}

# the `workloads` object of the default line: name -> constructor kwargs
EXTRA_WORKLOADS = [
    ("matmul_512", Matmul, {"size": 512}),
    ("matmul_1024", Matmul, {"size": 1024}),
    ("matmul_2048", Matmul, {"size": 2048}),
    ("matmul_4096", Matmul, {"size": 4096}),
    ("matmul_8192", Matmul, {"size": 8192}),
    ("matmul_8192_tf32x3", Matmul, {"size": 8192, "precision": "tf32x3"}),
    ("sdpa", Sdpa, {}),
    ("sdpa_bwd", SdpaBwd, {}),
    ("unet", Unet, {}),
    ("llama", Llama, {}),
]


# -------------------------------------------------------------- arms -----
def base_line(args, world, wl):
    return {"metric": METRIC, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": wl.scaling(),
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
            "config": wl.full_config()}


def run_reference(args, world, rank):
    """Reference arm: the reference's own CPU path (the oracle restatement of its
    CPU functions; the Rust/wgpu crate cannot be built or run here) on all host
    cores, on the headline config; rank 0 only.  Each step is a bounded sample
    of the workload (whole output rows), timed, and its TFLOPS extrapolate to
    the full step by FLOPs."""
    if rank != 0:
        return
    from oracle import oracle as orc
    orc.build()
    wl = WORKLOADS[args.workload](args, world, rank)
    vals, secs, sample = [], [], ""
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        v, sample = wl.cpu_sample(orc, args.ref_seconds)
        if i >= args.warmup:
            vals.append(v)
            secs.append(time.perf_counter() - t0)
    value = statistics.median(vals)
    line = base_line(args, world, wl)
    line.update({"impl": "reference", "value": value, "dtype": "f32",
                 "precision": "fp32 multiply-add with sequential fp32 sums (the reference's "
                              "CPU functions, restated in C), on the host CPU",
                 "ms_per_step": statistics.mean(secs) * 1e3,
                 "step": "one bounded sample of the workload (" + sample + "); value is its "
                         "FLOPs per second",
                 "ms_per_full_step_extrapolated": wl.flops / (value * 1e12) * 1e3,
                 "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": orc.num_threads(),
                                  "kind": "port", "sample": sample + " per step"},
                 "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}})
    print(json.dumps(line), flush=True)


class Ctx:
    """Per-process state shared by the measurements of one run."""

    def __init__(self, args, world, rank, local):
        import torch
        self.torch, self.args, self.world, self.rank, self.local = torch, args, world, rank, local
        self.peaks = load_peaks()
        self.host_group = None
        if world > 1:
            import torch.distributed as dist
            # host-side exchange and barriers of the copy-engine gathers (no
            # device work, so they never wait behind queued kernels)
            self.host_group = dist.new_group(backend="gloo",
                                             timeout=datetime.timedelta(seconds=180))

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[self.local])

    def max_over_ranks(self, vals):
        torch = self.torch
        t = torch.tensor(vals, dtype=torch.float64, device=f"cuda:{self.local}")
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()


def measure(ctx: Ctx, wl: Workload, cpu_seconds: float, cpu_single: float, e2e_steps: int,
            steps: int, warmup: int) -> dict:
    """Time one workload (device step, dominant kernel, e2e, CPU baseline) and
    return its entry (rank 0; other ranks return None)."""
    from any_gpu import GpuDevice
    torch, args = ctx.torch, ctx.args
    dev = GpuDevice.gpu(ctx.local)
    # A dedicated stream: the library launches on it and the CUDA events are
    # recorded on it (handle 0, torch's legacy default stream, would mean
    # "the library's own stream" at the C ABI).
    stream = torch.cuda.Stream(device=ctx.local)
    torch.cuda.set_stream(stream)
    wl.setup(torch, ctx.local)
    wl.make_gatherer(dev, ctx)
    prec = GpuDevice.precision(wl.precision) if wl.precision != "tf32" else \
        contextlib.nullcontext()
    try:
        with prec:
            entry = _measure(ctx, wl, dev, stream, cpu_seconds, cpu_single, e2e_steps, steps,
                             warmup)
    finally:
        torch.cuda.synchronize()
        wl.teardown()
        dev.close()
        torch.cuda.set_stream(torch.cuda.default_stream(ctx.local))
        torch.cuda.empty_cache()
    return entry


def _measure(ctx, wl, dev, stream, cpu_seconds, cpu_single, e2e_steps, steps, warmup):
    torch, args = ctx.torch, ctx.args
    tf32_peak = ctx.peaks["bf16_tflops"] / 2.0
    peak = tf32_peak / 3.0 if wl.precision == "tf32x3" else tf32_peak

    for _ in range(warmup):
        wl.step(dev, stream)
    torch.cuda.synchronize()
    ctx.barrier()
    torch.cuda.synchronize()

    use_graph = wl.graph_default if args.graph is None else args.graph
    use_graph = use_graph and not wl.sharded
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graph = None
    if use_graph:
        launches0 = dev.launch_count
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(steps):
                wl.step(dev, stream)
        launches = dev.launch_count - launches0
        graph.replay()  # untimed: uploads the graph
        torch.cuda.synchronize()
    clocks = ClockSampler(ctx.local)
    clocks.start()
    launches0 = dev.launch_count
    t_start.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for _ in range(steps):
            wl.step(dev, stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    if graph is None:
        launches = dev.launch_count - launches0
    clk = clocks.stop()
    ctx.barrier()
    torch.cuda.synchronize()
    total_ms = t_start.elapsed_time(t_end)
    chk = wl.checksum(torch) if ctx.rank == 0 else None

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]

    def loop_ms(fn):
        """Mean device time of `fn(stream)`: warm-up, then K runs, CUDA events
        around each on the launching stream."""
        for _ in range(2):
            fn(stream)
        torch.cuda.synchronize()
        for e0, e1 in evs:
            e0.record(stream)
            fn(stream)
            e1.record(stream)
        torch.cuda.synchronize()
        return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)

    compute_ms = gather_ms = 0.0
    if wl.sharded:
        compute_ms = loop_ms(lambda st: wl.step(dev, st, gather=False))
        ctx.barrier()
        gather_ms = loop_ms(wl.gather_only)
        ctx.barrier()
    if graph is not None:
        dom_ms = total_ms / steps
        del graph
    else:
        dom_ms = loop_ms(lambda st: wl.dom_step(dev, st))
    aux_ms = loop_ms(lambda st: wl.aux_step(dev, st)) if hasattr(wl, "aux_step") else None
    torch.cuda.synchronize()

    # e2e through the public API with host buffers (pinned), every copy timed:
    # the synchronous reference call sequence, and (where the workload has
    # one) the same step with its transfers pipelined over the async API
    e2e_n = max(1, min(steps, e2e_steps))

    def time_e2e(fn):
        fn(dev)
        ctx.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_n):
            fn(dev)
        return (time.perf_counter() - t0) / e2e_n

    e2e_seq_s = time_e2e(wl.e2e_step)
    pipelined = getattr(wl, "e2e_pipelined", None)
    e2e_pipe_s = time_e2e(pipelined) if pipelined is not None else e2e_seq_s
    torch.cuda.set_stream(stream)

    (total_ms, e2e_s, dom_ms, e2e_seq_s, aux_max, compute_ms, gather_ms) = ctx.max_over_ranks(
        [total_ms, e2e_pipe_s, dom_ms, e2e_seq_s, aux_ms or 0.0, compute_ms, gather_ms])
    aux_ms = aux_max if aux_ms is not None else None
    ms_per_step = total_ms / steps
    if ctx.rank != 0:
        return None

    achieved = wl.dom_flops / (dom_ms * 1e-3) / 1e12
    h2d, d2h = wl.e2e_bytes()
    e2e_flops = wl.flops
    entry = {
        "value": wl.flops / (ms_per_step * 1e-3) / 1e12, "unit": "TFLOPS",
        "ms_per_step": ms_per_step, "steps": steps, "warmup": warmup,
        "scaling": wl.scaling(), "dtype": wl.dtype,
        "precision": PRECISION_NOTE[wl.precision],
        "e2e": {"value": e2e_flops / e2e_s / 1e12, "unit": "TFLOPS",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "s_per_step": e2e_s, "steps": e2e_n,
                "how": wl.e2e_how if pipelined is not None else
                "upload -> ops -> read, each synchronous (the reference's call sequence)",
                "sequential": {"value": e2e_flops / e2e_seq_s / 1e12, "s_per_step": e2e_seq_s}},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": wl.traffic(),
                     "kernel": wl.dom_kernel,
                     "peak_note": (f"TF32 dense = bf16 {ctx.peaks['source']} "
                                   f"{ctx.peaks['bf16_tflops']} / 2"
                                   + (", / 3 for 3xTF32" if wl.precision == "tf32x3" else "")),
                     "ms_per_launch": dom_ms,
                     "launch_items": wl.local},
        "clocks": clk, "gpu_launches": launches, "output_check": chk,
    }
    if ctx.world > 1 and wl.sharded:
        entry["e2e"]["how"] += ("; each rank moves its own items' inputs up and its own "
                                "outputs down over its own PCIe link (no gather)")
    if wl.sharded:
        recv = (wl.total - wl.local) * wl.out_item * 4
        if ctx.args.comm == "ce":
            how = ("copy-engine pushes over CUDA IPC: each rank copies its run of every round "
                   f"into every peer's output (agpu_copy_async on {ctx.args.ce_streams} copy "
                   "stream(s), peers in rotated order, no SMs); the step ends on "
                   + ("device flag words (agpu_signal_peers / agpu_wait_flags)"
                      if ctx.args.ce_sync == "flags" else
                      "interprocess events + a host barrier"))
        elif all(r.even for r in wl.plan.spans):
            how = "in-place all_gather_into_tensor (ncclAllGather over NVLink) per round"
        else:
            how = "in-place broadcast per rank (uneven runs)"
        entry["comm"] = {
            "collective": how, "comm": ctx.args.comm,
            "rounds": len(wl.plan.spans), "recv_bytes_per_rank": recv,
            "gather_ms": gather_ms, "compute_ms": compute_ms,
            "exposed_gather_ms": ms_per_step - compute_ms,
            "recv_gbs": recv / (gather_ms * 1e-3) / 1e9 if gather_ms else None,
            "compute_only_value": wl.flops / (compute_ms * 1e-3) / 1e12,
            "note": "gather_ms: the step's gathers alone; compute_ms: the step without its "
                    "gathers (both max over ranks); exposed_gather_ms: step time minus "
                    "compute time"}
    entry.update(wl.extra(ms_per_step, dom_ms, ctx.peaks, aux_ms))
    if ctx.world == 1 and cpu_seconds > 0:
        from oracle import oracle as orc
        orc.build()
        v, sample = wl.cpu_sample(orc, cpu_seconds)
        entry["cpu_baseline"] = {"value": v, "unit": "TFLOPS", "cores": orc.num_threads(),
                                 "kind": "port", "sample": sample}
        if cpu_single > 0:
            v1, sample1 = wl.cpu_sample(orc, cpu_single, threads=False)
            entry["cpu_baseline"]["single_thread"] = {"value": v1, "unit": "TFLOPS",
                                                      "cores": 1, "sample": sample1}
    return entry


def run_agpu(args, world, rank, local):
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    ctx = Ctx(args, world, rank, local)
    wl = WORKLOADS[args.workload](args, world, rank, args.replicas)
    head = measure(ctx, wl, args.cpu_seconds, args.cpu_seconds_single, args.e2e_steps,
                   args.steps, args.warmup)
    extra = {}
    if args.workload == "bmm_softmax" and not args.no_workloads:
        for name, cls, kw in EXTRA_WORKLOADS:
            t0 = time.perf_counter()
            w = cls(args, world, rank, args.replicas, **kw)
            e = measure(ctx, w, args.cpu_seconds_workloads, 0.0,
                        min(args.e2e_steps, 2 if name == "llama" else 3), args.steps,
                        args.warmup)
            if rank == 0:
                e["config"] = w.full_config()
                e["wall_s"] = time.perf_counter() - t0
                extra[name] = e
    if rank == 0:
        line = base_line(args, world, wl)
        line.update(head)
        if extra:
            line["workloads"] = extra
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["agpu", "reference"], default="agpu")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="bmm_softmax")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: every rank runs the whole config, no collective (weak)")
    ap.add_argument("--comm", choices=["ce", "nccl"], default="ce",
                    help="N > 1 output gathers: copy engines over CUDA IPC, or NCCL collectives")
    ap.add_argument("--rounds", type=int, default=0,
                    help="N > 1: rounds of the sharded step (0: the workload's default)")
    ap.add_argument("--ce-streams", type=int, default=1,
                    help="copy streams of the copy-engine gathers (peers spread over them)")
    ap.add_argument("--ce-sync", choices=["flags", "events"], default="flags",
                    help="end of a copy-engine gather step: device flag words, or "
                         "interprocess events + a host barrier")
    ap.add_argument("--no-workloads", action="store_true",
                    help="headline only (no `workloads` object)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--cpu-seconds-single", type=float, default=5.0,
                    help="bounded single-thread CPU sample beside the all-cores one (0: skip)")
    ap.add_argument("--cpu-seconds-workloads", type=float, default=3.0)
    ap.add_argument("--ref-seconds", type=float, default=5.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--graph", dest="graph", action="store_true", default=None,
                    help="time the K steps as one CUDA graph (default: matmul workload only)")
    ap.add_argument("--no-graph", dest="graph", action="store_false")
    ap.add_argument("--batch", type=int, default=64,
                    help="bmm_softmax batch count (64 = the headline workload; smaller only "
                         "for profiler captures)")
    ap.add_argument("--size", type=int, default=512, help="matmul M = N = K")
    ap.add_argument("--precision", choices=["tf32", "tf32x3"], default="tf32",
                    help="matmul workload arithmetic")
    ap.add_argument("--bh", type=int, default=256, help="sdpa batch*heads (B8 x H32)")
    ap.add_argument("--seq", type=int, default=2048, help="sdpa sequence length")
    ap.add_argument("--images", type=int, default=16, help="unet batch N")
    ap.add_argument("--llama-batch", type=int, default=32, help="llama sequences of 2048")
    args = ap.parse_args()
    if args.no_cpu_baseline:
        args.cpu_seconds = args.cpu_seconds_workloads = 0.0
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_agpu(args, world, rank, local)


if __name__ == "__main__":
    main()
