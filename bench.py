#!/usr/bin/env python
"""Headline benchmark: fp32 batch_matmul -> row softmax on B200.

Workload (one "step"): C = batch_matmul(A, B) with batch 64, M = K = N = 2048,
A, B ~ N(0,1) * 0.05 (seeded), then S = softmax(C) over the last dim
(131072 rows x 2048).  The GEMM runs on tcgen05 tensor cores in TF32 with fp32
accumulate; softmax is the one-read-one-write warp-per-row kernel.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl agpu|reference]

One process per GPU (torchrun for N > 1).  Every rank runs the full workload
on its own GPU ("scaling": "weak"; batches are independent, no data-path
collective); `--gather` adds an NCCL all-gather of the softmax outputs.
Rank 0 prints one JSON line.

  value  : whole-job TFLOPS = N * 2*B*M*N*K / (max over ranks of the device
           time per step), inputs resident in HBM, CUDA events on the
           launching stream.  Inputs (2 GiB) + output (1 GiB) exceed the
           126 MB L2, so no flush is needed between steps.
  e2e    : the same FLOPs over the wall time of the public API call sequence
           upload(A), upload(B) from pinned host memory -> batch_matmul ->
           softmax -> read(S) into pinned host memory, max over ranks.
  roofline: the GEMM kernel's achieved TFLOP/s (CUDA events around each GEMM
           launch) against the TF32 dense peak = half the measured bf16 peak.
"""
from __future__ import annotations

import argparse
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

METRIC = "TFLOPS (matmul, SDPA) and GB/s (softmax/norm) at 1/2/4/8 B200, % of roofline"
BATCH, M, N, K = 64, 2048, 2048, 2048
GEMM_FLOPS = 2.0 * BATCH * M * N * K
SOFTMAX_BYTES = 2.0 * BATCH * M * N * 4  # one read + one write of C
SEED = 1235  # 1234 + config index

# dram bytes per GEMM launch from an ncu capture (profiles/gemm_tf32_*.md);
# None until captured for the current kernel.
GEMM_TRAFFIC_BYTES = None


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


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
            h = None
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


# ------------------------------------------------------------ helpers ----
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_inputs(rank: int):
    r = np.random.default_rng(SEED + 1000 * rank)
    a = r.standard_normal(BATCH * M * K, dtype=np.float32)
    a *= np.float32(0.05)
    b = r.standard_normal(BATCH * K * N, dtype=np.float32)
    b *= np.float32(0.05)
    return a, b


def cpu_sample(orc, threads: bool, target_s: float):
    """Time the oracle (reference CPU path) on a bounded sample of the step:
    rows of batch item 0 (batch_matmul rows then their softmax).  Grows the
    row count until about `target_s` seconds of work; returns TFLOPS."""
    r = np.random.default_rng(SEED)
    a = (r.standard_normal(M * K, dtype=np.float32) * np.float32(0.05))
    b = (r.standard_normal(K * N, dtype=np.float32) * np.float32(0.05))
    chunk = max(16, 2 * orc.num_threads())
    done, t_total, start = 0, 0.0, 0
    while t_total < target_s:
        rows = min(chunk, M - start)
        t0 = time.perf_counter()
        c = orc.matmul(a[start * K:(start + rows) * K], b, rows, N, K, threads=threads)
        orc.softmax(c, rows, N, threads=threads)
        t_total += time.perf_counter() - t0
        done += rows
        start = (start + rows) % M
    return 2.0 * done * N * K / t_total / 1e12, done, t_total


# -------------------------------------------------------------- arms -----
def run_reference(args, world, rank):
    """Reference arm: the reference's CPU path (the oracle restatement; the
    Rust/wgpu crate cannot be built or run here) on the host cores."""
    if rank != 0:
        return
    from oracle import oracle as orc
    orc.build()
    cores = orc.num_threads()
    per = []
    rows_done = 0
    for i in range(args.warmup + args.steps):
        v, rows, _ = cpu_sample(orc, threads=True, target_s=args.ref_seconds)
        if i >= args.warmup:
            per.append(v)
            rows_done = rows
    value = statistics.median(per)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": GEMM_FLOPS / (value * 1e12) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args, world),
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": cores, "kind": "port",
                         "sample": f"{rows_done} rows of batch item 0 per step (each: a "
                                   f"1x{K} by {K}x{N} matmul row + its softmax), "
                                   "extrapolated by FLOPs"},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(args, world):
    return {"workload": "batch_matmul+softmax", "batch": BATCH, "m": M, "n": N, "k": K,
            "inputs": "N(0,1)*0.05 seeded", "softmax_rows": BATCH * M, "softmax_cols": N,
            "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": "inputs 2 GiB + output 1 GiB > 126 MB L2 (no flush needed)",
            "precision": "tf32 multiply, fp32 accumulate, fp32 I/O",
            "gather": bool(args.gather)}


def run_agpu(args, world, rank, local):
    import torch
    from any_gpu import GpuDevice

    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    peaks = load_peaks()
    tf32_peak = peaks["bf16_tflops"] / 2.0
    dev = GpuDevice.gpu(local)

    a_np, b_np = make_inputs(rank)
    a_host = torch.from_numpy(a_np).pin_memory()
    b_host = torch.from_numpy(b_np).pin_memory()
    s_host = torch.empty(BATCH * M * N, dtype=torch.float32).pin_memory()
    del a_np, b_np
    A = a_host.to(f"cuda:{local}", non_blocking=False)
    B = b_host.to(f"cuda:{local}", non_blocking=False)
    C = torch.empty(BATCH * M * N, dtype=torch.float32, device=f"cuda:{local}")
    S = torch.empty_like(C)
    gathered = (torch.empty(world * BATCH * M * N, dtype=torch.float32,
                            device=f"cuda:{local}") if (args.gather and world > 1) else None)
    # A dedicated stream: the library launches on it and the CUDA events are
    # recorded on it (handle 0, torch's legacy default stream, would mean
    # "the library's own stream" at the C ABI).
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    assert sptr != 0

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        dev.launch_batch_matmul(A.data_ptr(), B.data_ptr(), C.data_ptr(), BATCH, M, N, K, sptr)
        if ev is not None:
            ev[1].record(stream)
        dev.launch_softmax(C.data_ptr(), S.data_ptr(), BATCH * M, N, sptr)
        if gathered is not None:
            import torch.distributed as dist
            dist.all_gather_into_tensor(gathered, S)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = dev.launch_count
    t_start.record(stream)
    for i in range(args.steps):
        step(evs[i])
    t_end.record(stream)
    torch.cuda.synchronize()
    launches = dev.launch_count - launches0
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    total_ms = t_start.elapsed_time(t_end)
    gemm_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)

    # ---------------------------------------------------------- e2e ----
    # public API: upload (H2D from pinned memory), batch_matmul, softmax,
    # read (D2H into pinned memory); wall clock includes every copy.
    a_view, b_view, s_view = a_host.numpy(), b_host.numpy(), s_host.numpy()
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def e2e_step():
        ga, gb = dev.upload(a_view), dev.upload(b_view)
        gc = dev.batch_matmul(ga, gb, BATCH, M, N, K)
        gs = dev.softmax(gc, BATCH * M, N)
        dev.read(gs, out=s_view)
        for buf in (ga, gb, gc, gs):
            buf.free()

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps

    # ------------------------------------------------ max over ranks ----
    vals = torch.tensor([total_ms, e2e_s, gemm_ms], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, e2e_s, gemm_ms = vals.tolist()
    ms_per_step = total_ms / args.steps
    value = world * GEMM_FLOPS / (ms_per_step * 1e-3) / 1e12
    sm_ms = ms_per_step - gemm_ms

    if rank == 0:
        achieved = GEMM_FLOPS / (gemm_ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "tf32",
            "data": "synthetic", "config": config_dict(args, world),
            "e2e": {"value": world * GEMM_FLOPS / e2e_s / 1e12, "unit": "TFLOPS",
                    "h2d_bytes_per_step": 2 * BATCH * M * K * 4,
                    "d2h_bytes_per_step": BATCH * M * N * 4,
                    "s_per_step": e2e_s, "steps": e2e_steps},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf32_peak,
                         "unit": "TFLOP/s", "frac": achieved / tf32_peak,
                         "traffic": GEMM_TRAFFIC_BYTES,
                         "kernel": "gemm_tf32_kernel<256,K-major A,MN-major B>",
                         "peak_note": f"TF32 dense = bf16 {peaks['source']} "
                                      f"{peaks['bf16_tflops']} / 2",
                         "ms_per_launch": gemm_ms},
            "softmax": {"ms": sm_ms, "gbs": SOFTMAX_BYTES / (sm_ms * 1e-3) / 1e9,
                        "frac_hbm": SOFTMAX_BYTES / (sm_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                        "note": "step time minus GEMM time"},
            "clocks": clk, "gpu_launches": launches,
        }
        if world == 1 and not args.no_cpu_baseline:
            from oracle import oracle as orc
            orc.build()
            v, rows, secs = cpu_sample(orc, threads=True, target_s=args.cpu_seconds)
            line["cpu_baseline"] = {
                "value": v, "unit": "TFLOPS", "cores": orc.num_threads(), "kind": "port",
                "sample": f"{rows} rows of batch item 0 (each: a 1x{K} by {K}x{N} matmul row + "
                          f"its softmax), {secs:.1f} s, extrapolated by FLOPs"}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    dev.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["agpu", "reference"], default="agpu")
    ap.add_argument("--gather", action="store_true",
                    help="NCCL all-gather of the softmax outputs inside each step")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-seconds", type=float, default=6.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=64,
                    help="batch count (64 = the headline workload; smaller only for "
                         "profiler captures)")
    args = ap.parse_args()
    global BATCH, GEMM_FLOPS, SOFTMAX_BYTES
    BATCH = args.batch
    GEMM_FLOPS = 2.0 * BATCH * M * N * K
    SOFTMAX_BYTES = 2.0 * BATCH * M * N * 4
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_agpu(args, world, rank, local)


if __name__ == "__main__":
    main()
