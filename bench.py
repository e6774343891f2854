#!/usr/bin/env python
"""Benchmark of the B200 dense-op path (one JSON line on rank 0).

Default workload (the headline): fp32 batch_matmul -> row softmax.
  One step = C = batch_matmul(A, B), batch 64, M = K = N = 2048, A, B ~ N(0,1)*0.05
  (seeded), then S = softmax(C) over the last dim (131072 rows x 2048), through
  the fused entry point agpu_launch_batch_matmul_softmax (the batch in pieces:
  the GEMMs back to back on one stream, each piece's softmax on a second stream
  beside the next piece's GEMM).  The GEMM runs
  on tcgen05 tensor cores in TF32 (operands rounded to nearest by TMA) with fp32
  accumulation; softmax is the one-read-one-write warp-per-row kernel.  The GEMM
  alone and the softmax alone are also timed, each in its own loop.

Other workloads (`--workload`), each one of the benchmark configurations:
  matmul   square fp32 matmul, A, B ~ U[-1,1)  (--size, default 512; sweep 64..8192)
  sdpa     scaled_dot_product_attention, B8 H32 S2048 D128, non-causal, N(0,1)
  unet     conv2d 3x3 s1 p1 (N16, 320->320, 64x64, Kaiming-uniform W, bias 0)
           -> group_norm (32 groups, eps 1e-5, gamma 1, beta 0) -> swish
  llama    LLaMA-style decoder layer forward: B32 S2048 d4096 H32x128 FFN 11008,
           RoPE base 1e4, W ~ N(0,0.02), x ~ N(0,1)

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl agpu|reference]
                    [--workload bmm_softmax|matmul|sdpa|unet|llama]

One process per GPU (torchrun for N > 1).  Every rank runs the full workload on
its own GPU ("scaling": "weak": batches/heads/images are independent, no
data-path collective); `--gather` adds an NCCL all-gather of the outputs.

  value    whole-job TFLOPS = N * FLOPs per step / (max over ranks of the device
           time per step); inputs resident in HBM; CUDA events on the launching
           stream.  Working sets exceed the 126 MB L2 (stated in `config.l2`);
           the small matmul sizes say so and re-read their inputs from L2.
  e2e      the same FLOPs over the wall time of the public API call sequence
           with host buffers (upload from pinned memory -> op(s) -> read into
           pinned memory), max over ranks.
  roofline the dominant kernel's FLOP/s (CUDA events around each launch) against
           the TF32 dense peak = half the measured bf16 peak.
  matmul steps are microseconds of device work, less than a host enqueue takes:
  their K steps are timed as one CUDA graph (`--no-graph`: host launches).
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

# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu
# capture of that kernel (dram__bytes_read.sum + dram__bytes_write.sum), for
# the default workload sizes; where the capture ran a smaller case, scaled by
# the units processed.
TRAFFIC_BYTES = {
    "bmm_softmax": 3.5e9,  # pair GEMM, batch-8 capture x 8
    "sdpa": 0.99e9,        # attention_pair_kernel, 64-head capture x 4
    "unet": 1.21e8,        # conv kernel, full workload
    "llama": 2.39e10,      # gate/up GEMM, batch-2 capture x 16
    "matmul": 2.13e6,      # split-K GEMM at 512^3, full capture (C stays in L2)
}


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
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


def _normal(r, n, scale=1.0):
    x = r.standard_normal(n, dtype=np.float32)
    if scale != 1.0:
        x *= np.float32(scale)
    return x


def _cores(orc, threads):
    """Host threads a CPU sample uses: all of the oracle's pool, or one."""
    return max(1, orc.num_threads()) if threads else 1


# ----------------------------------------------------------- workloads ---
class Workload:
    """One benchmark configuration.  Subclasses define the data, the device
    step (launch layer on a given stream) and the public-API e2e step."""
    name = ""
    dtype = "tf32"
    l2 = ""
    flops = 0.0       # FLOPs of one step
    dom_flops = 0.0   # FLOPs of one launch of the dominant kernel
    dom_kernel = ""
    graph_default = False  # time the steps as one CUDA graph (latency-bound steps)
    dom_separate = False   # dominant kernel timed in its own loop (dom_step), not per step

    def __init__(self, args, rank):
        self.args, self.rank = args, rank

    def config(self) -> dict:
        raise NotImplementedError

    def host_inputs(self) -> dict:
        raise NotImplementedError

    def out_elems(self) -> int:
        raise NotImplementedError

    def setup(self, torch, local):
        """Pinned host copies + device tensors."""
        self.host = {k: torch.from_numpy(v).pin_memory() for k, v in self.host_inputs().items()}
        self.dev_in = {k: v.to(f"cuda:{local}") for k, v in self.host.items()}
        self.out_host = torch.empty(self.out_elems(), dtype=torch.float32).pin_memory()

    def step(self, dev, sptr, ev=None):
        raise NotImplementedError

    def output(self):
        raise NotImplementedError

    def e2e_step(self, dev):
        raise NotImplementedError

    def e2e_bytes(self):
        h2d = sum(v.numel() * 4 for v in self.host.values())
        return h2d, self.out_elems() * 4

    def cpu_sample(self, orc, target_s, threads=True):
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
            bufs["_out"] = dev.alloc(self.out_elems())
            dev.synchronize()  # the zero fills finish before other streams write
            self._pipe = (bufs, [torch.cuda.Stream() for _ in range(3)])
        bufs, (up, comp, down) = self._pipe
        ptrs = {k: b.device_ptr for k, b in bufs.items()}
        for k in shared:
            n = self.host[k].numel()
            dev.write_async(bufs[k], self.host[k].data_ptr(), n, 0, up.cuda_stream)
        per_out = self.out_elems() // chunks
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

    def extra(self, ms_step, ms_dom, peaks, aux_ms=None) -> dict:
        return {}


class BmmSoftmax(Workload):
    name = "bmm_softmax"
    l2 = "inputs 2 GiB + output 1 GiB > 126 MB L2 (no flush needed)"

    def __init__(self, args, rank):
        super().__init__(args, rank)
        self.B, self.M, self.N, self.K = args.batch, 2048, 2048, 2048
        self.flops = self.dom_flops = 2.0 * self.B * self.M * self.N * self.K
        self.dom_kernel = "umma_tf32_pair_kernel<GemmPairPolicy<K-major A, MN-major B>> (256x256 CTA-pair tiles)"

    def config(self):
        return {"workload": "batch_matmul+softmax", "batch": self.B, "m": self.M, "n": self.N,
                "k": self.K, "inputs": "N(0,1)*0.05 seeded", "softmax_rows": self.B * self.M,
                "softmax_cols": self.N}

    def host_inputs(self):
        r = np.random.default_rng(1235 + 1000 * self.rank)
        return {"a": _normal(r, self.B * self.M * self.K, 0.05),
                "b": _normal(r, self.B * self.K * self.N, 0.05)}

    def out_elems(self):
        return self.B * self.M * self.N

    def setup(self, torch, local):
        super().setup(torch, local)
        self.C = torch.empty(self.out_elems(), dtype=torch.float32, device=f"cuda:{local}")
        self.S = torch.empty_like(self.C)

    # The step is the fused entry point (batch_matmul then softmax, the two
    # halves of the batch on two streams so that the first half's softmax
    # runs beside the second half's GEMM); the GEMM and the softmax are each
    # also timed alone, in their own loops after the timed region.
    dom_separate = True

    def step(self, dev, sptr, ev=None):
        dev.launch_batch_matmul_softmax(self.dev_in["a"].data_ptr(), self.dev_in["b"].data_ptr(),
                                        self.S.data_ptr(), self.B, self.M, self.N, self.K, sptr)

    def dom_step(self, dev, sptr):
        dev.launch_batch_matmul(self.dev_in["a"].data_ptr(), self.dev_in["b"].data_ptr(),
                                self.C.data_ptr(), self.B, self.M, self.N, self.K, sptr)

    def aux_step(self, dev, sptr):
        dev.launch_softmax(self.C.data_ptr(), self.S.data_ptr(), self.B * self.M, self.N, sptr)

    def output(self):
        return self.S

    def e2e_step(self, dev):
        ga, gb = dev.upload(self.host["a"].numpy()), dev.upload(self.host["b"].numpy())
        gc = dev.batch_matmul(ga, gb, self.B, self.M, self.N, self.K)
        gs = dev.softmax(gc, self.B * self.M, self.N)
        dev.read(gs, out=self.out_host.numpy())
        for b in (ga, gb, gc, gs):
            b.free()

    def e2e_pipelined(self, dev):
        import torch
        if not hasattr(self, "_pipe"):
            bufs = (dev.alloc(self.B * self.M * self.K), dev.alloc(self.B * self.K * self.N),
                    dev.alloc(self.out_elems()), dev.alloc(self.out_elems()))
            dev.synchronize()  # the zero fills finish before other streams write
            self._pipe = (bufs, [torch.cuda.Stream() for _ in range(3)])
        (ga, gb, gc, gs), (up, comp, down) = self._pipe
        chunks = next(c for c in (16, 8, 4, 2, 1) if self.B % c == 0)
        self.e2e_how = (f"batch split in {chunks} chunks; per chunk agpu_write_async of A and "
                        "B on an upload stream, batch_matmul + softmax (launch layer) on a "
                        "compute stream, agpu_read_async of S on a download stream: PCIe "
                        "both ways overlapped")
        per = self.B // chunks
        na, nb, nc = per * self.M * self.K, per * self.K * self.N, per * self.M * self.N
        ha, hb = self.host["a"].data_ptr(), self.host["b"].data_ptr()
        ho = self.out_host.data_ptr()
        pa, pb, pc, ps = (x.device_ptr for x in (ga, gb, gc, gs))
        for i in range(chunks):
            dev.write_async(ga, ha + 4 * i * na, na, i * na, up.cuda_stream)
            dev.write_async(gb, hb + 4 * i * nb, nb, i * nb, up.cuda_stream)
            e_up = torch.cuda.Event()
            e_up.record(up)
            comp.wait_event(e_up)
            dev.launch_batch_matmul(pa + 4 * i * na, pb + 4 * i * nb, pc + 4 * i * nc, per,
                                    self.M, self.N, self.K, comp.cuda_stream)
            dev.launch_softmax(pc + 4 * i * nc, ps + 4 * i * nc, per * self.M, self.N,
                               comp.cuda_stream)
            e_c = torch.cuda.Event()
            e_c.record(comp)
            down.wait_event(e_c)
            dev.read_async(gs, ho + 4 * i * nc, nc, i * nc, down.cuda_stream)
        down.synchronize()
        dev.synchronize()  # surfaces an expired device-side wait, if any

    def cpu_sample(self, orc, target_s, threads=True):
        r = np.random.default_rng(1235)
        a = _normal(r, self.M * self.K, 0.05)
        b = _normal(r, self.K * self.N, 0.05)
        chunk, done, t, start = max(16, 2 * _cores(orc, threads)), 0, 0.0, 0
        while t < target_s:
            rows = min(chunk, self.M - start)
            t0 = time.perf_counter()
            c = orc.matmul(a[start * self.K:(start + rows) * self.K], b, rows, self.N, self.K,
                           threads=threads)
            orc.softmax(c, rows, self.N, threads=threads)
            t += time.perf_counter() - t0
            done += rows
            start = (start + rows) % self.M
        v = 2.0 * done * self.N * self.K / t / 1e12
        return v, (f"{done} rows of batch item 0 (each: a 1x{self.K} by {self.K}x{self.N} "
                   f"matmul row + its softmax), {t:.1f} s, extrapolated by FLOPs")

    def extra(self, ms_step, ms_dom, peaks, aux_ms=None):
        nbytes = 2.0 * self.B * self.M * self.N * 4
        gbs = nbytes / (aux_ms * 1e-3) / 1e9
        return {"softmax": {"ms": aux_ms, "gbs": gbs, "frac_hbm": gbs / peaks["hbm_gbs"],
                            "exposed_ms": ms_step - ms_dom,
                            "note": "ms: softmax_warp_kernel alone over the 131072 x 2048 "
                                    "result (8 B per element); exposed_ms: step time minus "
                                    "GEMM time, the part of it the step does not hide"}}


class Matmul(Workload):
    name = "matmul"
    graph_default = True

    def __init__(self, args, rank):
        super().__init__(args, rank)
        self.n = args.size
        self.flops = self.dom_flops = 2.0 * self.n ** 3
        n = self.n
        self.dom_kernel = ("umma_tf32_kernel<GemmPolicy<128|256>> (single CTA)" if n < 256 else
                           "umma_tf32_pair_splitk_kernel<GemmPairPolicy<256>, 4|2> (cluster "
                           "split-K)" if n <= 1024 else
                           "umma_tf32_pair_kernel<GemmPairPolicy<256|512>>")
        ws = 3 * self.n * self.n * 4
        self.l2 = (f"working set {ws / 2**20:.1f} MiB "
                   + ("> 126 MB L2" if ws > 126e6 else "fits in L2: inputs re-read from L2"))

    def config(self):
        return {"workload": "matmul", "m": self.n, "n": self.n, "k": self.n,
                "inputs": "U[-1,1) seeded",
                "timing": "K steps captured in one CUDA graph" if self.args.graph is not False
                else "K steps launched from the host"}

    def host_inputs(self):
        r = np.random.default_rng(1234 + 1000 * self.rank)
        return {"a": r.uniform(-1, 1, self.n * self.n).astype(np.float32),
                "b": r.uniform(-1, 1, self.n * self.n).astype(np.float32)}

    def out_elems(self):
        return self.n * self.n

    def setup(self, torch, local):
        super().setup(torch, local)
        self.C = torch.empty(self.out_elems(), dtype=torch.float32, device=f"cuda:{local}")

    def step(self, dev, sptr, ev=None):
        if ev is not None:
            ev[0].record()
        dev.launch_batch_matmul(self.dev_in["a"].data_ptr(), self.dev_in["b"].data_ptr(),
                                self.C.data_ptr(), 1, self.n, self.n, self.n, sptr)
        if ev is not None:
            ev[1].record()

    def output(self):
        return self.C

    def e2e_step(self, dev):
        ga, gb = dev.upload(self.host["a"].numpy()), dev.upload(self.host["b"].numpy())
        gc = dev.matmul(ga, gb, self.n, self.n, self.n)
        dev.read(gc, out=self.out_host.numpy())
        for b in (ga, gb, gc):
            b.free()

    def cpu_sample(self, orc, target_s, threads=True):
        a, b = self.host_inputs().values()
        n = self.n
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

    def __init__(self, args, rank):
        super().__init__(args, rank)
        self.bh, self.s, self.d = args.bh, args.seq, 128
        self.flops = self.dom_flops = 4.0 * self.bh * self.s * self.s * self.d
        self.dom_kernel = "attention_pair_kernel<128, non-causal> (CTA-pair flash attention)"

    def config(self):
        return {"workload": "scaled_dot_product_attention", "batch_heads": self.bh,
                "seq_len": self.s, "d_k": self.d, "causal": False, "inputs": "N(0,1) seeded",
                "flops": "4*BH*S^2*D (QK^T + PV)"}

    def host_inputs(self):
        r = np.random.default_rng(1236 + 1000 * self.rank)
        n = self.bh * self.s * self.d
        return {"q": _normal(r, n), "k": _normal(r, n), "v": _normal(r, n)}

    def out_elems(self):
        return self.bh * self.s * self.d

    def setup(self, torch, local):
        super().setup(torch, local)
        self.O = torch.empty(self.out_elems(), dtype=torch.float32, device=f"cuda:{local}")

    def step(self, dev, sptr, ev=None):
        if ev is not None:
            ev[0].record()
        dev.launch_sdpa(self.dev_in["q"].data_ptr(), self.dev_in["k"].data_ptr(),
                        self.dev_in["v"].data_ptr(), self.O.data_ptr(), self.bh, self.s, self.d,
                        False, sptr)
        if ev is not None:
            ev[1].record()

    def output(self):
        return self.O

    def e2e_step(self, dev):
        g = [dev.upload(self.host[n].numpy()) for n in "qkv"]
        go = dev.scaled_dot_product_attention(*g, self.bh, self.s, self.d)
        dev.read(go, out=self.out_host.numpy())
        for b in g + [go]:
            b.free()

    def e2e_pipelined(self, dev):
        chunks = next(c for c in (8, 4, 2, 1) if self.bh % c == 0)
        per = self.bh // chunks
        hsz = self.s * self.d
        self.e2e_how = (f"batch*heads split in {chunks} chunks; per chunk agpu_write_async of "
                        "Q, K, V on an upload stream, attention (launch layer) on a compute "
                        "stream, agpu_read_async of O on a download stream")

        def launch(i, p, st):
            off = 4 * i * per * hsz
            dev.launch_sdpa(p["q"] + off, p["k"] + off, p["v"] + off, p["_out"] + off, per,
                            self.s, self.d, False, st)
        self._pipelined(dev, ["q", "k", "v"], [], chunks, launch)

    def cpu_sample(self, orc, target_s, threads=True):
        r = np.random.default_rng(1236)
        hsz = self.s * self.d
        heads = _cores(orc, threads)
        q, k, v = (_normal(r, heads * hsz) for _ in range(3))
        done, t = 0, 0.0
        while t < target_s:
            t0 = time.perf_counter()
            orc.attention(q, k, v, heads, self.s, self.d, threads=threads)
            t += time.perf_counter() - t0
            done += heads
        return (4.0 * done * self.s * self.s * self.d / t / 1e12,
                f"{done} heads of S={self.s}, D={self.d} (cpu_attention per head), {t:.1f} s")


class Unet(Workload):
    name = "unet"
    l2 = "x 80 MiB + conv out 80 MiB + y 80 MiB > 126 MB L2"

    def __init__(self, args, rank):
        super().__init__(args, rank)
        self.n, self.c, self.h, self.w, self.g = args.images, 320, 64, 64, 32
        self.flops = self.dom_flops = 2.0 * self.n * self.c * self.h * self.w * self.c * 9
        self.dom_kernel = ("umma_tf32_pair_kernel<ConvPairPolicy<320>> (implicit-GEMM conv2d, "
                           "staging included; timed in a separate loop of conv2d calls)")

    def config(self):
        return {"workload": "unet_block conv2d3x3->group_norm->swish", "n": self.n,
                "cin": self.c, "cout": self.c, "h": self.h, "w": self.w, "groups": self.g,
                "eps": 1e-5, "inputs": "x N(0,1); W Kaiming-uniform U(+-sqrt(6/2880)); bias 0",
                "flops": "conv only: 2*N*Cout*H*W*Cin*9"}

    def host_inputs(self):
        r = np.random.default_rng(1237 + 1000 * self.rank)
        bound = np.float32(np.sqrt(6.0 / (self.c * 9)))
        return {"x": _normal(r, self.n * self.c * self.h * self.w),
                "w": r.uniform(-bound, bound, self.c * self.c * 9).astype(np.float32),
                "gamma": np.ones(self.c, np.float32), "beta": np.zeros(self.c, np.float32)}

    def out_elems(self):
        return self.n * self.c * self.h * self.w

    def setup(self, torch, local):
        super().setup(torch, local)
        self.Y1 = torch.empty(self.out_elems(), dtype=torch.float32, device=f"cuda:{local}")
        self.Y = torch.empty_like(self.Y1)

    # The step is the fused entry point (conv2d -> group_norm -> swish in one
    # call, the group norm of one half of the batch beside the conv of the
    # other), so the conv's own time comes from a separate loop of conv2d
    # launches after the timed region.
    dom_separate = True

    def step(self, dev, sptr, ev=None):
        d = self.dev_in
        dev.launch_conv2d_group_norm_swish(
            d["x"].data_ptr(), d["w"].data_ptr(), 0, self.Y.data_ptr(), self.n, self.c, self.h,
            self.w, self.c, 3, 3, 1, 1, 1, 1, 1, 1, 1, d["gamma"].data_ptr(),
            d["beta"].data_ptr(), self.g, 1e-5, sptr)

    def dom_step(self, dev, sptr):
        d = self.dev_in
        dev.launch_conv2d(d["x"].data_ptr(), d["w"].data_ptr(), 0, self.Y1.data_ptr(), self.n,
                          self.c, self.h, self.w, self.c, 3, 3, 1, 1, 1, 1, 1, 1, 1, sptr)

    def aux_step(self, dev, sptr):
        d = self.dev_in
        dev.launch_group_norm(self.Y1.data_ptr(), d["gamma"].data_ptr(), d["beta"].data_ptr(),
                              self.Y.data_ptr(), self.n, self.c, self.h * self.w, self.g, 1e-5,
                              True, sptr)

    def output(self):
        return self.Y

    def e2e_step(self, dev):
        g = {k: dev.upload(v.numpy()) for k, v in self.host.items()}
        y = dev.conv2d_group_norm_swish(g["x"], g["w"], None, self.n, self.c, self.h, self.w,
                                        self.c, 3, 3, (1, 1), (1, 1), (1, 1), 1, gamma=g["gamma"],
                                        beta=g["beta"], gn_groups=self.g, eps=1e-5)
        dev.read(y, out=self.out_host.numpy())
        for b in list(g.values()) + [y]:
            b.free()

    def e2e_pipelined(self, dev):
        chunks = next(c for c in (4, 2, 1) if self.n % c == 0)
        per = self.n // chunks
        img = self.c * self.h * self.w
        self.e2e_how = (f"images split in {chunks} chunks; the weights, then per chunk the "
                        "images, up by agpu_write_async on an upload stream, the fused conv2d "
                        "-> group_norm -> swish (launch layer) on a compute stream, "
                        "agpu_read_async of the output on a download stream")

        def launch(i, p, st):
            off = 4 * i * per * img
            dev.launch_conv2d_group_norm_swish(
                p["x"] + off, p["w"], 0, p["_out"] + off, per, self.c, self.h, self.w, self.c,
                3, 3, 1, 1, 1, 1, 1, 1, 1, p["gamma"], p["beta"], self.g, 1e-5, st)
        self._pipelined(dev, ["x"], ["w", "gamma", "beta"], chunks, launch)

    def cpu_sample(self, orc, target_s, threads=True):
        x, w, gamma, beta = self.host_inputs().values()
        img = self.c * self.h * self.w
        done, t = 0, 0.0
        while t < target_s:
            t0 = time.perf_counter()
            y = orc.conv2d(x[:img], w, None, 1, self.c, self.h, self.w, self.c, 3, 3, (1, 1),
                           (1, 1), (1, 1), 1, threads=threads)
            y = orc.group_norm(y, gamma, beta, 1, self.c, self.h * self.w, self.g, 1e-5,
                               threads=threads)
            orc.elementwise("swish", y)
            t += time.perf_counter() - t0
            done += 1
        return (2.0 * done * img * self.c * 9 / t / 1e12,
                f"{done} image(s) of the block (cpu_conv2d + cpu_group_norm + swish), {t:.1f} s")

    def extra(self, ms_step, ms_dom, peaks, aux_ms=None):
        nbytes = 2.0 * self.out_elems() * 4
        # the group norm runs as two passes (stats, then normalise + swish):
        # counted per pass it moves x twice and y once
        pbytes = 3.0 * self.out_elems() * 4
        gbs, pgbs = nbytes / (aux_ms * 1e-3) / 1e9, pbytes / (aux_ms * 1e-3) / 1e9
        return {"group_norm_swish": {"ms": aux_ms, "gbs": gbs, "frac_hbm": gbs / peaks["hbm_gbs"],
                                     "gbs_per_pass": pgbs,
                                     "frac_hbm_per_pass": pgbs / peaks["hbm_gbs"],
                                     "exposed_ms": ms_step - ms_dom,
                                     "note": "ms: the group norm + swish alone (two kernels); "
                                             "gbs counts 8 B per element (x read once, y "
                                             "written once), gbs_per_pass the 12 B per "
                                             "element the two passes move; exposed_ms: step "
                                             "time minus conv time, the part the fused step "
                                             "does not hide behind the conv"}}


class Llama(Workload):
    name = "llama"
    l2 = "activations ~19 GB > 126 MB L2"

    def __init__(self, args, rank):
        super().__init__(args, rank)
        from any_gpu.llama import LlamaDims
        self.dims = LlamaDims(batch=args.llama_batch, seq=2048, d_model=4096, heads=32,
                              ffn=11008)
        dm = self.dims
        self.flops = dm.gemm_flops() + dm.attention_flops()
        self.dom_flops = 2.0 * dm.tokens * dm.d_model * 2 * dm.ffn
        self.dom_kernel = "umma_tf32_pair_kernel<GemmPairPolicy<K-major A, MN-major B>> (gate/up)"

    def config(self):
        dm = self.dims
        return {"workload": "llama_decoder_layer_forward", "batch": dm.batch, "seq": dm.seq,
                "d_model": dm.d_model, "heads": dm.heads, "head_dim": dm.head_dim,
                "ffn": dm.ffn, "rope_base": dm.rope_base, "causal": dm.causal,
                "inputs": "x N(0,1); W N(0,0.02); norm weights 1",
                "flops": "2*T*(4d^2+3dF) + 4*B*H*S^2*Dh"}

    def host_inputs(self):
        dm = self.dims
        d, Fd = dm.d_model, dm.ffn
        r = np.random.default_rng(1239 + 1000 * self.rank)
        return {"x": _normal(r, dm.tokens * d), "attn_norm": np.ones(d, np.float32),
                "ffn_norm": np.ones(d, np.float32), "wqkv": _normal(r, d * 3 * d, 0.02),
                "wo": _normal(r, d * d, 0.02), "wgu": _normal(r, d * 2 * Fd, 0.02),
                "wd": _normal(r, Fd * d, 0.02)}

    def out_elems(self):
        return self.dims.tokens * self.dims.d_model

    def setup(self, torch, local):
        super().setup(torch, local)
        self.ws = {k: torch.empty(n, dtype=torch.float32, device=f"cuda:{local}")
                   for k, n in self.dims.workspace_elems().items()}
        self.Y = torch.empty(self.out_elems(), dtype=torch.float32, device=f"cuda:{local}")

    def step(self, dev, sptr, ev=None):
        from any_gpu.llama import layer_forward
        w = {k: v.data_ptr() for k, v in self.dev_in.items() if k != "x"}
        ws = {k: v.data_ptr() for k, v in self.ws.items()}
        if ev is None:
            layer_forward(dev, self.dims, self.dev_in["x"].data_ptr(), w, ws, self.Y.data_ptr(),
                          sptr)
            return
        # same sequence with the gate/up GEMM bracketed by events
        dm = self.dims
        T, d, Fd = dm.tokens, dm.d_model, dm.ffn
        dev_hook = _EventHook(dev, ev, target=2)
        layer_forward(dev_hook, self.dims, self.dev_in["x"].data_ptr(), w, ws,
                      self.Y.data_ptr(), sptr)

    def output(self):
        return self.Y

    def e2e_step(self, dev):
        from any_gpu.llama import layer_forward
        g = {k: dev.upload(v.numpy()) for k, v in self.host.items()}
        ws = {k: dev.alloc(n) for k, n in self.dims.workspace_elems().items()}
        y = dev.alloc(self.out_elems())
        layer_forward(dev, self.dims, g["x"].device_ptr,
                      {k: b.device_ptr for k, b in g.items() if k != "x"},
                      {k: b.device_ptr for k, b in ws.items()}, y.device_ptr)
        dev.read(y, out=self.out_host.numpy())
        for b in list(g.values()) + list(ws.values()) + [y]:
            b.free()

    def cpu_sample(self, orc, target_s, threads=True):
        dm = self.dims
        d = dm.d_model
        r = np.random.default_rng(1239)
        x = _normal(r, 64 * d)
        wqkv = _normal(r, d * 3 * d, 0.02)
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


class _EventHook:
    """Wraps a GpuDevice so that the `target`-th launch_gemm_ex of a layer is
    bracketed by the two CUDA events in `ev` (0-based: 2 = the gate/up GEMM)."""

    def __init__(self, dev, ev, target):
        self._dev, self._ev, self._target, self._n = dev, ev, target, 0

    def __getattr__(self, name):
        return getattr(self._dev, name)

    def launch_gemm_ex(self, *a, **k):
        hit = self._n == self._target
        self._n += 1
        if hit:
            self._ev[0].record()
        self._dev.launch_gemm_ex(*a, **k)
        if hit:
            self._ev[1].record()


WORKLOADS = {"bmm_softmax": BmmSoftmax, "matmul": Matmul, "sdpa": Sdpa, "unet": Unet,
             "llama": Llama}


# -------------------------------------------------------------- arms -----
def base_line(args, world, wl):
    cfg = wl.config()
    cfg.update({"parallelism": f"replicas{world}" if world > 1 else "single", "l2": wl.l2,
                "precision": "tf32 multiply (operands rounded to nearest), fp32 accumulate, "
                             "fp32 I/O", "gather": bool(args.gather)})
    return {"metric": METRIC, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic", "config": cfg}


def run_reference(args, world, rank):
    """Reference arm: the reference's own CPU path (the oracle restatement of its
    CPU functions; the Rust/wgpu crate cannot be built or run here) on all host
    cores; rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as orc
    orc.build()
    wl = WORKLOADS[args.workload](args, 0)
    vals, sample = [], ""
    for i in range(args.warmup + args.steps):
        v, sample = wl.cpu_sample(orc, args.ref_seconds)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = base_line(args, world, wl)
    line.update({"impl": "reference", "value": value, "dtype": "f32",
                 "ms_per_step": wl.flops / (value * 1e12) * 1e3,
                 "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": orc.num_threads(),
                                  "kind": "port", "sample": sample + " per step"},
                 "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}})
    print(json.dumps(line), flush=True)


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
    wl = WORKLOADS[args.workload](args, rank)
    wl.setup(torch, local)
    # A dedicated stream: the library launches on it and the CUDA events are
    # recorded on it (handle 0, torch's legacy default stream, would mean
    # "the library's own stream" at the C ABI).
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    assert sptr != 0
    gathered = None
    if args.gather and world > 1:
        gathered = torch.empty(world * wl.out_elems(), dtype=torch.float32,
                               device=f"cuda:{local}")

    def step(ev=None):
        wl.step(dev, sptr, ev)
        if gathered is not None:
            import torch.distributed as dist
            dist.all_gather_into_tensor(gathered, wl.output())

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    # Latency-bound steps (a small matmul is a few microseconds of device work,
    # less than the host needs to enqueue it) are timed as one CUDA graph of
    # the K steps: the device runs them back to back, as a graph-captured
    # inner loop would in an application.  Per-step events cannot be recorded
    # inside a graph, so the dominant kernel's time is the step time there
    # (one launch per matmul step).
    def loop_ms(fn):
        """Mean time of `fn` alone: K launches, CUDA events around each."""
        for _ in range(2):
            fn(dev, sptr)
        torch.cuda.synchronize()
        for e0, e1 in evs:
            e0.record()
            fn(dev, sptr)
            e1.record()
        torch.cuda.synchronize()
        return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)

    use_graph = wl.graph_default if args.graph is None else args.graph
    use_graph = use_graph and world == 1 and not args.gather
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graph = None
    if use_graph:
        launches0 = dev.launch_count
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(args.steps):
                wl.step(dev, sptr, None)
        launches = dev.launch_count - launches0
        graph.replay()  # untimed: uploads the graph
        torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = dev.launch_count
    t_start.record()
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.steps):
            step(evs[i])
    t_end.record()
    torch.cuda.synchronize()
    if graph is None:
        launches = dev.launch_count - launches0
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    total_ms = t_start.elapsed_time(t_end)
    if graph is not None:
        dom_ms = total_ms / args.steps
        del graph
    else:
        dom_ms = (loop_ms(wl.dom_step) if wl.dom_separate else
                  statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs))
    aux_ms = loop_ms(wl.aux_step) if hasattr(wl, "aux_step") else None

    # e2e through the public API with host buffers (pinned), every copy timed:
    # the synchronous reference call sequence, and (where the workload has
    # one) the same step with its transfers pipelined over the async API
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def time_e2e(fn):
        fn(dev)
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            fn(dev)
        return (time.perf_counter() - t0) / e2e_steps

    e2e_seq_s = time_e2e(wl.e2e_step)
    pipelined = getattr(wl, "e2e_pipelined", None)
    e2e_pipe_s = time_e2e(pipelined) if pipelined is not None else e2e_seq_s
    torch.cuda.set_stream(stream)

    vals = torch.tensor([total_ms, e2e_pipe_s, dom_ms, e2e_seq_s, aux_ms or 0.0],
                        dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, e2e_s, dom_ms, e2e_seq_s, aux_max = vals.tolist()
    aux_ms = aux_max if aux_ms is not None else None
    ms_per_step = total_ms / args.steps

    if rank == 0:
        achieved = wl.dom_flops / (dom_ms * 1e-3) / 1e12
        h2d, d2h = wl.e2e_bytes()
        traffic = TRAFFIC_BYTES.get(wl.name)
        default_size = {"bmm_softmax": args.batch == 64, "sdpa": args.bh == 256 and args.seq == 2048,
                        "unet": args.images == 16, "llama": args.llama_batch == 32,
                        "matmul": args.size == 512}
        if not default_size.get(wl.name, False):
            traffic = None
        line = base_line(args, world, wl)
        line.update({
            "value": world * wl.flops / (ms_per_step * 1e-3) / 1e12,
            "ms_per_step": ms_per_step,
            "e2e": {"value": world * wl.flops / e2e_s / 1e12, "unit": "TFLOPS",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "s_per_step": e2e_s, "steps": e2e_steps,
                    "how": wl.e2e_how if pipelined is not None else
                    "upload -> ops -> read, each synchronous (the reference's call sequence)",
                    "sequential": {"value": world * wl.flops / e2e_seq_s / 1e12,
                                   "s_per_step": e2e_seq_s}},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf32_peak,
                         "unit": "TFLOP/s", "frac": achieved / tf32_peak, "traffic": traffic,
                         "kernel": wl.dom_kernel,
                         "peak_note": f"TF32 dense = bf16 {peaks['source']} "
                                      f"{peaks['bf16_tflops']} / 2",
                         "ms_per_launch": dom_ms},
            "clocks": clk, "gpu_launches": launches,
        })
        line.update(wl.extra(ms_per_step, dom_ms, peaks, aux_ms))
        if world == 1 and not args.no_cpu_baseline:
            from oracle import oracle as orc
            orc.build()
            v, sample = wl.cpu_sample(orc, args.cpu_seconds)
            line["cpu_baseline"] = {"value": v, "unit": "TFLOPS", "cores": orc.num_threads(),
                                    "kind": "port", "sample": sample}
            if args.cpu_seconds_single > 0:
                v1, sample1 = wl.cpu_sample(orc, args.cpu_seconds_single, threads=False)
                line["cpu_baseline"]["single_thread"] = {"value": v1, "unit": "TFLOPS",
                                                         "cores": 1, "sample": sample1}
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
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="bmm_softmax")
    ap.add_argument("--gather", action="store_true",
                    help="NCCL all-gather of the outputs inside each step")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--cpu-seconds-single", type=float, default=5.0,
                    help="bounded single-thread CPU sample beside the all-cores one (0: skip)")
    ap.add_argument("--ref-seconds", type=float, default=6.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--graph", dest="graph", action="store_true", default=None,
                    help="time the K steps as one CUDA graph (default: matmul workload only)")
    ap.add_argument("--no-graph", dest="graph", action="store_false")
    ap.add_argument("--batch", type=int, default=64,
                    help="bmm_softmax batch count (64 = the headline workload; smaller only "
                         "for profiler captures)")
    ap.add_argument("--size", type=int, default=512, help="matmul M = N = K")
    ap.add_argument("--bh", type=int, default=256, help="sdpa batch*heads (B8 x H32)")
    ap.add_argument("--seq", type=int, default=2048, help="sdpa sequence length")
    ap.add_argument("--images", type=int, default=16, help="unet batch N")
    ap.add_argument("--llama-batch", type=int, default=32, help="llama sequences of 2048")
    args = ap.parse_args()
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_agpu(args, world, rank, local)


if __name__ == "__main__":
    main()
