"""The bench's reference arm runs on the host alone: one JSON line with the
contract's keys (checked here on CPU with a tiny sample)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--ref-seconds", "0.2"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "data", "config"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "TFLOPS" and line["n_gpus"] == 1
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # the step is the bounded sample that ran, not the extrapolated full step
    assert line["ms_per_step"] < line["ms_per_full_step_extrapolated"]
    assert line["dtype"] == "f32" and "fp32" in line["precision"]
    assert "tf32" not in json.dumps(line["config"])


def test_bench_workload_plans_cpu():
    """The bench's workloads build their shard plans and job sizes on CPU: the
    job (items, FLOPs) is the same at every N, and each rank's share adds up."""
    sys.path.insert(0, str(ROOT))
    import argparse
    import bench
    args = argparse.Namespace(batch=64, size=512, precision="tf32", bh=256, seq=2048, images=16,
                              llama_batch=32, graph=None, rounds=0)
    for cls in (bench.BmmSoftmax, bench.Sdpa, bench.Unet, bench.Llama):
        one = cls(args, 1, 0)
        assert one.scaling() == "strong" and one.local == one.total
        for world in (2, 4, 8):
            ranks = [cls(args, world, r) for r in range(world)]
            assert all(w.flops == one.flops for w in ranks)
            assert sum(w.local for w in ranks) == one.total
            assert all(w.scaling() == "strong" and w.sharded for w in ranks)
            if cls is bench.BmmSoftmax:  # 8 items per rank per round
                assert all(len(w.plan.spans) == max(1, 64 // world // 8) for w in ranks)
            rep = cls(args, world, 0, replicas=True)
            assert rep.scaling() == "weak" and rep.flops == world * one.flops
    mm = bench.Matmul(args, 4, 1)
    assert not mm.sharded and mm.scaling() == "weak" and mm.flops == 4 * 2.0 * 512 ** 3


def test_bench_rounds_override_cpu():
    """`--rounds R` splits each rank's items into R rounds (at most one item
    each), and the job is the same whatever the split."""
    sys.path.insert(0, str(ROOT))
    import argparse
    import bench
    base = dict(batch=64, size=512, precision="tf32", bh=256, seq=2048, images=16,
                llama_batch=32, graph=None)
    one = bench.BmmSoftmax(argparse.Namespace(**base, rounds=0), 1, 0)
    for rounds, world, want in ((4, 8, 4), (1, 2, 1), (100, 8, 8)):
        ranks = [bench.BmmSoftmax(argparse.Namespace(**base, rounds=rounds), world, r)
                 for r in range(world)]
        assert all(len(w.plan.spans) == want for w in ranks)
        assert sum(w.local for w in ranks) == one.total
        assert all(w.flops == one.flops for w in ranks)
