"""Build libagpu.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python any-gpu_b200/build.py [--force] [-j N]

Objects go to any-gpu_b200/_build/, the shared library to
any-gpu_b200/any_gpu/libagpu.so (both git-ignored).  Every .cu under csrc/
is compiled with `-gencode arch=compute_100a,code=sm_100a -lineinfo`.
Incremental: a translation unit is rebuilt when it or any header is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "any_gpu" / "libagpu.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-v",
    "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path, force: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest:
        return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    logs = {}
    with cf.ThreadPoolExecutor(jobs) as ex:
        futs = {ex.submit(_compile, s, force): s for s in sources}
        objs = []
        for f in cf.as_completed(futs):
            obj, log = f.result()
            objs.append(obj)
            if log:
                logs[futs[f].name] = log
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest_obj:
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *sorted(map(str, objs)), "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    (BUILD / "ptxas.log").write_text("".join(f"== {k}\n{v}" for k, v in sorted(logs.items())))
    if verbose:
        for k, v in sorted(logs.items()):
            print(f"== {k}\n{v}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.v))
    sys.exit(0)
