"""Shared pytest setup.

Markers:
  gpu  -- needs a CUDA B200 (run with `pytest -m gpu`); everything else runs
          on a CPU-only machine.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "any-gpu_b200"))
sys.path.insert(0, str(ROOT))

KATS = json.loads((ROOT / "tests" / "golden" / "reference_kats.json").read_text())["cases"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA B200 GPU")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def dev():
    """One device shared by all GPU tests (reference: TEST_DEV, src/ops/mod.rs:151-153)."""
    from any_gpu import GpuDevice
    d = GpuDevice.gpu(0)
    yield d
    d.close()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.build()
    return oracle


def assert_approx(got, want, tol):
    """Per-element absolute tolerance, as the reference's assert_approx
    (src/ops/mod.rs:155-165)."""
    import numpy as np
    got = np.asarray(got, dtype=np.float32).reshape(-1)
    want = np.asarray(want, dtype=np.float32).reshape(-1)
    assert got.shape == want.shape, f"length mismatch: got {got.size} want {want.size}"
    diff = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bad = np.nonzero(~(diff < tol))[0]
    assert bad.size == 0, (f"index {bad[0]}: got {got[bad[0]]}, want {want[bad[0]]} "
                           f"(diff {diff[bad[0]]}, tol {tol}); {bad.size} bad")
