"""GPU: every reference known-answer test, through the C ABI.

Each case is one `#[test]` of the reference crate (file:line in the case);
literal expectations are asserted as the Rust test does (exact or per-element
tolerance), `*_vs_cpu` cases against the oracle, `is_err()` cases must raise
AnyGpuError with status AGPU_ERR_SHAPE."""
from __future__ import annotations

import pytest

from conftest import KATS
from kat_runner import GPU_OPS, check, run_gpu, run_oracle

pytestmark = pytest.mark.gpu

CASES = [c for c in KATS if c["op"] in GPU_OPS]


@pytest.mark.parametrize("prec", ["tf32", "tf32x3", "ffma"])
@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_kat(dev, orc, case, prec):
    from any_gpu import AnyGpuError
    if prec != "tf32" and case["op"] not in ("matmul", "batch_matmul"):
        pytest.skip("precision only affects contractions")
    dev.set_precision(prec)
    try:
        if case["expect_err"]:
            with pytest.raises(AnyGpuError) as e:
                run_gpu(dev, case)
            assert e.value.status == 1
            return
        got = run_gpu(dev, case)
        want = run_oracle(orc, case) if case["expect"] == "oracle" else None
        check(case, got, want)
    finally:
        dev.set_precision("tf32")
