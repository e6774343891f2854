"""GPU parity of the fp32-accuracy (3xTF32) contractions across the whole
benchmark range, through the C ABI.

The reference computes in exact fp32 (FFMA, src/ops/conv.rs:23-78); the
tensor-core 3xTF32 mode must stay within 1e-5 relative Frobenius error of
it at every size up to 8192^3.  At the large sizes the check is on sampled
output rows, against float64 and against the oracle's fp32 sequential sums
of the same rows (the oracle's own error grows with K, so the GPU must be
within 1e-5 of float64 and no further from the oracle than 1e-5 plus the
oracle's own distance from float64)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _uniform(seed, n):
    return np.random.default_rng(seed).uniform(-1, 1, n).astype(np.float32)


def _rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / np.linalg.norm(want))


@pytest.mark.parametrize("size", [2048, 4096, 8192])
def test_x3_square_large_k_sampled(dev, orc, size):
    """Square matmul in 3xTF32 at the top of the benchmark range (CTA-pair
    3xTF32 kernel, K segments summed in tensor memory)."""
    from any_gpu import GpuDevice
    m = n = k = size
    a, b = _uniform(40 + size, m * k), _uniform(41 + size, k * n)
    with GpuDevice.precision("tf32x3"):
        got = dev.read(dev.matmul(dev.upload(a), dev.upload(b), m, n, k)).reshape(m, n)
    rows = np.sort(np.random.default_rng(size).choice(m, 48, replace=False))
    A, B = a.reshape(m, k), b.reshape(k, n)
    want64 = A[rows].astype(np.float64) @ B.astype(np.float64)
    ref32 = orc.matmul(np.ascontiguousarray(A[rows]), b, len(rows), n, k,
                       threads=True).reshape(len(rows), n)
    e64 = _rel(got[rows], want64)
    eref = _rel(got[rows], ref32)
    ref_own = _rel(ref32, want64)
    assert e64 <= TOL, f"{size}^3: rel_fro vs float64 {e64:.3e}"
    assert eref <= TOL + ref_own, f"{size}^3: vs oracle {eref:.3e} (oracle vs f64 {ref_own:.3e})"
    # the tf32 result of the same product is measurably less accurate
    got32 = dev.read(dev.matmul(dev.upload(a), dev.upload(b), m, n, k)).reshape(m, n)
    assert _rel(got32[rows], want64) > 10 * e64


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("batch,m,n,k", [(2, 512, 768, 2048), (1, 300, 260, 1700)])
def test_x3_pair_operand_majors_and_tails(dev, orc, ta, tb, batch, m, n, k):
    """Every operand major on the 3xTF32 pair kernel, with tile tails in M, N
    and a K that is not a multiple of the segment length."""
    from any_gpu import GpuDevice
    r = np.random.default_rng(m + n + k)
    a = r.standard_normal(batch * m * k).astype(np.float32)
    b = r.standard_normal(batch * k * n).astype(np.float32)
    with GpuDevice.precision("tf32x3"):
        got = dev.read(dev.gemm(dev.upload(a), dev.upload(b), batch, m, n, k, ta, tb))
    A = a.reshape(batch, k, m).transpose(0, 2, 1) if ta else a.reshape(batch, m, k)
    B = b.reshape(batch, n, k).transpose(0, 2, 1) if tb else b.reshape(batch, k, n)
    want = np.matmul(A.astype(np.float64), B.astype(np.float64))
    assert _rel(got, want) <= TOL


@pytest.mark.parametrize("act", [0, 1, 2])
def test_x3_pair_fused_epilogue(dev, orc, act):
    """Bias, residual and activation applied once, after the last K segment."""
    from any_gpu import GpuDevice
    m, n, k = 512, 512, 1536
    r = np.random.default_rng(act)
    a = r.standard_normal(m * k).astype(np.float32)
    b = (r.standard_normal(k * n) / np.sqrt(k)).astype(np.float32)
    bias = r.standard_normal(n).astype(np.float32)
    res = r.standard_normal(m * n).astype(np.float32)
    with GpuDevice.precision("tf32x3"):
        got = dev.read(dev.gemm_ex(dev.upload(a), dev.upload(b), 1, m, n, k,
                                   bias=dev.upload(bias), resid=dev.upload(res), act=act))
    z = (a.reshape(m, k).astype(np.float64) @ b.reshape(k, n).astype(np.float64)
         + bias.astype(np.float64) + res.reshape(m, n).astype(np.float64))
    want = {0: z, 1: z / (1 + np.exp(-z)), 2: np.maximum(z, 0)}[act]
    assert _rel(got, want) <= TOL


def test_x3_batch_matmul_headline_shape_sampled(dev, orc):
    """The headline batch_matmul shape (batch 8 of 2048^3, N(0,1)*0.05) in
    3xTF32, sampled rows of each batch item against float64."""
    from any_gpu import GpuDevice
    batch, m, n, k = 8, 2048, 2048, 2048
    r = np.random.default_rng(77)
    a = (r.standard_normal(batch * m * k) * 0.05).astype(np.float32)
    b = (r.standard_normal(batch * k * n) * 0.05).astype(np.float32)
    with GpuDevice.precision("tf32x3"):
        got = dev.read(dev.batch_matmul(dev.upload(a), dev.upload(b), batch, m, n, k))
    got = got.reshape(batch, m, n)
    A, B = a.reshape(batch, m, k), b.reshape(batch, k, n)
    rows = np.arange(0, m, 97)
    for i in range(batch):
        want = A[i, rows].astype(np.float64) @ B[i].astype(np.float64)
        assert _rel(got[i, rows], want) <= TOL, i


def test_x3_conv2d_unet_full_size_sampled(dev, orc):
    """The UNet block's conv (16 x 320 x 64 x 64, 3x3, pad 1) in 3xTF32:
    sampled output planes against float64."""
    from any_gpu import GpuDevice
    n, c, h, w = 16, 320, 64, 64
    r = np.random.default_rng(5)
    x = r.standard_normal(n * c * h * w).astype(np.float32)
    bound = np.sqrt(6.0 / (c * 9))
    wt = r.uniform(-bound, bound, c * c * 9).astype(np.float32)
    with GpuDevice.precision("tf32x3"):
        y = dev.read(dev.conv2d(dev.upload(x), dev.upload(wt), None, n, c, h, w, c, 3, 3,
                                (1, 1), (1, 1))).reshape(n, c, h, w)
    X = np.pad(x.reshape(n, c, h, w).astype(np.float64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    W = wt.reshape(c, c, 3, 3).astype(np.float64)
    for img, oc in ((0, 0), (7, 161), (15, 319)):
        want = np.zeros((h, w))
        for dy in range(3):
            for dx in range(3):
                want += np.tensordot(W[oc, :, dy, dx], X[img, :, dy:dy + h, dx:dx + w], axes=1)
        assert _rel(y[img, oc], want) <= TOL, (img, oc)
