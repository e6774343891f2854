"""GPU parity of the attention backward (agpu_sdpa_backward) through the C ABI.

Against the oracle's restatement of the reference's SDPA composition
differentiated with its own rules (oracle.attention_backward), in TF32
(rel. Frobenius <= 1e-3) and in 3xTF32 / FFMA against float64 (<= 1e-5);
at the SDPA benchmark size (B8 H32 S2048 D128), sampled heads against
float64."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / np.linalg.norm(want))


def _f64_backward(q, k, v, do, s, d, causal):
    """dQ, dK, dV of one head in float64."""
    Q, K, V, dO = (x.reshape(s, d).astype(np.float64) for x in (q, k, v, do))
    sc = Q @ K.T / np.sqrt(d)
    if causal:
        sc[np.triu_indices(s, 1)] = -np.inf
    P = np.exp(sc - sc.max(axis=1, keepdims=True))
    P /= P.sum(axis=1, keepdims=True)
    dV = P.T @ dO
    dP = dO @ V.T
    dS = P * (dP - (P * dP).sum(axis=1, keepdims=True)) / np.sqrt(d)
    return dS @ K, dS.T @ Q, dV


def _inputs(bh, s, d, seed):
    r = np.random.default_rng(seed)
    return [r.standard_normal(bh * s * d).astype(np.float32) for _ in range(4)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("bh,s,d", [(4, 256, 128), (3, 200, 64), (2, 130, 64), (1, 512, 128)])
def test_sdpa_backward_tf32_vs_oracle(dev, orc, bh, s, d, causal):
    q, k, v, do = _inputs(bh, s, d, bh * s + d + causal)
    g = [dev.upload(x) for x in (q, k, v, do)]
    got = [dev.read(x) for x in dev.sdpa_backward(*g, bh, s, d, causal=causal)]
    want = orc.attention_backward(q, k, v, do, bh, s, d, causal=causal)
    for name, a, b in zip(("dq", "dk", "dv"), got, want):
        assert _rel(a, b) <= 1e-3, (name, _rel(a, b))


@pytest.mark.parametrize("prec", ["tf32x3", "ffma"])
def test_sdpa_backward_fp32_modes_vs_float64(dev, orc, prec):
    from any_gpu import GpuDevice
    bh, s, d = 2, 256, 64
    q, k, v, do = _inputs(bh, s, d, 5)
    g = [dev.upload(x) for x in (q, k, v, do)]
    with GpuDevice.precision(prec):
        got = [dev.read(x) for x in dev.sdpa_backward(*g, bh, s, d)]
    hs = s * d
    for h in range(bh):
        sl = slice(h * hs, (h + 1) * hs)
        want = _f64_backward(q[sl], k[sl], v[sl], do[sl], s, d, False)
        for name, a, w in zip(("dq", "dk", "dv"), got, want):
            assert _rel(a[sl], w) <= 1e-5, (prec, h, name, _rel(a[sl], w))


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("bh,s,d", [(16, 1024, 128), (24, 768, 64), (6, 1000, 64), (5, 2048, 128)])
def test_sdpa_backward_epilogue_way_vs_float64(dev, bh, s, d, causal):
    """Shapes whose S-sized products run on the CTA-pair GEMM: P formed in the
    S product's epilogue from the forward's row log-sum-exp, dS in the dP
    product's epilogue in place over P (D = rowsum(dO o O)).  Sampled heads
    against float64 within the TF32 tolerance."""
    q, k, v, do = _inputs(bh, s, d, bh + s + d + causal)
    g = [dev.upload(x) for x in (q, k, v, do)]
    got = [dev.read(x) for x in dev.sdpa_backward(*g, bh, s, d, causal=causal)]
    hs = s * d
    for h in sorted({0, bh // 2, bh - 1}):
        sl = slice(h * hs, (h + 1) * hs)
        want = _f64_backward(q[sl], k[sl], v[sl], do[sl], s, d, causal)
        for name, a, w in zip(("dq", "dk", "dv"), got, want):
            assert _rel(a[sl], w) <= 1e-3, (h, name, _rel(a[sl], w))


def test_sdpa_backward_head_chunks(dev):
    """S 4096: at most 2^30 score elements per chunk, so 70 heads run as 64 +
    6 (the epilogue way's last, smaller chunk included).  Heads on both sides
    of the chunk boundary against float64."""
    bh, s, d = 70, 4096, 64
    q, k, v, do = _inputs(bh, s, d, 70)
    g = [dev.upload(x) for x in (q, k, v, do)]
    got = [dev.read(x) for x in dev.sdpa_backward(*g, bh, s, d)]
    hs = s * d
    for h in (0, 63, 64, 69):
        sl = slice(h * hs, (h + 1) * hs)
        want = _f64_backward(q[sl], k[sl], v[sl], do[sl], s, d, False)
        for name, a, w in zip(("dq", "dk", "dv"), got, want):
            assert _rel(a[sl], w) <= 1e-3, (h, name, _rel(a[sl], w))


def test_sdpa_backward_launch_layer_unaligned_grad(dev):
    """Launch layer with dO 4 bytes off a 16-byte boundary at a shape that
    otherwise takes the epilogue way: the call checks every operand before
    launching and runs the row-kernel way (its dO products on the exact
    SIMT GEMM), still correct."""
    import torch
    bh, s, d = 16, 1024, 64
    q, k, v, do = _inputs(bh, s, d, 16)
    Q, K, V = (torch.from_numpy(x).cuda() for x in (q, k, v))
    DO = torch.zeros(bh * s * d + 1, device="cuda")
    DO[1:] = torch.from_numpy(do).cuda()
    dq, dk, dv = (torch.empty(bh * s * d, device="cuda") for _ in range(3))
    st = torch.cuda.Stream()
    dev.launch_sdpa_backward(Q.data_ptr(), K.data_ptr(), V.data_ptr(), DO.data_ptr() + 4,
                             dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), bh, s, d, False,
                             st.cuda_stream)
    st.synchronize()
    dev.synchronize()
    got = [x.cpu().numpy() for x in (dq, dk, dv)]
    hs = s * d
    for h in (0, bh - 1):
        sl = slice(h * hs, (h + 1) * hs)
        want = _f64_backward(q[sl], k[sl], v[sl], do[sl], s, d, False)
        for name, a, w in zip(("dq", "dk", "dv"), got, want):
            assert _rel(a[sl], w) <= 1e-3, (h, name, _rel(a[sl], w))


def test_sdpa_backward_both_ways_agree(dev, tmp_path):
    """The row-kernel way (AGPU_SDPA_BWD_FUSED=0, in a child process) and the
    epilogue way give the same gradients within the TF32 tolerance."""
    import os
    import subprocess
    import sys
    bh, s, d = 8, 1024, 128
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = [{os.path.join(root, 'any-gpu_b200')!r}, {root!r}]\n"
        "from tests.test_attention_bwd_gpu import _inputs\n"
        "from any_gpu import GpuDevice\n"
        "d = GpuDevice.gpu(0)\n"
        f"q, k, v, do = _inputs({bh}, {s}, {d}, 41)\n"
        "g = [d.upload(x) for x in (q, k, v, do)]\n"
        f"out = [d.read(x) for x in d.sdpa_backward(*g, {bh}, {s}, {d}, causal=True)]\n"
        f"np.save({str(tmp_path)!r} + '/g.npy', np.stack(out))\n"
        "d.close()\n")
    r = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True,
                       timeout=300, env=dict(os.environ, AGPU_SDPA_BWD_FUSED="0"))
    assert r.returncode == 0, r.stderr[-2000:]
    rows = np.load(tmp_path / "g.npy")
    q, k, v, do = _inputs(bh, s, d, 41)
    g = [dev.upload(x) for x in (q, k, v, do)]
    got = [dev.read(x) for x in dev.sdpa_backward(*g, bh, s, d, causal=True)]
    for name, a, b in zip(("dq", "dk", "dv"), got, rows):
        assert _rel(a, b) <= 1e-3, (name, _rel(a, b))


def test_sdpa_backward_benchmark_size_sampled(dev):
    """B8 H32 S2048 D128 (the SDPA benchmark config, the epilogue way): three
    heads against float64."""
    bh, s, d = 256, 2048, 128
    q, k, v, do = _inputs(bh, s, d, 77)
    g = [dev.upload(x) for x in (q, k, v, do)]
    got = [dev.read(x) for x in dev.sdpa_backward(*g, bh, s, d)]
    hs = s * d
    for h in (0, 131, 255):
        sl = slice(h * hs, (h + 1) * hs)
        want = _f64_backward(q[sl], k[sl], v[sl], do[sl], s, d, False)
        for name, a, w in zip(("dq", "dk", "dv"), got, want):
            assert _rel(a[sl], w) <= 1e-3, (h, name, _rel(a[sl], w))


def test_sdpa_backward_errors(dev):
    from any_gpu import AnyGpuError
    q = dev.upload(np.zeros(2 * 8 * 4, np.float32))
    bad = dev.upload(np.zeros(10, np.float32))
    with pytest.raises(AnyGpuError) as e:
        dev.sdpa_backward(q, q, q, bad, 2, 8, 4)
    assert e.value.status == 1
    with pytest.raises(AnyGpuError) as e:
        dev.sdpa_backward(q, bad, q, q, 2, 8, 4)
    assert e.value.status == 1
