"""GPU parity: seeded inputs through the C ABI against the oracle.

Tolerances (max relative Frobenius error vs the fp32 oracle):
  TF32 contractions          <= 1e-3
  3xTF32 / FFMA contractions <= 1e-5
  softmax / elementwise      <= 1e-5 (exact for add/sub/mul/relu/scale/transpose)
At full workload sizes the checks are sampled rows against float64 plus
size-independent properties (softmax rows sum to 1)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {"tf32": 1e-3, "tf32x3": 1e-5, "ffma": 1e-5}


def _uniform(seed, n):
    return np.random.default_rng(seed).uniform(-1, 1, n).astype(np.float32)


@pytest.mark.parametrize("prec", ["tf32", "tf32x3", "ffma"])
@pytest.mark.parametrize("size", [64, 128, 256, 512, 1024])
def test_matmul_square_sweep(dev, orc, size, prec):
    """Config: square matmul, A,B ~ U[-1,1), the bench sweep 64..1024."""
    m = n = k = size
    a, b = _uniform(1234, m * k), _uniform(1235, k * n)
    dev.set_precision(prec)
    try:
        got = dev.read(dev.matmul(dev.upload(a), dev.upload(b), m, n, k))
    finally:
        dev.set_precision("tf32")
    want = orc.matmul(a, b, m, n, k, threads=True)
    err = orc.rel_fro(got, want)
    assert err <= TOL[prec], f"{prec} {size}: rel_fro {err:.3e}"


@pytest.mark.parametrize("prec", ["tf32", "tf32x3"])
@pytest.mark.parametrize("m,n,k", [(300, 260, 100), (256, 96, 64), (128, 8, 36), (4, 512, 40),
                                   (520, 1000, 8), (129, 132, 516)])
def test_matmul_ragged_tensor_core(dev, orc, m, n, k, prec):
    """Tile tails in M, N and K on the tensor-core path (pitches % 16 B == 0)."""
    a, b = _uniform(m, m * k), _uniform(n + 7, k * n)
    dev.set_precision(prec)
    try:
        before = dev.launch_count
        got = dev.read(dev.matmul(dev.upload(a), dev.upload(b), m, n, k))
        # one GEMM launch; 3xTF32 on CTA pairs (m, n >= 256) adds its lo-split pass
        pair_x3 = prec == "tf32x3" and m >= 256 and n >= 256
        assert dev.launch_count == before + (2 if pair_x3 else 1)
    finally:
        dev.set_precision("tf32")
    want = orc.matmul(a, b, m, n, k, threads=True)
    assert orc.rel_fro(got, want) <= TOL[prec]


@pytest.mark.parametrize("m,n,k", [(17, 13, 11), (33, 65, 127), (1, 1, 1000), (200, 3, 7)])
def test_matmul_unaligned_simt(dev, orc, m, n, k):
    """Pitches that TMA cannot address run on the exact-fp32 SIMT kernel."""
    a, b = _uniform(5, m * k), _uniform(6, k * n)
    got = dev.read(dev.matmul(dev.upload(a), dev.upload(b), m, n, k))
    assert orc.rel_fro(got, orc.matmul(a, b, m, n, k)) <= 1e-5


@pytest.mark.parametrize("prec", ["tf32", "tf32x3"])
def test_batch_matmul_parity(dev, orc, prec):
    batch, m, n, k = 5, 256, 384, 512
    r = np.random.default_rng(2)
    a = (r.standard_normal(batch * m * k) * 0.05).astype(np.float32)
    b = (r.standard_normal(batch * k * n) * 0.05).astype(np.float32)
    dev.set_precision(prec)
    try:
        got = dev.read(dev.batch_matmul(dev.upload(a), dev.upload(b), batch, m, n, k))
    finally:
        dev.set_precision("tf32")
    want = orc.batch_matmul(a, b, batch, m, n, k, threads=True)
    assert orc.rel_fro(got, want) <= TOL[prec]


@pytest.mark.parametrize("prec", ["tf32", "tf32x3"])
@pytest.mark.parametrize("ta,tb", [(False, True), (True, False), (True, True)])
@pytest.mark.parametrize("batch,m,n,k", [(2, 256, 320, 96), (1, 132, 100, 516)])
def test_gemm_transposed_operands(dev, orc, ta, tb, batch, m, n, k, prec):
    """The backward GEMMs: MN-major A (A stored [k,m]) and K-major B (B stored [n,k])."""
    r = np.random.default_rng(batch * m + n)
    a = r.uniform(-1, 1, batch * m * k).astype(np.float32)
    b = r.uniform(-1, 1, batch * k * n).astype(np.float32)
    A = a.reshape(batch, k, m).transpose(0, 2, 1) if ta else a.reshape(batch, m, k)
    B = b.reshape(batch, n, k).transpose(0, 2, 1) if tb else b.reshape(batch, k, n)
    dev.set_precision(prec)
    try:
        got = dev.read(dev.gemm(dev.upload(a), dev.upload(b), batch, m, n, k, ta, tb))
    finally:
        dev.set_precision("tf32")
    want = orc.batch_matmul(np.ascontiguousarray(A), np.ascontiguousarray(B), batch, m, n, k)
    assert orc.rel_fro(got, want) <= TOL[prec]


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("batch,m,n,k", [(1, 256, 256, 256),     # 2 tiles of 256x128, 4 slices
                                         (1, 1024, 1024, 1024),  # 32 tiles of 256x128, 2 slices
                                         (2, 512, 512, 2048),    # 8 tiles of 256x256, 4 slices
                                         (1, 1280, 1536, 512),   # 30 tiles of 256x256, 2 slices
                                         (1, 300, 520, 132)])    # 256x128, ragged M, N and K
def test_gemm_split_k_cluster(dev, orc, ta, tb, batch, m, n, k):
    """GEMMs with too few 256 x 256 tiles for the SM pairs run K-split over a
    cluster of pairs (256 x 256 or 256 x 128 tiles, 4 or 2 slices), the
    partials summed through distributed shared memory."""
    r = np.random.default_rng(m + n + k)
    a = r.uniform(-1, 1, batch * m * k).astype(np.float32)
    b = r.uniform(-1, 1, batch * k * n).astype(np.float32)
    A = a.reshape(batch, k, m).transpose(0, 2, 1) if ta else a.reshape(batch, m, k)
    B = b.reshape(batch, n, k).transpose(0, 2, 1) if tb else b.reshape(batch, k, n)
    before = dev.launch_count
    got = dev.read(dev.gemm(dev.upload(a), dev.upload(b), batch, m, n, k, ta, tb))
    assert dev.launch_count - before == 1
    want = orc.batch_matmul(np.ascontiguousarray(A), np.ascontiguousarray(B), batch, m, n, k,
                            threads=True)
    assert orc.rel_fro(got, want) <= 1e-3
    again = dev.read(dev.gemm(dev.upload(a), dev.upload(b), batch, m, n, k, ta, tb))
    np.testing.assert_array_equal(got, again)  # fixed summation order


_CHUNK_CASES = [(1, 512, 1024, 768, True, False, "tf32"),    # split-K, MN-major A and B
                 (2, 1024, 2048, 512, True, False, "tf32"),   # pair kernel, MN-major A and B
                 (1, 2048, 2048, 256, False, False, "tf32"),  # pair kernel, MN-major B
                 (2, 128, 1024, 384, True, False, "tf32"),    # single-CTA kernel (m < 256)
                 (1, 384, 512, 256, True, False, "tf32x3")]   # single-CTA 3xTF32 (exact maps)


def _chunk_case_inputs(batch, m, n, k):
    r = np.random.default_rng(m + 3 * n + 7 * k)
    return (r.uniform(-1, 1, batch * m * k).astype(np.float32),
            r.uniform(-1, 1, batch * k * n).astype(np.float32))


def test_gemm_chunked_operand_maps_bit_identical(dev, tmp_path):
    """MN-major operands with MN % 32 == 0 load through one 4-D TMA box per
    stage; the shared-memory image, hence every output bit, equals the one
    the per-32-column loads give (AGPU_GEMM_CHUNKED=0, in a child process)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = [{os.path.join(root, 'any-gpu_b200')!r}, {root!r}]\n"
        "from tests.test_parity_gpu import _CHUNK_CASES, _chunk_case_inputs\n"
        "from any_gpu import GpuDevice\n"
        "d = GpuDevice.gpu(0)\n"
        "for i, (batch, m, n, k, ta, tb, prec) in enumerate(_CHUNK_CASES):\n"
        "    a, b = _chunk_case_inputs(batch, m, n, k)\n"
        "    d.set_precision(prec)\n"
        "    got = d.read(d.gemm(d.upload(a), d.upload(b), batch, m, n, k, ta, tb))\n"
        f"    np.save({str(tmp_path)!r} + f'/c{{i}}.npy', got)\n"
        "d.close()\n")
    env = dict(os.environ, AGPU_GEMM_CHUNKED="0")
    out = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    for i, (batch, m, n, k, ta, tb, prec) in enumerate(_CHUNK_CASES):
        a, b = _chunk_case_inputs(batch, m, n, k)
        dev.set_precision(prec)
        try:
            got = dev.read(dev.gemm(dev.upload(a), dev.upload(b), batch, m, n, k, ta, tb))
        finally:
            dev.set_precision("tf32")
        np.testing.assert_array_equal(got, np.load(tmp_path / f"c{i}.npy"))


@pytest.mark.parametrize("act", [0, 1, 2])
def test_gemm_split_k_epilogue(dev, orc, act):
    """bias + residual + activation applied once, after the K-slice sum."""
    m, n, k = 512, 768, 1024
    r = np.random.default_rng(act)
    a = (r.standard_normal(m * k) * 0.05).astype(np.float32)
    b = (r.standard_normal(k * n) * 0.05).astype(np.float32)
    bias = r.standard_normal(n).astype(np.float32)
    res = r.standard_normal(m * n).astype(np.float32)
    got = dev.read(dev.gemm_ex(dev.upload(a), dev.upload(b), 1, m, n, k, bias=dev.upload(bias),
                               resid=dev.upload(res), act=act))
    z = orc.matmul(a, b, m, n, k, threads=True).reshape(m, n) + bias + res.reshape(m, n)
    want = {0: z, 1: z / (1 + np.exp(-z)), 2: np.maximum(z, 0)}[act].ravel()
    assert orc.rel_fro(got, want) <= 1e-3


@pytest.mark.parametrize("rows,cols", [(1000, 2048), (513, 1000), (64, 4), (77, 37),
                                       (9, 5000), (3, 1), (4096, 128), (2, 100000)])
def test_softmax_parity(dev, orc, rows, cols):
    """Against the oracle within 1e-5, except where the reference's own
    sequential fp32 sum drifts (long rows): then the GPU must be at least as
    close to the float64 softmax as the reference algorithm is."""
    x = (np.random.default_rng(rows * cols).standard_normal(rows * cols) * 3).astype(np.float32)
    got = dev.read(dev.softmax(dev.upload(x), rows, cols))
    want = orc.softmax(x, rows, cols, threads=True)
    X = x.reshape(rows, cols).astype(np.float64)
    E = np.exp(X - X.max(1, keepdims=True))
    ref64 = E / E.sum(1, keepdims=True)
    err_orc = orc.rel_fro(want, ref64)
    assert orc.rel_fro(got, ref64) <= max(1e-5, err_orc)
    assert orc.rel_fro(got, want) <= 1e-5 + err_orc
    sums = got.reshape(rows, cols).astype(np.float64).sum(1)
    assert np.all(np.abs(sums - 1) < 1e-4)


EXACT = ["add", "sub", "mul", "relu", "scale", "relu_backward"]
APPROX = ["sigmoid", "swish", "tanh", "sigmoid_backward", "swish_backward", "tanh_backward"]


@pytest.mark.parametrize("n", [1, 3, 1000003, 4 << 20])
@pytest.mark.parametrize("op", EXACT + APPROX)
def test_elementwise_parity(dev, orc, op, n):
    r = np.random.default_rng(n)
    a = (r.standard_normal(n) * 4).astype(np.float32)
    b = (r.standard_normal(n) * 4).astype(np.float32)
    if op in ("sigmoid_backward",):
        b = (1 / (1 + np.exp(-b))).astype(np.float32)
    if op in ("tanh_backward",):
        b = np.tanh(b).astype(np.float32)
    A, B = dev.upload(a), dev.upload(b)
    if op == "scale":
        got, want = dev.read(dev.scale(A, -0.37)), orc.elementwise("scale", a, None, -0.37)
    elif op in ("relu", "sigmoid", "swish"):
        got, want = dev.read(getattr(dev, op)(A)), orc.elementwise(op, a)
    elif op == "tanh":
        got, want = dev.read(dev.tanh_act(A)), orc.elementwise("tanh", a)
    else:
        got, want = dev.read(getattr(dev, op)(A, B)), orc.elementwise(op, a, b)
    if op in EXACT:
        np.testing.assert_array_equal(got, want)
    else:
        assert orc.rel_fro(got, want) <= 1e-5
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("outer,d0,d1,inner", [(1, 1000, 700, 1), (256, 2048, 128, 1),
                                               (3, 5, 7, 9), (2, 64, 33, 128), (1, 1, 1, 1)])
def test_transpose_parity(dev, orc, outer, d0, d1, inner):
    a = np.arange(outer * d0 * d1 * inner, dtype=np.float32)
    got = dev.read(dev.transpose(dev.upload(a), outer, d0, d1, inner))
    np.testing.assert_array_equal(got, orc.transpose(a, outer, d0, d1, inner))
    back = dev.read(dev.transpose(dev.upload(got), outer, d1, d0, inner))
    np.testing.assert_array_equal(back, a)


def test_add_per_col_parity(dev, orc):
    r = np.random.default_rng(11)
    for rows, cols in [(1000, 4096), (7, 13)]:
        a = r.standard_normal(rows * cols).astype(np.float32)
        b = r.standard_normal(cols).astype(np.float32)
        got = dev.read(dev.add_per_col(dev.upload(a), dev.upload(b), rows, cols))
        np.testing.assert_array_equal(got, orc.add_per_col(a, b, rows, cols))


def test_batch_matmul_softmax_full_config(dev, orc):
    """The headline workload at full size: batch 64, M=K=N=2048, inputs
    N(0,1)*0.05, then row softmax.  Checked on sampled rows against float64
    and by the row-sum property on every row."""
    batch = m = None
    batch, m, n, k = 64, 2048, 2048, 2048
    r = np.random.default_rng(1235)
    a = (r.standard_normal(batch * m * k, dtype=np.float32) * np.float32(0.05))
    b = (r.standard_normal(batch * k * n, dtype=np.float32) * np.float32(0.05))
    A, B = dev.upload(a), dev.upload(b)
    C = dev.batch_matmul(A, B, batch, m, n, k)
    S = dev.softmax(C, batch * m, n)
    c = dev.read(C).reshape(batch, m, n)
    s = dev.read(S).reshape(batch, m, n)
    sums = s.astype(np.float64).sum(-1)
    assert np.abs(sums - 1).max() < 1e-4
    av, bv = a.reshape(batch, m, k), b.reshape(batch, k, n)
    for bi in (0, 31, 63):
        rows = np.array([0, 1, 777, 2047])
        want = av[bi, rows].astype(np.float64) @ bv[bi].astype(np.float64)
        assert orc.rel_fro(c[bi, rows], want) <= 1e-3
        e = np.exp(want - want.max(-1, keepdims=True))
        assert orc.rel_fro(s[bi, rows], e / e.sum(-1, keepdims=True)) <= 1e-3


def _gn64(x, gamma, beta, n, c, s, g, eps):
    X = np.asarray(x, np.float64).reshape(n, g, -1)
    Y = (X - X.mean(-1, keepdims=True)) / np.sqrt(X.var(-1, keepdims=True) + eps)
    return (Y.reshape(n, c, s) * np.asarray(gamma, np.float64)[None, :, None]
            + np.asarray(beta, np.float64)[None, :, None]).ravel()


@pytest.mark.parametrize("swish", [False, True])
@pytest.mark.parametrize("n,c,s,g", [(16, 320, 4096, 32),   # UNet block: 5 chunks per group
                                     (2, 40, 4096, 8),       # ragged last chunk (20480)
                                     (2, 64, 4096, 4),       # 65536 per group: 8-CTA cluster
                                     (1, 64, 4096, 2),       # 16 chunks per group
                                     (2, 64, 1024, 32),      # 2 channels x 1024 per group
                                     (3, 12, 37, 4),         # spatial % 4 != 0: chunked path
                                     (1, 4, 300000, 2),      # 600k-element groups: chunked
                                     (1, 2, 2621440, 1),     # 640 chunks in one group: more
                                                             # than the resident CTAs roll
                                     (2, 6, 8, 6)])          # per-channel groups
def test_group_norm_parity(dev, orc, n, c, s, g, swish):
    """The UNet block's group_norm (eps 1e-5, gamma 1, beta 0 there) and ragged shapes
    against the oracle; tolerance as for softmax (the reference's E[x^2]-mean^2
    in sequential fp32 drifts on large groups)."""
    r = np.random.default_rng(n * c + s)
    x = r.standard_normal(n * c * s).astype(np.float32)
    gamma = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    beta = (0.1 * r.standard_normal(c)).astype(np.float32)
    X, G, B = dev.upload(x), dev.upload(gamma), dev.upload(beta)
    fn = dev.group_norm_swish if swish else dev.group_norm
    got = dev.read(fn(X, G, B, n, c, s, g, 1e-5))
    want = orc.group_norm(x, gamma, beta, n, c, s, g, 1e-5, threads=True)
    ref64 = _gn64(x, gamma, beta, n, c, s, g, 1e-5)
    if swish:
        want = orc.elementwise("swish", want)
        ref64 = ref64 / (1 + np.exp(-ref64))
    err_orc = orc.rel_fro(want, ref64)
    assert orc.rel_fro(got, ref64) <= max(1e-5, err_orc)
    assert orc.rel_fro(got, want) <= 1e-5 + err_orc


@pytest.mark.parametrize("n,c,s,g", [(16, 320, 4096, 32),   # UNet block shape
                                     (1, 4, 10000, 2),       # rows of 3 chunks (4096 each)
                                     (3, 12, 37, 4),         # ragged rows
                                     (2, 64, 1, 32),         # one element per row
                                     (2, 6, 8, 6)])          # per-channel groups
def test_group_norm_backward_parity(dev, orc, n, c, s, g):
    """group_norm_backward (src/ops/norm.rs:282) against the oracle's
    restatement of the reference shaders and against torch autograd in
    float64; the GPU must be within 1e-5 of float64 or as close as the
    oracle (the shaders' E[x^2]-mean^2 and sequential fp32 sums drift)."""
    from test_oracle import gn_backward_f64
    r = np.random.default_rng(n * c + s + 7)
    x = r.standard_normal(n * c * s).astype(np.float32)
    dy = r.standard_normal(n * c * s).astype(np.float32)
    gamma = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    outs = dev.group_norm_backward(dev.upload(dy), dev.upload(x), dev.upload(gamma), n, c, s, g,
                                   1e-5)
    got = [dev.read(o) for o in outs]
    want = orc.group_norm_backward(dy, x, gamma, n, c, s, g, 1e-5)
    ref = gn_backward_f64(dy, x, gamma, n, c, s, g, 1e-5)
    for name, a, b, f in zip(("d_input", "d_gamma", "d_beta"), got, want, ref):
        err_orc = orc.rel_fro(b, f)
        assert orc.rel_fro(a, f) <= max(1e-5, err_orc), name
        assert orc.rel_fro(a, b) <= 1e-5 + err_orc, name


def test_group_norm_backward_errors(dev):
    from any_gpu import AnyGpuError
    ones = lambda k: dev.upload(np.ones(k, np.float32))
    cases = [((ones(16), ones(10), ones(4)), (1, 4, 4, 2)),   # input size mismatch
             ((ones(10), ones(16), ones(4)), (1, 4, 4, 2)),   # grad_out size mismatch
             ((ones(16), ones(16), ones(3)), (1, 4, 4, 2)),   # gamma size
             ((ones(5), ones(5), ones(5)), (1, 5, 1, 2))]     # channels % groups
    for (go, x, gm), args in cases:
        with pytest.raises(AnyGpuError) as e:
            dev.group_norm_backward(go, x, gm, *args, 1e-5)
        assert e.value.status == 1


@pytest.mark.parametrize("batch,m,n,k", [(3, 300, 264, 520), (2, 256, 2048, 256)])
def test_batch_matmul_softmax(dev, orc, batch, m, n, k):
    """The fused entry point equals batch_matmul followed by softmax."""
    r = np.random.default_rng(m + n)
    a = (r.standard_normal(batch * m * k) * 0.05).astype(np.float32)
    b = (r.standard_normal(batch * k * n) * 0.05).astype(np.float32)
    got = dev.read(dev.batch_matmul_softmax(dev.upload(a), dev.upload(b), batch, m, n, k))
    prod = np.concatenate([orc.matmul(a[i * m * k:(i + 1) * m * k], b[i * k * n:(i + 1) * k * n],
                                      m, n, k, threads=True) for i in range(batch)])
    want = orc.softmax(prod, batch * m, n, threads=True)
    assert orc.rel_fro(got, want) <= 1e-3
    # and exactly the two separate calls
    sep = dev.read(dev.softmax(dev.batch_matmul(dev.upload(a), dev.upload(b), batch, m, n, k),
                               batch * m, n))
    np.testing.assert_array_equal(got, sep)


@pytest.mark.parametrize("batch,k", [(8, 256),    # 2 pieces of 4 x 64 tiles
                                     (13, 64),    # 4 pieces of 3-4 x 64 tiles
                                     (24, 32)])   # 8 pieces of 3 x 64 tiles
def test_batch_matmul_softmax_two_streams(dev, batch, k):
    """A batch large enough to run in pieces on two streams (each piece's
    softmax beside the next piece's GEMM) equals the separate calls, through
    both the buffer and the launch layer."""
    import torch
    m = n = 2048
    r = np.random.default_rng(batch)
    a = (r.standard_normal(batch * m * k) * 0.05).astype(np.float32)
    b = (r.standard_normal(batch * k * n) * 0.05).astype(np.float32)
    A, B = dev.upload(a), dev.upload(b)
    got = dev.read(dev.batch_matmul_softmax(A, B, batch, m, n, k))
    sep = dev.read(dev.softmax(dev.batch_matmul(A, B, batch, m, n, k), batch * m, n))
    np.testing.assert_array_equal(got, sep)
    out = torch.empty(batch * m * n, device="cuda")
    s = torch.cuda.Stream()
    dev.launch_batch_matmul_softmax(A.device_ptr, B.device_ptr, out.data_ptr(), batch, m, n, k,
                                    s.cuda_stream)
    s.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), sep)


@pytest.mark.parametrize("n,c,s,g", [(16, 320, 4096, 32), (3, 12, 37, 4)])
def test_group_norm_in_place(dev, orc, n, c, s, g):
    """y may alias x: every chunk is read (twice) before it is overwritten."""
    r = np.random.default_rng(n + c + s)
    x = r.standard_normal(n * c * s).astype(np.float32)
    gamma = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
    beta = (0.1 * r.standard_normal(c)).astype(np.float32)
    X, G, B = dev.upload(x), dev.upload(gamma), dev.upload(beta)
    want = dev.read(dev.group_norm_swish(X, G, B, n, c, s, g, 1e-5))
    dev.launch_group_norm(X.device_ptr, G.device_ptr, B.device_ptr, X.device_ptr, n, c, s, g,
                          1e-5, swish=True)
    np.testing.assert_array_equal(dev.read(X), want)


def test_group_norm_errors(dev):
    from any_gpu import AnyGpuError
    x = dev.upload(np.ones(10, np.float32))
    g = dev.upload(np.ones(5, np.float32))
    for args in [(1, 5, 2, 2), (1, 5, 2, 3), (2, 5, 2, 5)]:
        with pytest.raises(AnyGpuError) as e:
            dev.group_norm(x, g, g, *args, 1e-5)
        assert e.value.status == 1


CONV_CASES = [
    # n, cin, h, w, cout, k, stride, pad, dil, groups
    (2, 320, 32, 32, 320, 3, 1, 1, 1, 1),   # UNet block channels (tensor-core path, BN=160)
    (1, 3, 17, 19, 64, 3, 1, 1, 1, 1),      # Cin=3 staged to 4 channels, ragged 19-wide rows
    (2, 64, 56, 56, 128, 1, 1, 0, 1, 1),    # 1x1
    (1, 32, 24, 24, 48, 5, 1, 2, 1, 1),     # 5x5, Cout=48 (BN=64 tail)
    (1, 40, 20, 30, 256, 3, 1, 2, 2, 1),    # dilation 2
    (1, 16, 33, 33, 32, 3, 2, 1, 1, 1),     # stride 2 -> direct kernel
    (2, 8, 12, 12, 8, 3, 1, 1, 1, 2),       # groups 2 -> direct kernel
    (5, 64, 20, 24, 320, 3, 1, 1, 1, 1),    # 5 images: halves of 2 and 3 on two streams
    (4, 96, 16, 16, 256, 3, 1, 1, 1, 1),    # 4 images, 256-wide pair tiles, two halves
]


@pytest.mark.parametrize("prec", ["tf32", "tf32x3"])
@pytest.mark.parametrize("case", CONV_CASES, ids=[str(c) for c in CONV_CASES])
def test_conv2d_parity(dev, orc, case, prec):
    n, cin, h, w, cout, k, s, p, d, g = case
    r = np.random.default_rng(cin * cout + h)
    x = r.standard_normal(n * cin * h * w).astype(np.float32)
    bound = np.sqrt(6.0 / (cin // g * k * k))  # Kaiming-uniform, gain sqrt(2)
    wt = r.uniform(-bound, bound, cout * (cin // g) * k * k).astype(np.float32)
    bias = r.standard_normal(cout).astype(np.float32)
    dev.set_precision(prec)
    try:
        got = dev.read(dev.conv2d(dev.upload(x), dev.upload(wt), dev.upload(bias), n, cin, h, w,
                                  cout, k, k, (s, s), (p, p), (d, d), g))
    finally:
        dev.set_precision("tf32")
    want = orc.conv2d(x, wt, bias, n, cin, h, w, cout, k, k, (s, s), (p, p), (d, d), g,
                      threads=True)
    assert orc.rel_fro(got, want) <= TOL[prec]


def test_conv2d_unet_full_size_sampled(dev, orc):
    """The UNet block's conv at full size (N16, 320->320, 64x64, 3x3 pad 1), Kaiming-
    uniform weights, bias 0: sampled output planes against float64."""
    n, c, h, w = 16, 320, 64, 64
    r = np.random.default_rng(1237)
    x = r.standard_normal(n * c * h * w, dtype=np.float32)
    bound = np.float32(np.sqrt(6.0 / (c * 9)))
    wt = r.uniform(-bound, bound, c * c * 9).astype(np.float32)
    y = dev.read(dev.conv2d(dev.upload(x), dev.upload(wt), None, n, c, h, w, c, 3, 3, (1, 1),
                            (1, 1), (1, 1), 1)).reshape(n, c, h, w)
    X = np.pad(x.reshape(n, c, h, w).astype(np.float64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    W = wt.reshape(c, c, 3, 3).astype(np.float64)
    for ni, oc in [(0, 0), (7, 159), (15, 319), (3, 160)]:
        ref = np.zeros((h, w))
        for i in range(3):
            for j in range(3):
                ref += np.einsum("chw,c->hw", X[ni, :, i:i + h, j:j + w], W[oc, :, i, j])
        assert orc.rel_fro(y[ni, oc], ref) <= 1e-3


def test_conv_backward_ops_parity(dev, orc):
    r = np.random.default_rng(77)
    n, cin, h, w, cout, k = 2, 6, 9, 8, 4, 3
    x = r.standard_normal(n * cin * h * w).astype(np.float32)
    oh = ow_ = None
    for s, p, d in [(1, 1, 1), (2, 0, 1), (1, 2, 2)]:
        oh = (h + 2 * p - d * (k - 1) - 1) // s + 1
        ow_ = (w + 2 * p - d * (k - 1) - 1) // s + 1
        gy = r.standard_normal(n * cout * oh * ow_).astype(np.float32)
        gw = dev.read(dev.conv2d_grad_weight(dev.upload(x), dev.upload(gy), n, cin, h, w, cout,
                                             oh, ow_, k, k, s, s, p, p, d, d, 1))
        want = orc.conv2d_grad_weight(x, gy, n, cin, h, w, cout, oh, ow_, k, k, s, s, p, p, d, d,
                                      1)
        assert orc.rel_fro(gw, want) <= 1e-5
        gb = dev.read(dev.conv2d_grad_bias(dev.upload(gy), n, cout, oh, ow_))
        assert orc.rel_fro(gb, orc.conv2d_grad_bias(gy, n, cout, oh, ow_)) <= 1e-5
    # transposed conv with stride, padding, output padding, groups
    for s, p, op_, d, g in [(2, 1, 1, 1, 1), (1, 0, 0, 2, 2), (3, 2, 0, 1, 1)]:
        wt = r.standard_normal(cin * (cout // g) * k * k).astype(np.float32)
        bias = r.standard_normal(cout).astype(np.float32)
        got = dev.read(dev.conv_transpose2d(dev.upload(x), dev.upload(wt), dev.upload(bias), n,
                                            cin, h, w, cout, k, k, (s, s), (p, p), (op_, op_),
                                            (d, d), g))
        want = orc.conv_transpose2d(x, wt, bias, n, cin, h, w, cout, k, k, (s, s), (p, p),
                                    (op_, op_), (d, d), g)
        assert orc.rel_fro(got, want) <= 1e-5


@pytest.mark.parametrize("prec,tol", [("tf32", 1e-3), ("tf32x3", 1e-5)])
@pytest.mark.parametrize("p,d,bias", [(1, 1, True), (2, 2, False), (0, 1, True)])
def test_conv_transpose2d_tensor_core(dev, orc, prec, tol, p, d, bias):
    """Stride-1 conv_transpose2d (the conv backward's input gradient) on the
    tensor-core implicit GEMM: conv2d with the channel-swapped, tap-reversed
    weight and padding d*(k-1)-p, against the oracle's restatement of the
    reference shader."""
    n, cin, h, w, cout, k = 2, 96, 32, 24, 64, 3
    r = np.random.default_rng(p * 10 + d)
    x = r.standard_normal(n * cin * h * w).astype(np.float32)
    wt = (r.standard_normal(cin * cout * k * k) * 0.05).astype(np.float32)
    b = r.standard_normal(cout).astype(np.float32) if bias else None
    dev.set_precision(prec)
    try:
        got = dev.read(dev.conv_transpose2d(dev.upload(x), dev.upload(wt),
                                            dev.upload(b) if bias else None, n, cin, h, w, cout,
                                            k, k, (1, 1), (p, p), (0, 0), (d, d), 1))
    finally:
        dev.set_precision("tf32")
    want = orc.conv_transpose2d(x, wt, b, n, cin, h, w, cout, k, k, (1, 1), (p, p), (0, 0),
                                (d, d), 1)
    assert orc.rel_fro(got, want) <= tol


@pytest.mark.parametrize("prec,tol", [("tf32", 1e-3), ("tf32x3", 1e-5)])
@pytest.mark.parametrize("cin,cout,p,d", [(96, 64, 1, 1), (320, 160, 2, 2), (40, 48, 1, 1)])
def test_conv2d_grad_weight_tensor_core(dev, orc, prec, tol, cin, cout, p, d):
    """Stride-1 weight gradient as per-tap implicit GEMMs on the tensor cores
    (K split over pixel ranges, ranges summed in order), against the oracle's
    restatement of the reference shader."""
    n, h, w, k = 2, 16, 64, 3
    ho, wo = h + 2 * p - d * (k - 1), w + 2 * p - d * (k - 1)
    r = np.random.default_rng(cin + p)
    x = r.standard_normal(n * cin * h * w).astype(np.float32)
    gy = r.standard_normal(n * cout * ho * wo).astype(np.float32)
    dev.set_precision(prec)
    try:
        got = dev.read(dev.conv2d_grad_weight(dev.upload(x), dev.upload(gy), n, cin, h, w, cout,
                                              ho, wo, k, k, 1, 1, p, p, d, d, 1))
    finally:
        dev.set_precision("tf32")
    want = orc.conv2d_grad_weight(x, gy, n, cin, h, w, cout, ho, wo, k, k, 1, 1, p, p, d, d, 1)
    assert orc.rel_fro(got, want) <= tol


def test_adamw_multi_tensor(dev, orc):
    """AdamW (src/optim.rs:53-138) over three steps on tensors of ragged sizes
    (one launch per step), against the oracle's restatement of the shader."""
    from any_gpu import AdamW
    r = np.random.default_rng(21)
    sizes = [1, 7, 1000, (1 << 20) + 3, 4096]
    ps = [r.standard_normal(n).astype(np.float32) for n in sizes]
    bufs = [dev.upload(p) for p in ps]
    opt = AdamW(lr=1e-3)
    ms = [np.zeros(n, np.float32) for n in sizes]
    vs = [np.zeros(n, np.float32) for n in sizes]
    for t in (1, 2, 3):
        gs = [r.standard_normal(n).astype(np.float32) for n in sizes]
        opt.step(dev, bufs, [dev.upload(g) for g in gs])
        for i in range(len(sizes)):
            ps[i], ms[i], vs[i] = orc.adamw(ps[i], gs[i], ms[i], vs[i], 1e-3, 0.9, 0.999, 1e-8,
                                            0.01, t)
    # per element: the GPU contracts a*b + c into one FMA where the oracle
    # rounds twice, and m = 0.9 m + 0.1 g can nearly cancel for a single value
    for i, b in enumerate(bufs):
        np.testing.assert_allclose(dev.read(b), ps[i], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(dev.read(opt.states[i][0]), ms[i], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(dev.read(opt.states[i][1]), vs[i], rtol=1e-5, atol=1e-6)


def test_adamw_reference_tests(dev):
    """The reference's AdamW tests (src/optim.rs:149-240) through AdamW.step."""
    from any_gpu import AdamW
    up = lambda *x: dev.upload(np.array(x, np.float32))
    opt = AdamW(lr=0.01)
    opt.weight_decay = 0.0
    p = up(1, 2, 3)
    opt.step(dev, [p], [up(0.1, 0.2, 0.3)])
    assert (dev.read(p) < np.array([1, 2, 3], np.float32)).all()
    opt, p, g = AdamW(lr=0.1), up(10), up(1)
    opt.weight_decay = 0.0
    for _ in range(10):
        opt.step(dev, [p], [g])
    assert dev.read(p)[0] < 10.0
    opt, p = AdamW(lr=0.01), up(10)
    opt.weight_decay = 0.1
    opt.step(dev, [p], [up(0)])
    assert abs(dev.read(p)[0] - 9.99) <= 1e-3
    opt, p = AdamW(lr=0.01), up(5)
    opt.weight_decay = 0.0
    opt.step(dev, [p], [up(-1)])
    assert dev.read(p)[0] > 5.0
    opt, p = AdamW(lr=0.0), up(10)                     # test_adamw_lr_zero
    opt.weight_decay = 0.0
    opt.step(dev, [p], [up(100)])
    assert abs(dev.read(p)[0] - 10.0) <= 1e-5
    opt = AdamW(lr=0.001)                              # test_adamw_defaults
    assert (opt.lr, opt.beta1, opt.beta2, opt.eps, opt.weight_decay) == (0.001, 0.9, 0.999, 1e-8,
                                                                          0.01)


def test_adamw_errors(dev):
    from any_gpu import AdamW, AnyGpuError
    opt = AdamW(lr=1e-3)
    with pytest.raises(AnyGpuError) as e:  # src/optim.rs:95
        opt.step(dev, [dev.upload(np.ones(4, np.float32))], [dev.upload(np.ones(5, np.float32))])
    assert e.value.status == 1
    with pytest.raises(AnyGpuError):  # src/optim.rs:83: two params, one grad
        AdamW(lr=0.01).step(dev, [dev.upload(np.ones(1, np.float32))] * 2,
                            [dev.upload(np.ones(1, np.float32))])


def test_alloc_is_zero_filled(dev):
    assert not dev.read(dev.alloc(12345)).any()


def _attn64(q, k, v, bh, s, d, causal=False, rows=None):
    Q = q.reshape(bh, s, d).astype(np.float64)
    K = k.reshape(bh, s, d).astype(np.float64)
    V = v.reshape(bh, s, d).astype(np.float64)
    if rows is not None:
        Q = Q[:, rows]
    S = Q @ K.transpose(0, 2, 1) / np.sqrt(d)
    if causal:
        r = np.arange(s) if rows is None else np.asarray(rows)
        S = np.where(np.arange(s)[None, None, :] > r[None, :, None], -np.inf, S)
    P = np.exp(S - S.max(-1, keepdims=True))
    P /= P.sum(-1, keepdims=True)
    return P @ V


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("bh,s,d", [(4, 256, 128), (2, 200, 64), (3, 64, 128), (6, 128, 128), (2, 333, 128),
                                    (1, 1000, 64), (5, 7, 16), (2, 65, 32)])
def test_sdpa_parity(dev, orc, bh, s, d, causal):
    """Tensor-core flash kernel (d 64/128) and the SIMT kernel (other d) against
    the oracle; Q,K,V ~ N(0,1) as in the SDPA config; TF32 tolerance."""
    r = np.random.default_rng(bh * s + d)
    q, k, v = (r.standard_normal(bh * s * d).astype(np.float32) for _ in range(3))
    Q, K, V = dev.upload(q), dev.upload(k), dev.upload(v)
    fn = dev.sdpa_causal if causal else dev.scaled_dot_product_attention
    got = dev.read(fn(Q, K, V, bh, s, d))
    want = orc.attention(q, k, v, bh, s, d, threads=not causal, causal=causal)
    assert orc.rel_fro(got, want) <= 1e-3
    assert orc.rel_fro(got, _attn64(q, k, v, bh, s, d, causal).ravel()) <= 1e-3


@pytest.mark.parametrize("prec", ["tf32x3", "ffma"])
def test_sdpa_fp32_modes_are_exact(dev, orc, prec):
    bh, s, d = 2, 192, 128
    r = np.random.default_rng(5)
    q, k, v = (r.standard_normal(bh * s * d).astype(np.float32) for _ in range(3))
    dev.set_precision(prec)
    try:
        got = dev.read(dev.scaled_dot_product_attention(dev.upload(q), dev.upload(k),
                                                        dev.upload(v), bh, s, d))
    finally:
        dev.set_precision("tf32")
    assert orc.rel_fro(got, orc.attention(q, k, v, bh, s, d, threads=True)) <= 1e-5


def test_sdpa_full_config_sampled(dev, orc):
    """SDPA config: B8 H32 S2048 D128, non-causal, Q/K/V ~ N(0,1): sampled
    rows of several heads against float64."""
    bh, s, d = 256, 2048, 128
    r = np.random.default_rng(1236)
    q, k, v = (r.standard_normal(bh * s * d, dtype=np.float32) for _ in range(3))
    out = dev.read(dev.scaled_dot_product_attention(dev.upload(q), dev.upload(k), dev.upload(v),
                                                    bh, s, d)).reshape(bh, s, d)
    rows = [0, 1, 127, 128, 1000, 2047]
    for h in (0, 77, 255):
        sl = slice(h * s * d, (h + 1) * s * d)
        ref = _attn64(q[sl], k[sl], v[sl], 1, s, d, rows=rows)[0]
        assert orc.rel_fro(out[h, rows], ref) <= 1e-3


def test_sdpa_errors(dev):
    from any_gpu import AnyGpuError
    a = dev.upload(np.ones(12, np.float32))
    b = dev.upload(np.ones(10, np.float32))
    with pytest.raises(AnyGpuError) as e:
        dev.scaled_dot_product_attention(a, a, b, 1, 3, 4)
    assert e.value.status == 1


# ----------------------------------------------------------------- tape ops --
@pytest.mark.parametrize("outer,ai,bi", [(2, 2, 4), (16, 320 * 64, 320 * 64), (7, 5, 3),
                                         (3, 1, 1), (1000, 12, 8)])
def test_concat_slice_parity(dev, orc, outer, ai, bi):
    """concat (src/ops/tensor_ops.rs:229) and its backward slice_per_block
    (:274): copies, bit-exact, float4 and scalar paths."""
    r = np.random.default_rng(outer + ai)
    a = r.standard_normal(outer * ai).astype(np.float32)
    b = r.standard_normal(outer * bi).astype(np.float32)
    got = dev.concat(dev.upload(a), dev.upload(b), outer, ai, bi)
    np.testing.assert_array_equal(dev.read(got), orc.concat(a, b, outer, ai, bi))
    np.testing.assert_array_equal(dev.read(dev.slice_per_block(got, outer, ai, 0, ai + bi)), a)
    np.testing.assert_array_equal(dev.read(dev.slice_per_block(got, outer, bi, ai, ai + bi)), b)


@pytest.mark.parametrize("n,c,h,w,sh,sw", [(1, 1, 2, 2, 2, 2), (2, 3, 5, 7, 3, 2),
                                           (16, 320, 32, 32, 2, 2), (1, 1, 1, 1, 3, 3)])
def test_upsample_parity(dev, orc, n, c, h, w, sh, sw):
    """upsample_nearest2d and its backward (src/ops/upsample.rs:94-137):
    the forward is a gather, the backward sums each window in the shader's
    order, so both are bit-exact."""
    r = np.random.default_rng(n * c + h)
    x = r.standard_normal(n * c * h * w).astype(np.float32)
    got = dev.read(dev.upsample_nearest2d(dev.upload(x), n, c, h, w, sh, sw))
    np.testing.assert_array_equal(got, orc.upsample_nearest2d(x, n, c, h, w, sh, sw))
    go = r.standard_normal(got.size).astype(np.float32)
    gi = dev.read(dev.upsample_nearest2d_backward(dev.upload(go), n, c, h, w, sh, sw))
    np.testing.assert_array_equal(gi, orc.upsample_nearest2d_backward(go, n, c, h, w, sh, sw))


@pytest.mark.parametrize("outer,inner", [(1, 1), (3, 5), (320, 65536), (65536, 64),
                                         (2, 1000003), (7, 2049)])
def test_broadcast_add_and_sum_inner_parity(dev, orc, outer, inner):
    """add_broadcast (bit-exact) and sum_inner, its bias gradient, against the
    oracle's serial sums: within 1e-5 of float64 or as close as the oracle."""
    r = np.random.default_rng(outer + inner)
    a = r.standard_normal(outer * inner).astype(np.float32)
    b = r.standard_normal(outer).astype(np.float32)
    A = dev.upload(a)
    np.testing.assert_array_equal(dev.read(dev.add_broadcast(A, dev.upload(b), outer, inner)),
                                  orc.add_broadcast(a, b, outer, inner))
    got = dev.read(dev.sum_inner(A, outer, inner))
    want = orc.sum_inner(a, outer, inner)
    ref = a.reshape(outer, inner).astype(np.float64).sum(1)
    assert orc.rel_fro(got, ref) <= max(1e-5, orc.rel_fro(want, ref))


@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 3), (65536, 64), (300, 11008), (100003, 5),
                                       (2, 70000)])
def test_sum_rows_parity(dev, orc, rows, cols):
    """sum_rows (src/ops/tensor_ops.rs:356), the add_per_col bias gradient."""
    r = np.random.default_rng(rows + cols)
    a = r.standard_normal(rows * cols).astype(np.float32)
    got = dev.read(dev.sum_rows(dev.upload(a), rows, cols))
    want = orc.sum_rows(a, rows, cols)
    ref = a.reshape(rows, cols).astype(np.float64).sum(0)
    assert orc.rel_fro(got, ref) <= max(1e-5, orc.rel_fro(want, ref))


@pytest.mark.parametrize("n", [1, 3, 4097, 1 << 22, 10000019])
def test_mse_loss_parity(dev, orc, n):
    """mse_loss (src/ops/attention.rs:172): a deterministic tree sum against
    the shader's serial fp32 sum."""
    r = np.random.default_rng(n)
    p = r.standard_normal(n).astype(np.float32)
    t = r.standard_normal(n).astype(np.float32)
    P, T = dev.upload(p), dev.upload(t)
    got = dev.read(dev.mse_loss(P, T))
    d = p.astype(np.float64) - t
    ref = (d * d).mean()
    want = orc.mse_loss(p, t)[0]
    assert abs(got[0] - ref) / ref <= max(1e-6, abs(want - ref) / ref)
    assert got[0] == dev.read(dev.mse_loss(P, T))[0]  # deterministic


def test_tape_ops_errors(dev):
    from any_gpu import AnyGpuError
    up = lambda k: dev.upload(np.ones(k, np.float32))
    calls = [lambda: dev.concat(up(5), up(4), 1, 4, 4),            # a size
             lambda: dev.concat(up(4), up(5), 1, 4, 4),            # b size
             lambda: dev.slice_per_block(up(8), 2, 3, 2, 4),       # offset + size > combined
             lambda: dev.slice_per_block(up(9), 2, 2, 0, 4),       # src size
             lambda: dev.add_broadcast(up(6), up(2), 3, 2),        # b size
             lambda: dev.sum_inner(up(5), 2, 2),
             lambda: dev.sum_rows(up(5), 2, 2),
             lambda: dev.upsample_nearest2d(up(5), 1, 1, 2, 2, 2, 2),
             lambda: dev.upsample_nearest2d_backward(up(5), 1, 1, 1, 1, 2, 2),
             lambda: dev.mse_loss(up(3), up(4))]
    for c in calls:
        with pytest.raises(AnyGpuError) as e:
            c()
        assert e.value.status == 1


def test_async_partial_copies(dev):
    """agpu_write_async / agpu_read_async: element ranges of a buffer on a
    caller's stream, bounds checked like the synchronous calls."""
    import torch
    from any_gpu import AnyGpuError
    n = 1 << 20
    host = torch.arange(n, dtype=torch.float32).pin_memory()
    out = torch.zeros(n, dtype=torch.float32).pin_memory()
    buf = dev.alloc(n)
    dev.synchronize()
    s = torch.cuda.Stream()
    half = n // 2
    dev.write_async(buf, host.data_ptr() + 4 * half, half, half, s.cuda_stream)  # upper half
    dev.write_async(buf, host.data_ptr(), half, 0, s.cuda_stream)                # lower half
    dev.read_async(buf, out.data_ptr() + 4 * 7, n - 7, 7, s.cuda_stream)
    s.synchronize()
    np.testing.assert_array_equal(out.numpy()[7:], host.numpy()[7:])
    assert not out.numpy()[:7].any()
    np.testing.assert_array_equal(dev.read(buf), host.numpy())
    for call in (lambda: dev.write_async(buf, host.data_ptr(), 2, n - 1, s.cuda_stream),
                 lambda: dev.read_async(buf, out.data_ptr(), 1, n, s.cuda_stream)):
        with pytest.raises(AnyGpuError) as e:
            call()
        assert e.value.status == 1


def test_tape_ops_empty_and_degenerate(dev):
    """Zero-size inputs: empty outputs, zero sums, and the shader's 0/0 = NaN
    for the mean of an empty mse."""
    up = lambda k: dev.upload(np.ones(k, np.float32))
    assert dev.concat(up(0), up(0), 0, 3, 4).len == 0
    assert dev.slice_per_block(up(0), 0, 2, 1, 4).len == 0
    np.testing.assert_array_equal(dev.read(dev.sum_rows(up(0), 0, 5)), np.zeros(5, np.float32))
    np.testing.assert_array_equal(dev.read(dev.sum_inner(up(0), 4, 0)), np.zeros(4, np.float32))
    assert dev.upsample_nearest2d(up(0), 0, 3, 4, 4, 2, 2).len == 0
    assert np.isnan(dev.read(dev.mse_loss(up(0), up(0)))[0])


@pytest.mark.parametrize("n,cin,h,w,cout,g", [(16, 320, 64, 64, 320, 32), (5, 64, 20, 24, 320, 32),
                                              (1, 32, 16, 16, 64, 8), (2, 3, 17, 19, 64, 4)])
def test_conv2d_group_norm_swish_fused(dev, n, cin, h, w, cout, g):
    """The fused UNet block equals conv2d followed by group_norm_swish, bit for
    bit (the same kernels, the group norm per half of the batch)."""
    r = np.random.default_rng(n + cin + cout)
    x = r.standard_normal(n * cin * h * w).astype(np.float32)
    bound = np.sqrt(6.0 / (cin * 9))
    wt = r.uniform(-bound, bound, cout * cin * 9).astype(np.float32)
    bias = (0.1 * r.standard_normal(cout)).astype(np.float32)
    gamma = (1 + 0.1 * r.standard_normal(cout)).astype(np.float32)
    beta = (0.1 * r.standard_normal(cout)).astype(np.float32)
    X, W, B, G, Bt = (dev.upload(v) for v in (x, wt, bias, gamma, beta))
    got = dev.read(dev.conv2d_group_norm_swish(X, W, B, n, cin, h, w, cout, 3, 3, (1, 1), (1, 1),
                                               gamma=G, beta=Bt, gn_groups=g, eps=1e-5))
    y = dev.conv2d(X, W, B, n, cin, h, w, cout, 3, 3, (1, 1), (1, 1))
    want = dev.read(dev.group_norm_swish(y, G, Bt, n, cout, h * w, g, 1e-5))
    np.testing.assert_array_equal(got, want)
    from any_gpu import AnyGpuError
    with pytest.raises(AnyGpuError) as e:
        dev.conv2d_group_norm_swish(X, W, B, n, cin, h, w, cout, 3, 3, (1, 1), (1, 1), gamma=G,
                                    beta=Bt, gn_groups=cout + 1)
    assert e.value.status == 1
