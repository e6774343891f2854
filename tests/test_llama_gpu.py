"""GPU: the ops of the LLaMA-style decoder layer (RMSNorm, RoPE, SwiGLU product,
GEMM with fused bias/residual/activation, strided SDPA) and the composed
layer, against the oracle.  RMSNorm and RoPE have no reference code, so their
parity is unpinned: the oracle is the standard formula (checked against float64
here too)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32 = 4


@pytest.mark.parametrize("rows,cols", [(64, 4096), (7, 1000), (5, 37), (3, 10000)])
def test_rmsnorm_parity(dev, orc, rows, cols):
    r = np.random.default_rng(rows + cols)
    x = r.standard_normal(rows * cols).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(cols)).astype(np.float32)
    got = dev.read(dev.rmsnorm(dev.upload(x), dev.upload(w), rows, cols, 1e-5))
    want = orc.rmsnorm(x, w, rows, cols, 1e-5)
    X = x.reshape(rows, cols).astype(np.float64)
    ref = (X / np.sqrt((X * X).mean(1, keepdims=True) + 1e-5) * w).ravel()
    assert orc.rel_fro(got, ref) <= max(1e-5, orc.rel_fro(want, ref))
    assert orc.rel_fro(got, want) <= 1e-5


@pytest.mark.parametrize("b,s,h,d", [(2, 64, 4, 128), (1, 2048, 2, 128), (3, 5, 3, 6)])
def test_rope_parity(dev, orc, b, s, h, d):
    r = np.random.default_rng(b * s + d)
    x = r.standard_normal(b * s * h * d).astype(np.float32)
    got = dev.read(dev.rope(dev.upload(x), b, s, h, d, 10000.0))
    want = orc.rope(x, b, s, h, d, 10000.0)
    assert orc.rel_fro(got, want) <= 1e-6


def test_swish_mul_parity(dev, orc):
    r = np.random.default_rng(4)
    for n in (1, 7, 1 << 20):
        g = (r.standard_normal(n) * 3).astype(np.float32)
        u = r.standard_normal(n).astype(np.float32)
        got = dev.read(dev.swish_mul(dev.upload(g), dev.upload(u)))
        want = orc.elementwise("mul", orc.elementwise("swish", g), u)
        np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("prec,tol", [("tf32", 1e-3), ("tf32x3", 1e-5), ("ffma", 1e-5)])
@pytest.mark.parametrize("act", [0, 1, 2])
def test_gemm_fused_epilogue(dev, orc, prec, tol, act):
    """C = act(A B + bias + resid): the Linear bias (add_per_col), a residual
    add and swish / relu fused into the GEMM's epilogue."""
    m, n, k = 300, 264, 520
    r = np.random.default_rng(act)
    a = r.uniform(-1, 1, m * k).astype(np.float32)
    b = r.uniform(-1, 1, k * n).astype(np.float32)
    bias = r.standard_normal(n).astype(np.float32)
    res = r.standard_normal(m * n).astype(np.float32)
    dev.set_precision(prec)
    try:
        got = dev.read(dev.gemm_ex(dev.upload(a), dev.upload(b), 1, m, n, k,
                                   bias=dev.upload(bias), resid=dev.upload(res), act=act))
    finally:
        dev.set_precision("tf32")
    want = orc.elementwise("add", orc.add_per_col(orc.matmul(a, b, m, n, k, threads=True),
                                                  bias, m, n), res)
    if act == 1:
        want = orc.elementwise("swish", want)
    elif act == 2:
        want = orc.elementwise("relu", want)
    assert orc.rel_fro(got, want) <= tol


def _swiglu_blocks(c, m, n):
    """swish(gate) * up over 32-column block pairs: gate j = [64j, 64j+32),
    up j = [64j+32, 64j+64) -> [m, n/2]."""
    blk = np.asarray(c, np.float64).reshape(m, n // 64, 2, 32)
    g, u = blk[:, :, 0], blk[:, :, 1]
    return (g / (1 + np.exp(-g)) * u).reshape(-1)


@pytest.mark.parametrize("prec,tol", [("tf32", 1e-3), ("tf32x3", 1e-5), ("ffma", 1e-5)])
@pytest.mark.parametrize("batch,m,n,k", [(1, 2048, 2048, 256),   # fused in the pair kernel
                                         (1, 1024, 5120, 384),   # fused, 256x512 tiles
                                         (2, 300, 640, 96),      # GEMM, then swish * up
                                         (1, 64, 128, 40)])      # small: SIMT, then swish * up
def test_gemm_swiglu_epilogue(dev, orc, prec, tol, batch, m, n, k):
    """act 3 (SwiGLU): the LLaMA gate/up projection writes swish(gate) * up
    directly, from B's interleaved 32-column gate / up blocks."""
    r = np.random.default_rng(m + n)
    a = (r.standard_normal(batch * m * k) * 0.5).astype(np.float32)
    b = (r.standard_normal(batch * k * n) * 0.1).astype(np.float32)
    dev.set_precision(prec)
    try:
        got = dev.read(dev.gemm_ex(dev.upload(a), dev.upload(b), batch, m, n, k, act=3))
    finally:
        dev.set_precision("tf32")
    assert got.size == batch * m * n // 2
    prods = [orc.matmul(a[i * m * k:(i + 1) * m * k], b[i * k * n:(i + 1) * k * n], m, n, k,
                        threads=True) for i in range(batch)]
    want = np.concatenate([_swiglu_blocks(c, m, n) for c in prods])
    assert orc.rel_fro(got, want) <= tol


def test_gemm_swiglu_errors(dev):
    from any_gpu import AnyGpuError
    up = lambda k: dev.upload(np.ones(k, np.float32))
    for call in (lambda: dev.gemm_ex(up(4 * 8), up(8 * 96), 1, 4, 96, 8, act=3),  # n % 64
                 lambda: dev.gemm_ex(up(4 * 8), up(8 * 64), 1, 4, 64, 8, bias=up(64), act=3)):
        with pytest.raises(AnyGpuError) as e:
            call()
        assert e.value.status == 1


def test_sdpa_strided_packed_qkv(dev, orc):
    """Q, K, V read in place from a packed [B, S, 3, H, D] projection, output
    written as [B, S, H, D] (the layer's layout) -- tensor-core and SIMT paths."""
    for (B, S, H, D) in [(2, 200, 3, 128), (2, 300, 2, 128), (1, 70, 2, 64), (2, 9, 2, 16)]:
        r = np.random.default_rng(S)
        qkv = r.standard_normal(B * S * 3 * H * D).astype(np.float32)
        Q = dev.upload(qkv)
        O = dev.alloc(B * S * H * D)
        st = (3 * H * D, D, S * 3 * H * D)
        p = Q.device_ptr
        dev.launch_sdpa_strided(p, p + H * D * F32, p + 2 * H * D * F32, O.device_ptr, B, H, S,
                                D, st, st, st, (H * D, D, S * H * D))
        got = dev.read(O).reshape(B, S, H, D).transpose(0, 2, 1, 3)
        P = qkv.reshape(B, S, 3, H, D)
        heads = [np.ascontiguousarray(P[:, :, i].transpose(0, 2, 1, 3)).ravel() for i in range(3)]
        want = orc.attention(*heads, B * H, S, D, threads=True).reshape(B, H, S, D)
        assert orc.rel_fro(got, want) <= 1e-3


def _layer_oracle(orc, x, w, dims):
    """The layer restated with the oracle's functions (fp32)."""
    B, S, d, H, Fd = dims.batch, dims.seq, dims.d_model, dims.heads, dims.ffn
    T, Dh = B * S, d // H
    h1 = orc.rmsnorm(x, w["attn_norm"], T, d, dims.eps)
    qkv = orc.matmul(h1, w["wqkv"], T, 3 * d, d, threads=True).reshape(B, S, 3, H, Dh)
    q = orc.rope(np.ascontiguousarray(qkv[:, :, 0]), B, S, H, Dh, dims.rope_base)
    k = orc.rope(np.ascontiguousarray(qkv[:, :, 1]), B, S, H, Dh, dims.rope_base)
    v = np.ascontiguousarray(qkv[:, :, 2])
    tr = lambda t: np.ascontiguousarray(t.reshape(B, S, H, Dh).transpose(0, 2, 1, 3)).ravel()
    o = orc.attention(tr(q), tr(k), tr(v), B * H, S, Dh, threads=not dims.causal,
                      causal=dims.causal)
    o = np.ascontiguousarray(o.reshape(B, H, S, Dh).transpose(0, 2, 1, 3)).ravel()
    x2 = orc.elementwise("add", x, orc.matmul(o, w["wo"], T, d, d, threads=True))
    h2 = orc.rmsnorm(x2, w["ffn_norm"], T, d, dims.eps)
    gu = orc.matmul(h2, w["wgu"], T, 2 * Fd, d, threads=True).reshape(T, 2 * Fd)
    if dims.fused_swiglu:  # Wgu in interleaved 32-column gate / up blocks
        a = _swiglu_blocks(gu, T, 2 * Fd).astype(np.float32)
    else:
        a = orc.elementwise("mul", orc.elementwise("swish", np.ascontiguousarray(gu[:, :Fd])),
                            np.ascontiguousarray(gu[:, Fd:]))
    return orc.elementwise("add", x2, orc.matmul(a, w["wd"], T, d, Fd, threads=True))


@pytest.mark.parametrize("ffn", [344, 352])  # [Wg | Wu] halves; interleaved blocks, fused
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("prec,tol", [("tf32", 2e-3), ("tf32x3", 1e-5)])
def test_llama_layer_small(dev, orc, prec, tol, causal, ffn):
    """The LLaMA-style layer of the benchmark configs at a small size (B2, S128,
    d256, H2 x 128, FFN 344; weights N(0, 0.02), x N(0,1)) against the layer
    restated with the oracle.  TF32: the layer chains five TF32 contractions,
    so its bound is 2e-3; 3xTF32 (attention on the exact kernel) stays at 1e-5."""
    from any_gpu.llama import LlamaDims, layer_forward
    dims = LlamaDims(batch=2, seq=128, d_model=256, heads=2, ffn=ffn, causal=causal)
    d, Fd, T = dims.d_model, dims.ffn, dims.tokens
    r = np.random.default_rng(1238)
    w = {"attn_norm": (1 + 0.1 * r.standard_normal(d)).astype(np.float32),
         "ffn_norm": (1 + 0.1 * r.standard_normal(d)).astype(np.float32),
         "wqkv": (r.standard_normal(d * 3 * d) * 0.02).astype(np.float32),
         "wo": (r.standard_normal(d * d) * 0.02).astype(np.float32),
         "wgu": (r.standard_normal(d * 2 * Fd) * 0.02).astype(np.float32),
         "wd": (r.standard_normal(Fd * d) * 0.02).astype(np.float32)}
    x = r.standard_normal(T * d).astype(np.float32)
    bufs = {k: dev.upload(v) for k, v in w.items()}
    X, Y = dev.upload(x), dev.alloc(T * d)
    ws = {k: dev.alloc(n) for k, n in dims.workspace_elems().items()}
    dev.set_precision(prec)
    try:
        layer_forward(dev, dims, X.device_ptr, {k: b.device_ptr for k, b in bufs.items()},
                      {k: b.device_ptr for k, b in ws.items()}, Y.device_ptr)
        got = dev.read(Y)
    finally:
        dev.set_precision("tf32")
    want = _layer_oracle(orc, x, w, dims)
    assert orc.rel_fro(got, want) <= tol


def test_llama_layer_benchmark_size_sampled(dev, orc):
    """The decoder layer at its benchmark size (B32 S2048 d4096 H32x128 FFN
    11008, weights N(0, 0.02), x N(0, 1)): the last sequence of the batch-32
    output against the layer in float64 (products and attention in float64;
    RMSNorm and RoPE from the oracle), and the first sequence against a
    batch-1 run of the same sequence (the batch split must not change it)."""
    from any_gpu.llama import LlamaDims, layer_forward
    full = LlamaDims(batch=32, seq=2048, d_model=4096, heads=32, ffn=11008)
    d, Fd, S, H = full.d_model, full.ffn, full.seq, full.heads
    Dh = d // H
    r = np.random.default_rng(1239)
    w = {"attn_norm": np.ones(d, np.float32), "ffn_norm": np.ones(d, np.float32)}
    for k, n in (("wqkv", d * 3 * d), ("wo", d * d), ("wgu", d * 2 * Fd), ("wd", Fd * d)):
        w[k] = (r.standard_normal(n, dtype=np.float32) * np.float32(0.02))
    x = r.standard_normal(full.tokens * d, dtype=np.float32)
    bufs = {k: dev.upload(v) for k, v in w.items()}
    wp = {k: b.device_ptr for k, b in bufs.items()}

    def run(dims, xs):
        X, Y = dev.upload(xs), dev.alloc(dims.tokens * d)
        ws = {k: dev.alloc(n) for k, n in dims.workspace_elems().items()}
        layer_forward(dev, dims, X.device_ptr, wp, {k: b.device_ptr for k, b in ws.items()},
                      Y.device_ptr)
        return dev.read(Y)

    got = run(full, x).reshape(full.batch, S * d)
    one = LlamaDims(batch=1, seq=S, d_model=d, heads=H, ffn=Fd)
    assert orc.rel_fro(got[0], run(one, x[:S * d])) <= 1e-6

    # float64 layer of the last sequence
    xs = x[-S * d:]
    f64 = lambda a: np.asarray(a, np.float64)
    h1 = orc.rmsnorm(xs, w["attn_norm"], S, d, full.eps)
    qkv = (f64(h1).reshape(S, d) @ f64(w["wqkv"]).reshape(d, 3 * d)).reshape(S, 3, H, Dh)
    q = f64(orc.rope(np.ascontiguousarray(qkv[:, 0], np.float32), 1, S, H, Dh, full.rope_base))
    k = f64(orc.rope(np.ascontiguousarray(qkv[:, 1], np.float32), 1, S, H, Dh, full.rope_base))
    v = qkv[:, 2]
    q, k = q.reshape(S, H, Dh).transpose(1, 0, 2), k.reshape(S, H, Dh).transpose(1, 0, 2)
    sc = q @ k.transpose(0, 2, 1) / np.sqrt(Dh)
    p = np.exp(sc - sc.max(axis=2, keepdims=True))
    p /= p.sum(axis=2, keepdims=True)
    o = (p @ v.transpose(1, 0, 2)).transpose(1, 0, 2).reshape(S, d)
    x2 = f64(xs).reshape(S, d) + o @ f64(w["wo"]).reshape(d, d)
    h2 = f64(orc.rmsnorm(x2.astype(np.float32).ravel(), w["ffn_norm"], S, d, full.eps))
    gu = h2.reshape(S, d) @ f64(w["wgu"]).reshape(d, 2 * Fd)
    a = _swiglu_blocks(gu, S, 2 * Fd)  # interleaved 32-column gate / up blocks
    want = x2 + a.reshape(S, Fd) @ f64(w["wd"]).reshape(Fd, d)
    assert orc.rel_fro(got[-1], want.ravel()) <= 2e-3
