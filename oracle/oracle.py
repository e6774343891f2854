"""TEST INFRASTRUCTURE ONLY: numpy front-end of the C oracle (oracle.c).

The oracle restates the reference's own CPU implementations (Rust crate
any-gpu; file:line per function in oracle.c).  tests/ use it as the parity
checker; bench.py's cpu_baseline and `--impl reference` legs time it.  The
product (libagpu.so and the any_gpu package) never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_i64, _f32 = C.c_int64, C.c_float
_p = C.c_void_p
_SIG = {
    "oracle_num_threads": (C.c_int, []),
    "oracle_matmul": (None, [_p, _p, _p, _i64, _i64, _i64]),
    "oracle_matmul_mt": (None, [_p, _p, _p, _i64, _i64, _i64]),
    "oracle_batch_matmul": (None, [_p, _p, _p, _i64, _i64, _i64, _i64]),
    "oracle_batch_matmul_mt": (None, [_p, _p, _p, _i64, _i64, _i64, _i64]),
    "oracle_softmax": (None, [_p, _p, _i64, _i64]),
    "oracle_softmax_mt": (None, [_p, _p, _i64, _i64]),
    "oracle_attention": (None, [_p, _p, _p, _p, _i64, _i64, _i64]),
    "oracle_attention_mt": (None, [_p, _p, _p, _p, _i64, _i64, _i64]),
    "oracle_attention_causal": (None, [_p, _p, _p, _p, _i64, _i64, _i64]),
    "oracle_conv_out": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "oracle_conv2d": (None, [_p, _p, _p, _p] + [_i64] * 14),
    "oracle_conv2d_mt": (None, [_p, _p, _p, _p] + [_i64] * 14),
    "oracle_conv_transpose2d": (None, [_p, _p, _p, _p] + [_i64] * 16),
    "oracle_conv2d_grad_weight": (None, [_p, _p, _p] + [_i64] * 16),
    "oracle_conv2d_grad_bias": (None, [_p, _p, _i64, _i64, _i64, _i64]),
    "oracle_group_norm": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _f32]),
    "oracle_group_norm_mt": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _f32]),
    "oracle_group_norm_backward": (None, [_p] * 6 + [_i64, _i64, _i64, _i64, _f32]),
    "oracle_sigmoid1": (_f32, [_f32]),
    "oracle_swish1": (_f32, [_f32]),
    "oracle_elementwise": (None, [C.c_int, _p, _p, _f32, _p, _i64]),
    "oracle_transpose": (None, [_p, _p, _i64, _i64, _i64, _i64]),
    "oracle_add_per_col": (None, [_p, _p, _p, _i64, _i64]),
    "oracle_add_broadcast": (None, [_p, _p, _p, _i64, _i64]),
    "oracle_sum_inner": (None, [_p, _p, _i64, _i64]),
    "oracle_sum_rows": (None, [_p, _p, _i64, _i64]),
    "oracle_concat": (None, [_p, _p, _p, _i64, _i64, _i64]),
    "oracle_slice_per_block": (None, [_p, _p, _i64, _i64, _i64, _i64]),
    "oracle_upsample_nearest2d": (None, [_p, _p] + [_i64] * 6),
    "oracle_upsample_nearest2d_backward": (None, [_p, _p] + [_i64] * 6),
    "oracle_mse_loss": (_f32, [_p, _p, _i64]),
    "oracle_rmsnorm": (None, [_p, _p, _p, _i64, _i64, _f32]),
    "oracle_rope": (None, [_p, _p, _i64, _i64, _i64, _i64, _f32]),
    "oracle_adamw": (None, [_p, _p, _p, _p, _i64, _f32, _f32, _f32, _f32, _f32, _i64]),
}

ELEMENTWISE = {"add": 0, "sub": 1, "mul": 2, "relu": 3, "sigmoid": 4, "swish": 5, "tanh": 6,
               "scale": 7, "relu_backward": 8, "sigmoid_backward": 9, "swish_backward": 10,
               "tanh_backward": 11}

_lib = None


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, no GPU)."""
    src = HERE / "oracle.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        l = C.CDLL(os.fspath(LIB))
        for name, (res, args) in _SIG.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _a(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(x: np.ndarray):
    return x.ctypes.data_as(C.c_void_p)


def num_threads() -> int:
    return lib().oracle_num_threads()


def matmul(a, b, m, n, k, threads: bool = False) -> np.ndarray:
    a, b = _a(a), _a(b)
    out = np.empty(m * n, np.float32)
    (lib().oracle_matmul_mt if threads else lib().oracle_matmul)(_ptr(a), _ptr(b), _ptr(out),
                                                                  m, n, k)
    return out


def batch_matmul(a, b, batch, m, n, k, threads: bool = False) -> np.ndarray:
    a, b = _a(a), _a(b)
    out = np.empty(batch * m * n, np.float32)
    fn = lib().oracle_batch_matmul_mt if threads else lib().oracle_batch_matmul
    fn(_ptr(a), _ptr(b), _ptr(out), batch, m, n, k)
    return out


def softmax(x, rows, cols, threads: bool = False) -> np.ndarray:
    x = _a(x)
    out = np.empty(rows * cols, np.float32)
    (lib().oracle_softmax_mt if threads else lib().oracle_softmax)(_ptr(x), _ptr(out), rows, cols)
    return out


def attention(q, k, v, bh, seq, dk, threads: bool = False, causal: bool = False) -> np.ndarray:
    q, k, v = _a(q), _a(k), _a(v)
    out = np.empty(bh * seq * dk, np.float32)
    if causal:
        fn = lib().oracle_attention_causal
    else:
        fn = lib().oracle_attention_mt if threads else lib().oracle_attention
    fn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), bh, seq, dk)
    return out


def attention_backward(q, k, v, dout, bh, seq, dk, causal: bool = False):
    """dQ, dK, dV of attention: the reference's SDPA composition
    (src/ops/attention.rs:149-169: kt = transpose(K); scores = batch_matmul(Q,
    kt); scaled = scale(scores, 1/sqrt(dk)); attn = softmax(scaled); out =
    batch_matmul(attn, V)) differentiated in reverse with its own rules: the
    matmul rule of src/autograd.rs:357-366 (dA = dC B^T, dB = A^T dC, through
    transposes), the scale rule (:317-320) and the softmax Jacobian-vector
    product dx = y * (dy - sum(y * dy)) per row (the reference's tape has no
    softmax node; this is the derivative of cpu_softmax).  Per head, with
    cpu_matmul / cpu_softmax / transpose from the C restatement; the causal
    variant masks scaled scores above the diagonal to -inf before softmax."""
    q, k, v, dout = _a(q), _a(k), _a(v), _a(dout)
    c = np.float32(1.0 / np.sqrt(np.float32(dk)))
    hs = seq * dk
    dq, dkk, dv = (np.empty(bh * hs, np.float32) for _ in range(3))
    for h in range(bh):
        sl = slice(h * hs, (h + 1) * hs)
        qh, kh, vh, doh = q[sl], k[sl], v[sl], dout[sl]
        kt = transpose(kh, 1, seq, dk, 1)                       # [dk, seq]
        scores = matmul(qh, kt, seq, seq, dk)
        scaled = elementwise("scale", scores, None, float(c))
        if causal:
            sc = scaled.reshape(seq, seq)
            sc[np.triu_indices(seq, 1)] = -np.inf
        attn = softmax(scaled, seq, seq)
        # out = attn @ V
        vt = transpose(vh, 1, seq, dk, 1)
        d_attn = matmul(doh, vt, seq, seq, dk)                  # dO V^T
        at = transpose(attn, 1, seq, seq, 1)
        dv[sl] = matmul(at, doh, seq, dk, seq)                  # attn^T dO
        # attn = softmax(scaled)
        y, dy = attn.reshape(seq, seq), d_attn.reshape(seq, seq)
        rows = np.sum(y * dy, axis=1, dtype=np.float32, keepdims=True)
        d_scaled = (y * (dy - rows)).astype(np.float32).reshape(-1)
        d_scores = elementwise("scale", d_scaled, None, float(c))
        # scores = Q @ kt
        ktt = transpose(kt, 1, dk, seq, 1)                      # kt^T = K
        dq[sl] = matmul(d_scores, ktt, seq, dk, seq)
        qt = transpose(qh, 1, seq, dk, 1)
        d_kt = matmul(qt, d_scores, dk, seq, seq)               # Q^T dS  [dk, seq]
        dkk[sl] = transpose(d_kt, 1, dk, seq, 1)                # back through transpose(K)
    return dq, dkk, dv


def conv_out(n, k, stride, pad, dil) -> int:
    return int(lib().oracle_conv_out(n, k, stride, pad, dil))


def conv2d(inp, w, bias, batch, in_c, in_h, in_w, out_c, kh, kw, stride=(1, 1), padding=(0, 0),
           dilation=(1, 1), groups=1, threads: bool = False) -> np.ndarray:
    inp, w = _a(inp), _a(w)
    b = _a(bias) if bias is not None else None
    oh = conv_out(in_h, kh, stride[0], padding[0], dilation[0])
    ow = conv_out(in_w, kw, stride[1], padding[1], dilation[1])
    out = np.empty(batch * out_c * oh * ow, np.float32)
    fn = lib().oracle_conv2d_mt if threads else lib().oracle_conv2d
    fn(_ptr(inp), _ptr(w), _ptr(b) if b is not None else None, _ptr(out), batch, in_c, in_h, in_w,
       out_c, kh, kw, stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1],
       groups)
    return out


def conv_transpose2d(inp, w, bias, batch, in_c, in_h, in_w, out_c, kh, kw, stride=(1, 1),
                     padding=(0, 0), output_padding=(0, 0), dilation=(1, 1), groups=1):
    inp, w = _a(inp), _a(w)
    b = _a(bias) if bias is not None else None
    oh = (in_h - 1) * stride[0] - 2 * padding[0] + dilation[0] * (kh - 1) + output_padding[0] + 1
    ow = (in_w - 1) * stride[1] - 2 * padding[1] + dilation[1] * (kw - 1) + output_padding[1] + 1
    out = np.empty(batch * out_c * oh * ow, np.float32)
    lib().oracle_conv_transpose2d(_ptr(inp), _ptr(w), _ptr(b) if b is not None else None,
                                  _ptr(out), batch, in_c, in_h, in_w, out_c, kh, kw, stride[0],
                                  stride[1], padding[0], padding[1], output_padding[0],
                                  output_padding[1], dilation[0], dilation[1], groups)
    return out


def conv2d_grad_weight(inp, grad_out, batch, in_c, in_h, in_w, out_c, out_h, out_w, kh, kw,
                       sh, sw, ph, pw, dh, dw, groups):
    inp, go = _a(inp), _a(grad_out)
    out = np.empty(out_c * (in_c // groups) * kh * kw, np.float32)
    lib().oracle_conv2d_grad_weight(_ptr(inp), _ptr(go), _ptr(out), batch, in_c, in_h, in_w,
                                    out_c, out_h, out_w, kh, kw, sh, sw, ph, pw, dh, dw, groups)
    return out


def conv2d_grad_bias(grad_out, batch, out_c, out_h, out_w):
    go = _a(grad_out)
    out = np.empty(out_c, np.float32)
    lib().oracle_conv2d_grad_bias(_ptr(go), _ptr(out), batch, out_c, out_h, out_w)
    return out


def group_norm(x, gamma, beta, batch, channels, spatial, groups, eps,
               threads: bool = False) -> np.ndarray:
    x, g, b = _a(x), _a(gamma), _a(beta)
    out = np.empty(x.size, np.float32)
    fn = lib().oracle_group_norm_mt if threads else lib().oracle_group_norm
    fn(_ptr(x), _ptr(g), _ptr(b), _ptr(out), batch, channels, spatial, groups, eps)
    return out


def group_norm_backward(grad_out, x, gamma, batch, channels, spatial, groups, eps):
    go, x, g = _a(grad_out), _a(x), _a(gamma)
    di = np.empty(x.size, np.float32)
    dg = np.empty(channels, np.float32)
    db = np.empty(channels, np.float32)
    lib().oracle_group_norm_backward(_ptr(go), _ptr(x), _ptr(g), _ptr(di), _ptr(dg), _ptr(db),
                                     batch, channels, spatial, groups, eps)
    return di, dg, db


def elementwise(op: str, a, b=None, s: float = 0.0) -> np.ndarray:
    a = _a(a)
    bb = _a(b) if b is not None else a
    out = np.empty(a.size, np.float32)
    lib().oracle_elementwise(ELEMENTWISE[op], _ptr(a), _ptr(bb), s, _ptr(out), a.size)
    return out


def sigmoid1(x: float) -> float:
    return float(lib().oracle_sigmoid1(x))


def swish1(x: float) -> float:
    return float(lib().oracle_swish1(x))


def transpose(a, outer, d0, d1, inner) -> np.ndarray:
    a = _a(a)
    out = np.empty(a.size, np.float32)
    lib().oracle_transpose(_ptr(a), _ptr(out), outer, d0, d1, inner)
    return out


def add_broadcast(a, b, outer, inner) -> np.ndarray:
    a, b = _a(a), _a(b)
    out = np.empty(a.size, np.float32)
    lib().oracle_add_broadcast(_ptr(a), _ptr(b), _ptr(out), outer, inner)
    return out


def sum_inner(src, outer, inner) -> np.ndarray:
    src = _a(src)
    out = np.empty(outer, np.float32)
    lib().oracle_sum_inner(_ptr(src), _ptr(out), outer, inner)
    return out


def sum_rows(src, rows, cols) -> np.ndarray:
    src = _a(src)
    out = np.empty(cols, np.float32)
    lib().oracle_sum_rows(_ptr(src), _ptr(out), rows, cols)
    return out


def concat(a, b, outer, a_inner, b_inner) -> np.ndarray:
    a, b = _a(a), _a(b)
    out = np.empty(outer * (a_inner + b_inner), np.float32)
    lib().oracle_concat(_ptr(a), _ptr(b), _ptr(out), outer, a_inner, b_inner)
    return out


def slice_per_block(src, outer, size, offset, combined) -> np.ndarray:
    src = _a(src)
    out = np.empty(outer * size, np.float32)
    lib().oracle_slice_per_block(_ptr(src), _ptr(out), outer, size, offset, combined)
    return out


def upsample_nearest2d(x, batch, channels, in_h, in_w, sh, sw) -> np.ndarray:
    x = _a(x)
    out = np.empty(batch * channels * in_h * sh * in_w * sw, np.float32)
    lib().oracle_upsample_nearest2d(_ptr(x), _ptr(out), batch, channels, in_h, in_w, sh, sw)
    return out


def upsample_nearest2d_backward(go, batch, channels, in_h, in_w, sh, sw) -> np.ndarray:
    go = _a(go)
    out = np.empty(batch * channels * in_h * in_w, np.float32)
    lib().oracle_upsample_nearest2d_backward(_ptr(go), _ptr(out), batch, channels, in_h, in_w,
                                             sh, sw)
    return out


def mse_loss(pred, target) -> np.ndarray:
    p, t = _a(pred), _a(target)
    return np.array([lib().oracle_mse_loss(_ptr(p), _ptr(t), p.size)], np.float32)


def add_per_col(a, b, rows, cols) -> np.ndarray:
    a, b = _a(a), _a(b)
    out = np.empty(a.size, np.float32)
    lib().oracle_add_per_col(_ptr(a), _ptr(b), _ptr(out), rows, cols)
    return out


def rmsnorm(x, w, rows, cols, eps) -> np.ndarray:
    x, w = _a(x), _a(w)
    out = np.empty(x.size, np.float32)
    lib().oracle_rmsnorm(_ptr(x), _ptr(w), _ptr(out), rows, cols, eps)
    return out


def rope(x, batch, seq, heads, dim, base=10000.0) -> np.ndarray:
    x = _a(x)
    out = np.empty(x.size, np.float32)
    lib().oracle_rope(_ptr(x), _ptr(out), batch, seq, heads, dim, base)
    return out


def rel_fro(got, want) -> float:
    """Relative Frobenius error ||got - want||_F / ||want||_F, in float64."""
    g = np.asarray(got, np.float64).reshape(-1)
    w = np.asarray(want, np.float64).reshape(-1)
    den = np.linalg.norm(w)
    return float(np.linalg.norm(g - w) / (den if den > 0 else 1.0))


def adamw(param, grad, m, v, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=1):
    """One AdamW step (updates copies; returns (param, m, v))."""
    p, g, mm, vv = (np.array(_a(t), copy=True) for t in (param, grad, m, v))
    lib().oracle_adamw(_ptr(p), _ptr(g), _ptr(mm), _ptr(vv), p.size, lr, beta1, beta2, eps,
                       weight_decay, step)
    return p, mm, vv
