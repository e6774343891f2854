"""A CPU stand-in for `any_gpu.GpuDevice` built on the oracle, for testing
host-side logic (the autograd tape's backward rules) without a GPU.

Test infrastructure only: every method computes with the oracle's C
restatement of the reference's CPU functions and shaders, and the buffers are
numpy arrays.  The product path never uses it.
"""
from __future__ import annotations

import numpy as np


class OracleBuffer:
    __slots__ = ("data", "len")

    def __init__(self, data):
        self.data = np.ascontiguousarray(np.asarray(data, np.float32).reshape(-1))
        self.len = self.data.size


class OracleDevice:
    def __init__(self, orc):
        self.o = orc

    def upload(self, data):
        return OracleBuffer(data)

    def read(self, buf):
        return buf.data.copy()

    # elementwise
    def _ew(self, op, a, b=None, s=0.0):
        if b is not None and a.len != b.len:
            from any_gpu import AnyGpuError
            raise AnyGpuError(1, f"{op}: length mismatch")
        return OracleBuffer(self.o.elementwise(op, a.data, None if b is None else b.data, s))

    def add(self, a, b): return self._ew("add", a, b)
    def sub(self, a, b): return self._ew("sub", a, b)
    def mul(self, a, b): return self._ew("mul", a, b)
    def scale(self, a, s): return self._ew("scale", a, None, s)
    def relu(self, a): return self._ew("relu", a)
    def sigmoid(self, a): return self._ew("sigmoid", a)
    def swish(self, a): return self._ew("swish", a)
    def tanh_act(self, a): return self._ew("tanh", a)
    def relu_backward(self, g, x): return self._ew("relu_backward", g, x)
    def sigmoid_backward(self, g, y): return self._ew("sigmoid_backward", g, y)
    def swish_backward(self, g, x): return self._ew("swish_backward", g, x)
    def tanh_backward(self, g, y): return self._ew("tanh_backward", g, y)

    # contractions
    def matmul(self, a, b, m, n, k):
        return OracleBuffer(self.o.matmul(a.data, b.data, m, n, k))

    def gemm(self, a, b, batch, m, n, k, trans_a=False, trans_b=False):
        assert batch == 1
        A = a.data.reshape(k, m).T if trans_a else a.data.reshape(m, k)
        B = b.data.reshape(n, k).T if trans_b else b.data.reshape(k, n)
        return OracleBuffer(self.o.matmul(np.ascontiguousarray(A), np.ascontiguousarray(B),
                                          m, n, k))

    def gemm_ex(self, a, b, batch, m, n, k, bias=None, resid=None, act=0, trans_a=False,
                trans_b=False):
        assert batch == 1 and resid is None and act in (0, 2)
        c = self.gemm(a, b, batch, m, n, k, trans_a, trans_b)
        if bias is not None:
            c = self.add_per_col(c, bias, m, n)
        return self.relu(c) if act == 2 else c

    def scaled_dot_product_attention(self, q, k, v, bh, s, d):
        return OracleBuffer(self.o.attention(q.data, k.data, v.data, bh, s, d))

    def sdpa_causal(self, q, k, v, bh, s, d):
        return OracleBuffer(self.o.attention(q.data, k.data, v.data, bh, s, d, causal=True))

    def sdpa_backward(self, q, k, v, go, bh, s, d, causal=False):
        return tuple(OracleBuffer(x) for x in self.o.attention_backward(
            q.data, k.data, v.data, go.data, bh, s, d, causal=causal))

    def mse_loss(self, p, t):
        return OracleBuffer(self.o.mse_loss(p.data, t.data))

    def conv2d(self, x, w, bias, batch, in_c, in_h, in_w, out_c, kh, kw, stride=(1, 1),
               padding=(0, 0), dilation=(1, 1), groups=1):
        return OracleBuffer(self.o.conv2d(x.data, w.data, None if bias is None else bias.data,
                                          batch, in_c, in_h, in_w, out_c, kh, kw, stride,
                                          padding, dilation, groups))

    def conv_transpose2d(self, x, w, bias, batch, in_c, in_h, in_w, out_c, kh, kw,
                         stride=(1, 1), padding=(0, 0), output_padding=(0, 0), dilation=(1, 1),
                         groups=1):
        return OracleBuffer(self.o.conv_transpose2d(
            x.data, w.data, None if bias is None else bias.data, batch, in_c, in_h, in_w, out_c,
            kh, kw, stride, padding, output_padding, dilation, groups))

    def conv2d_grad_weight(self, x, go, batch, in_c, in_h, in_w, out_c, out_h, out_w, kh, kw,
                           sh, sw, ph, pw, dh, dw, groups):
        return OracleBuffer(self.o.conv2d_grad_weight(x.data, go.data, batch, in_c, in_h, in_w,
                                                      out_c, out_h, out_w, kh, kw, sh, sw, ph,
                                                      pw, dh, dw, groups))

    def conv2d_grad_bias(self, go, batch, out_c, out_h, out_w):
        return OracleBuffer(self.o.conv2d_grad_bias(go.data, batch, out_c, out_h, out_w))

    # norms and tensor ops
    def group_norm(self, x, g, b, batch, channels, spatial, groups, eps):
        return OracleBuffer(self.o.group_norm(x.data, g.data, b.data, batch, channels, spatial,
                                              groups, eps))

    def group_norm_backward(self, go, x, g, batch, channels, spatial, groups, eps):
        outs = self.o.group_norm_backward(go.data, x.data, g.data, batch, channels, spatial,
                                          groups, eps)
        return tuple(OracleBuffer(o) for o in outs)

    def concat(self, a, b, outer, ai, bi):
        return OracleBuffer(self.o.concat(a.data, b.data, outer, ai, bi))

    def slice_per_block(self, src, outer, size, offset, combined):
        return OracleBuffer(self.o.slice_per_block(src.data, outer, size, offset, combined))

    def upsample_nearest2d(self, x, batch, channels, in_h, in_w, sh, sw):
        return OracleBuffer(self.o.upsample_nearest2d(x.data, batch, channels, in_h, in_w, sh,
                                                      sw))

    def upsample_nearest2d_backward(self, go, batch, channels, in_h, in_w, sh, sw):
        return OracleBuffer(self.o.upsample_nearest2d_backward(go.data, batch, channels, in_h,
                                                               in_w, sh, sw))

    def add_broadcast(self, a, b, outer, inner):
        return OracleBuffer(self.o.add_broadcast(a.data, b.data, outer, inner))

    def sum_inner(self, src, outer, inner):
        return OracleBuffer(self.o.sum_inner(src.data, outer, inner))

    def add_per_col(self, a, b, rows, cols):
        return OracleBuffer(self.o.add_per_col(a.data, b.data, rows, cols))

    def sum_rows(self, src, rows, cols):
        return OracleBuffer(self.o.sum_rows(src.data, rows, cols))
