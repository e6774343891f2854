"""Python host mirror of any-gpu's `GpuDevice` API over the libagpu C ABI.

Method names, argument order and error behaviour follow the reference crate
(`src/device.rs`, `src/ops/*.rs`): every op returns a new `GpuBuffer`, size
mismatches raise `AnyGpuError` (the reference returns `Err` from `ensure!`),
`read` blocks until the device stream has drained.

    dev = GpuDevice.gpu()
    c = dev.matmul(dev.upload(a), dev.upload(b), m, n, k)   # (m, n, k) order
    out = dev.read(c)

All compute runs in libagpu.so's sm_100a kernels; this module only marshals
handles and host arrays.
"""
from __future__ import annotations

import contextlib
import ctypes as C
from typing import Optional, Sequence

import numpy as np

from . import _lib

__all__ = ["GpuDevice", "GpuBuffer", "AnyGpuError", "PRECISIONS"]

PRECISIONS = {"tf32": 0, "tf32x3": 1, "ffma": 2}
_STATUS_NAMES = {0: "OK", 1: "SHAPE", 2: "INVALID", 3: "CUDA", 4: "OOM", 5: "NO_DEVICE",
                 6: "TIMEOUT", 7: "UNSUPPORTED"}


class AnyGpuError(RuntimeError):
    """A failed C-ABI call; `.status` holds the agpu_status code."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[{_STATUS_NAMES.get(status, status)}] {msg}")
        self.status = status


def _check(status: int) -> None:
    if status != 0:
        lib = _lib.load()
        raise AnyGpuError(status, lib.agpu_last_error_message().decode(errors="replace"))


class GpuBuffer:
    """Owned device buffer of f32 (reference: `GpuBuffer`, src/device.rs:22-26)."""

    __slots__ = ("_h", "_dev", "len")

    def __init__(self, handle: int, dev: "GpuDevice"):
        self._h = C.c_void_p(handle)
        self._dev = dev
        self.len = int(_lib.load().agpu_buffer_len(self._h))

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @property
    def device_ptr(self) -> int:
        return int(_lib.load().agpu_buffer_device_ptr(self._h) or 0)

    def free(self) -> None:
        if self._h and self._h.value:
            _lib.load().agpu_buffer_free(self._h)
            self._h = C.c_void_p(None)

    def __del__(self):  # Drop
        try:
            self.free()
        except Exception:
            pass

    def __len__(self) -> int:
        return self.len


def _f32(data) -> np.ndarray:
    arr = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
    return arr


class GpuDevice:
    """One CUDA device, its stream and memory pool (reference: `GpuDevice`)."""

    def __init__(self, ordinal: int = 0):
        lib = _lib.load()
        h = C.c_void_p()
        _check(lib.agpu_device_create(ordinal, C.byref(h)))
        self._h = h
        name = C.create_string_buffer(256)
        _check(lib.agpu_device_name(h, name, 256))
        self.adapter_name = name.value.decode()
        self.backend = "CUDA sm_100a"
        self.ordinal = ordinal

    @classmethod
    def gpu(cls, ordinal: int = 0) -> "GpuDevice":
        """Reference: `GpuDevice::gpu()` (src/device.rs:31)."""
        return cls(ordinal)

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            _lib.load().agpu_device_destroy(self._h)
            self._h = C.c_void_p(None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ plumbing --
    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @property
    def stream(self) -> int:
        return int(_lib.load().agpu_device_stream(self._h) or 0)

    @property
    def sm_count(self) -> int:
        v = C.c_int()
        _check(_lib.load().agpu_device_sm_count(self._h, C.byref(v)))
        return v.value

    @property
    def launch_count(self) -> int:
        return int(_lib.load().agpu_device_launch_count(self._h))

    def synchronize(self) -> None:
        _check(_lib.load().agpu_synchronize(self._h))

    def set_precision(self, mode: str) -> None:
        _check(_lib.load().agpu_set_precision(self._h, PRECISIONS[mode]))

    def get_precision(self) -> str:
        v = C.c_int()
        _check(_lib.load().agpu_get_precision(self._h, C.byref(v)))
        return {v_: k for k, v_ in PRECISIONS.items()}[v.value]

    @staticmethod
    @contextlib.contextmanager
    def precision(mode: str):
        """Per-call precision: contractions enqueued by this thread inside the
        block use `mode`; the devices' own settings and other threads are
        untouched (agpu_set_thread_precision)."""
        lib = _lib.load()
        prev = lib.agpu_get_thread_precision()
        _check(lib.agpu_set_thread_precision(PRECISIONS[mode]))
        try:
            yield
        finally:
            lib.agpu_set_thread_precision(prev)

    def selftest_wait_timeout(self, limit_us: int = 1000, stream: int = 0) -> None:
        """Launch the bounded-wait failure self-test (agpu_selftest_wait_timeout):
        the next synchronize() on the device stream raises a TIMEOUT error."""
        _check(_lib.load().agpu_selftest_wait_timeout(self._h, int(limit_us),
                                                      C.c_void_p(stream or None)))

    def _new(self, fn, *args) -> GpuBuffer:
        out = C.c_void_p()
        _check(fn(self._h, *args, C.byref(out)))
        return GpuBuffer(out.value, self)

    # ------------------------------------------------------------- buffers --
    def upload(self, data) -> GpuBuffer:
        """Reference: `upload(&[f32])` (src/device.rs:80)."""
        arr = _f32(data)
        out = C.c_void_p()
        _check(_lib.load().agpu_upload(self._h, arr.ctypes.data_as(C.c_void_p), arr.size,
                                       C.byref(out)))
        # the H2D copy is stream-ordered from pageable memory: it has completed
        # (or been staged) before agpu_upload returns, so `arr` may be dropped.
        return GpuBuffer(out.value, self)

    def alloc(self, n: int) -> GpuBuffer:
        """Reference: `alloc(n)` (src/device.rs:97)."""
        out = C.c_void_p()
        _check(_lib.load().agpu_alloc(self._h, int(n), C.byref(out)))
        return GpuBuffer(out.value, self)

    def read(self, buf: GpuBuffer, out: Optional[np.ndarray] = None) -> np.ndarray:
        """Reference: `read(&GpuBuffer) -> Vec<f32>` (src/device.rs:115)."""
        if out is None:
            out = np.empty(buf.len, dtype=np.float32)
        _check(_lib.load().agpu_read(self._h, buf.handle, out.ctypes.data_as(C.c_void_p),
                                     out.size))
        return out

    def write(self, buf: GpuBuffer, data: np.ndarray) -> None:
        arr = _f32(data)
        _check(_lib.load().agpu_write(self._h, buf.handle, arr.ctypes.data_as(C.c_void_p),
                                      arr.size))

    def write_async(self, buf: GpuBuffer, host_ptr: int, n: int, offset: int = 0,
                    stream: int = 0) -> None:
        """Copy n floats from host address `host_ptr` into buf[offset:offset+n] on
        `stream` without waiting (the host memory must outlive the copy)."""
        _check(_lib.load().agpu_write_async(self._h, buf.handle, int(offset), host_ptr, int(n),
                                            stream or None))

    def read_async(self, buf: GpuBuffer, host_ptr: int, n: int, offset: int = 0,
                   stream: int = 0) -> None:
        """Copy buf[offset:offset+n] to host address `host_ptr` on `stream` without
        waiting."""
        _check(_lib.load().agpu_read_async(self._h, buf.handle, int(offset), host_ptr, int(n),
                                           stream or None))

    # -------------------------------------------------------- contractions --
    def matmul(self, a: GpuBuffer, b: GpuBuffer, m: int, n: int, k: int) -> GpuBuffer:
        """C[m,n] = A[m,k] B[k,n]; reference `matmul(a,b,m,n,k)` (src/ops/conv.rs:416)."""
        return self._new(_lib.load().agpu_matmul, a.handle, b.handle, m, n, k)

    def batch_matmul(self, a, b, batch: int, m: int, n: int, k: int) -> GpuBuffer:
        """Reference: `batch_matmul(a,b,batch,m,n,k)` (src/ops/conv.rs:426)."""
        return self._new(_lib.load().agpu_batch_matmul, a.handle, b.handle, batch, m, n, k)

    def batch_matmul_softmax(self, a, b, batch: int, m: int, n: int, k: int) -> GpuBuffer:
        """batch_matmul then a row softmax over the result, in one call (the
        softmax runs in place on the product)."""
        return self._new(_lib.load().agpu_batch_matmul_softmax, a.handle, b.handle, batch, m,
                         n, k)

    def gemm(self, a, b, batch: int, m: int, n: int, k: int, trans_a: bool = False,
             trans_b: bool = False) -> GpuBuffer:
        """C[b] = op(A[b]) op(B[b]); op = transpose when trans_* (autograd backward GEMMs)."""
        return self._new(_lib.load().agpu_gemm, a.handle, b.handle, batch, m, n, k,
                         int(trans_a), int(trans_b))

    def gemm_ex(self, a, b, batch: int, m: int, n: int, k: int, bias=None, resid=None,
                act: int = 0, trans_a: bool = False, trans_b: bool = False) -> GpuBuffer:
        """C = act(op(A) op(B) + bias[col] + resid); act 0 none, 1 swish, 2 relu."""
        return self._new(_lib.load().agpu_gemm_ex, a.handle, b.handle,
                         bias.handle if bias is not None else None,
                         resid.handle if resid is not None else None, batch, m, n, k,
                         int(trans_a), int(trans_b), int(act))

    def softmax(self, x: GpuBuffer, rows: int, cols: int) -> GpuBuffer:
        """Reference: `softmax(input, rows, cols)` (src/ops/attention.rs:91)."""
        return self._new(_lib.load().agpu_softmax, x.handle, rows, cols)

    # -------------------------------------------------------------- conv2d --
    def conv2d(self, input, weight, bias, batch, in_c, in_h, in_w, out_c, kh, kw,
               stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1) -> GpuBuffer:
        """Reference: `conv2d(input, weight, bias, batch, in_c, in_h, in_w, out_c, kh, kw,
        stride, padding, dilation, groups)` (src/ops/conv.rs:437)."""
        return self._new(_lib.load().agpu_conv2d, input.handle, weight.handle,
                         bias.handle if bias is not None else None, batch, in_c, in_h, in_w,
                         out_c, kh, kw, stride[0], stride[1], padding[0], padding[1],
                         dilation[0], dilation[1], groups)

    def conv2d_group_norm_swish(self, input, weight, bias, batch, in_c, in_h, in_w, out_c, kh,
                                kw, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1,
                                gamma=None, beta=None, gn_groups=32, eps=1e-5) -> GpuBuffer:
        """swish(group_norm(conv2d(...))) in one call (the UNet block)."""
        return self._new(_lib.load().agpu_conv2d_group_norm_swish, input.handle, weight.handle,
                         bias.handle if bias is not None else None, batch, in_c, in_h, in_w,
                         out_c, kh, kw, stride[0], stride[1], padding[0], padding[1],
                         dilation[0], dilation[1], groups, gamma.handle, beta.handle, gn_groups,
                         C.c_float(eps))

    def conv_transpose2d(self, input, weight, bias, batch, in_c, in_h, in_w, out_c, kh, kw,
                         stride=(1, 1), padding=(0, 0), output_padding=(0, 0),
                         dilation=(1, 1), groups=1) -> GpuBuffer:
        """Reference: `conv_transpose2d(...)` (src/ops/conv.rs:484)."""
        return self._new(_lib.load().agpu_conv_transpose2d, input.handle, weight.handle,
                         bias.handle if bias is not None else None, batch, in_c, in_h, in_w,
                         out_c, kh, kw, stride[0], stride[1], padding[0], padding[1],
                         output_padding[0], output_padding[1], dilation[0], dilation[1], groups)

    def conv2d_grad_weight(self, input, grad_out, batch, in_c, in_h, in_w, out_c, out_h, out_w,
                           kh, kw, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w,
                           groups) -> GpuBuffer:
        """Reference: `conv2d_grad_weight(...)` (src/ops/conv.rs:531)."""
        return self._new(_lib.load().agpu_conv2d_grad_weight, input.handle, grad_out.handle,
                         batch, in_c, in_h, in_w, out_c, out_h, out_w, kh, kw, stride_h,
                         stride_w, pad_h, pad_w, dil_h, dil_w, groups)

    def conv2d_grad_bias(self, grad_out, batch, out_c, out_h, out_w) -> GpuBuffer:
        """Reference: `conv2d_grad_bias(...)` (src/ops/conv.rs:551)."""
        return self._new(_lib.load().agpu_conv2d_grad_bias, grad_out.handle, batch, out_c,
                         out_h, out_w)

    # ---------------------------------------------------------- group norm --
    def group_norm(self, x, gamma, beta, batch: int, channels: int, spatial: int, groups: int,
                   eps: float) -> GpuBuffer:
        """Reference: `group_norm(input, gamma, beta, batch, channels, spatial, groups, eps)`
        (src/ops/norm.rs:210)."""
        return self._new(_lib.load().agpu_group_norm, x.handle, gamma.handle, beta.handle, batch,
                         channels, spatial, groups, C.c_float(eps))

    def group_norm_swish(self, x, gamma, beta, batch: int, channels: int, spatial: int,
                         groups: int, eps: float) -> GpuBuffer:
        """group_norm then swish in one pass."""
        return self._new(_lib.load().agpu_group_norm_swish, x.handle, gamma.handle, beta.handle,
                         batch, channels, spatial, groups, C.c_float(eps))

    def group_norm_backward(self, grad_out, x, gamma, batch: int, channels: int, spatial: int,
                            groups: int, eps: float):
        """Reference: `group_norm_backward(grad_out, input, gamma, batch, channels, spatial,
        groups, eps) -> (d_input, d_gamma, d_beta)` (src/ops/norm.rs:282)."""
        outs = [C.c_void_p() for _ in range(3)]
        _check(_lib.load().agpu_group_norm_backward(self._h, grad_out.handle, x.handle,
                                                    gamma.handle, batch, channels, spatial,
                                                    groups, C.c_float(eps),
                                                    *[C.byref(o) for o in outs]))
        return tuple(GpuBuffer(o.value, self) for o in outs)

    # ---------------------------------------------------------------- sdpa --
    def scaled_dot_product_attention(self, q, k, v, batch_heads: int, seq_len: int,
                                     d_k: int) -> GpuBuffer:
        """Reference: `scaled_dot_product_attention(q, k, v, batch_heads, seq_len, d_k)`
        (src/ops/attention.rs:149)."""
        return self._new(_lib.load().agpu_scaled_dot_product_attention, q.handle, k.handle,
                         v.handle, batch_heads, seq_len, d_k)

    def sdpa_causal(self, q, k, v, batch_heads: int, seq_len: int, d_k: int) -> GpuBuffer:
        return self._new(_lib.load().agpu_sdpa_causal, q.handle, k.handle, v.handle,
                         batch_heads, seq_len, d_k)

    def sdpa_backward(self, q, k, v, grad_out, batch_heads: int, seq_len: int, d_k: int,
                      causal: bool = False):
        """dQ, dK, dV of scaled_dot_product_attention from dO (agpu_sdpa_backward)."""
        outs = [C.c_void_p(), C.c_void_p(), C.c_void_p()]
        _check(_lib.load().agpu_sdpa_backward(self._h, q.handle, k.handle, v.handle,
                                              grad_out.handle, batch_heads, seq_len, d_k,
                                              int(causal), *(C.byref(o) for o in outs)))
        return tuple(GpuBuffer(o.value, self) for o in outs)

    def launch_sdpa_backward(self, q_ptr, k_ptr, v_ptr, do_ptr, dq_ptr, dk_ptr, dv_ptr, bh, s, d,
                             causal=False, stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_sdpa_backward(self._h, q_ptr, k_ptr, v_ptr, do_ptr, dq_ptr,
                                                     dk_ptr, dv_ptr, bh, s, d, int(causal),
                                                     stream or None))

    def launch_sdpa(self, q_ptr, k_ptr, v_ptr, o_ptr, bh, s, d, causal=False,
                    stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_sdpa(self._h, q_ptr, k_ptr, v_ptr, o_ptr, bh, s, d,
                                            int(causal), stream or None))

    # ----------------------------------------------------- LLaMA-layer ops --
    def rmsnorm(self, x, w, rows: int, cols: int, eps: float) -> GpuBuffer:
        return self._new(_lib.load().agpu_rmsnorm, x.handle, w.handle, rows, cols,
                         C.c_float(eps))

    def rope(self, x, batch: int, seq: int, heads: int, dim: int,
             base: float = 10000.0) -> GpuBuffer:
        return self._new(_lib.load().agpu_rope, x.handle, batch, seq, heads, dim,
                         C.c_float(base))

    def swish_mul(self, gate, up) -> GpuBuffer:
        return self._new(_lib.load().agpu_swish_mul, gate.handle, up.handle)

    def launch_gemm_ex(self, a_ptr, b_ptr, c_ptr, batch, m, n, k, trans_a=False,
                       trans_b=False, bias_ptr=0, resid_ptr=0, act=0, stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_gemm_ex(self._h, a_ptr, b_ptr, c_ptr, batch, m, n, k,
                                               int(trans_a), int(trans_b), bias_ptr or None,
                                               resid_ptr or None, int(act), stream or None))

    def launch_sdpa_strided(self, q_ptr, k_ptr, v_ptr, o_ptr, batch, heads, seq, d, q_strides,
                            k_strides, v_strides, o_strides, causal=False,
                            stream: int = 0) -> None:
        """*_strides = (seq_stride, head_stride, batch_stride) in elements."""
        lay = [_lib.AttnLayout(*map(int, st)) for st in (q_strides, k_strides, v_strides,
                                                          o_strides)]
        _check(_lib.load().agpu_launch_sdpa_strided(self._h, q_ptr, k_ptr, v_ptr, o_ptr, batch,
                                                    heads, seq, d, *[C.byref(x) for x in lay],
                                                    int(causal), stream or None))

    def launch_rmsnorm(self, x_ptr, w_ptr, y_ptr, rows, cols, eps, stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_rmsnorm(self._h, x_ptr, w_ptr, y_ptr, rows, cols,
                                               C.c_float(eps), stream or None))

    def launch_rope(self, x_ptr, y_ptr, batch, seq, heads, dim, row_stride, base=10000.0,
                    stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_rope(self._h, x_ptr, y_ptr, batch, seq, heads, dim,
                                            row_stride, C.c_float(base), stream or None))

    def launch_swish_mul(self, g_ptr, u_ptr, o_ptr, rows, cols, g_stride, u_stride, o_stride,
                         stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_swish_mul(self._h, g_ptr, u_ptr, o_ptr, rows, cols,
                                                 g_stride, u_stride, o_stride, stream or None))

    # --------------------------------------------------------- elementwise --
    def add(self, a, b): return self._new(_lib.load().agpu_add, a.handle, b.handle)
    def sub(self, a, b): return self._new(_lib.load().agpu_sub, a.handle, b.handle)
    def mul(self, a, b): return self._new(_lib.load().agpu_mul, a.handle, b.handle)
    def relu(self, a): return self._new(_lib.load().agpu_relu, a.handle)
    def sigmoid(self, a): return self._new(_lib.load().agpu_sigmoid, a.handle)
    def swish(self, a): return self._new(_lib.load().agpu_swish, a.handle)
    def tanh_act(self, a): return self._new(_lib.load().agpu_tanh_act, a.handle)

    def scale(self, a, s: float):
        return self._new(_lib.load().agpu_scale, a.handle, C.c_float(s))

    def relu_backward(self, grad_out, input):
        return self._new(_lib.load().agpu_relu_backward, grad_out.handle, input.handle)

    def sigmoid_backward(self, grad_out, output):
        return self._new(_lib.load().agpu_sigmoid_backward, grad_out.handle, output.handle)

    def swish_backward(self, grad_out, input):
        return self._new(_lib.load().agpu_swish_backward, grad_out.handle, input.handle)

    def tanh_backward(self, grad_out, output):
        return self._new(_lib.load().agpu_tanh_backward, grad_out.handle, output.handle)

    # ---------------------------------------------------------- tensor ops --
    def transpose(self, a, outer_size: int, d0: int, d1: int, inner: int):
        """Reference: `transpose(a, outer, d0, d1, inner)` (src/ops/tensor_ops.rs:251)."""
        return self._new(_lib.load().agpu_transpose, a.handle, outer_size, d0, d1, inner)

    def add_per_col(self, a, b, rows: int, cols: int):
        """Reference: `add_per_col(a, b, rows, cols)` (src/ops/tensor_ops.rs:336)."""
        return self._new(_lib.load().agpu_add_per_col, a.handle, b.handle, rows, cols)

    def add_broadcast(self, a, b, outer: int, inner: int):
        """Reference: `add_broadcast(a, b, outer, inner)` (src/ops/tensor_ops.rs:298)."""
        return self._new(_lib.load().agpu_add_broadcast, a.handle, b.handle, outer, inner)

    def sum_inner(self, src, outer: int, inner: int):
        """Reference: `sum_inner(src, outer, inner)` (src/ops/tensor_ops.rs:318)."""
        return self._new(_lib.load().agpu_sum_inner, src.handle, outer, inner)

    def sum_rows(self, src, rows: int, cols: int):
        """Reference: `sum_rows(src, rows, cols)` (src/ops/tensor_ops.rs:356)."""
        return self._new(_lib.load().agpu_sum_rows, src.handle, rows, cols)

    def concat(self, a, b, outer_size: int, a_inner: int, b_inner: int):
        """Reference: `concat(a, b, outer_size, a_inner, b_inner)` (src/ops/tensor_ops.rs:229)."""
        return self._new(_lib.load().agpu_concat, a.handle, b.handle, outer_size, a_inner,
                         b_inner)

    def slice_per_block(self, src, outer: int, slice_size: int, slice_offset: int,
                        combined: int):
        """Reference: `slice_per_block(src, outer, slice_size, slice_offset, combined)`
        (src/ops/tensor_ops.rs:274)."""
        return self._new(_lib.load().agpu_slice_per_block, src.handle, outer, slice_size,
                         slice_offset, combined)

    def upsample_nearest2d(self, input, batch: int, channels: int, in_h: int, in_w: int,
                           scale_h: int, scale_w: int):
        """Reference: `upsample_nearest2d(...)` (src/ops/upsample.rs:94)."""
        return self._new(_lib.load().agpu_upsample_nearest2d, input.handle, batch, channels,
                         in_h, in_w, scale_h, scale_w)

    def upsample_nearest2d_backward(self, grad_out, batch: int, channels: int, in_h: int,
                                    in_w: int, scale_h: int, scale_w: int):
        """Reference: `upsample_nearest2d_backward(...)` (src/ops/upsample.rs:116)."""
        return self._new(_lib.load().agpu_upsample_nearest2d_backward, grad_out.handle, batch,
                         channels, in_h, in_w, scale_h, scale_w)

    def mse_loss(self, pred, target):
        """Reference: `mse_loss(pred, target)` (src/ops/attention.rs:172): 1 element."""
        return self._new(_lib.load().agpu_mse_loss, pred.handle, target.handle)

    # ------------------------------------------- launch layer (raw pointers) --
    def launch_batch_matmul(self, a_ptr: int, b_ptr: int, c_ptr: int, batch: int, m: int,
                            n: int, k: int, stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_batch_matmul(self._h, a_ptr, b_ptr, c_ptr, batch, m, n,
                                                    k, stream or None))

    def launch_conv2d(self, x_ptr, w_ptr, bias_ptr, y_ptr, batch, in_c, in_h, in_w, out_c, kh,
                      kw, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w, groups,
                      stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_conv2d(self._h, x_ptr, w_ptr, bias_ptr or None, y_ptr,
                                              batch, in_c, in_h, in_w, out_c, kh, kw, stride_h,
                                              stride_w, pad_h, pad_w, dil_h, dil_w, groups,
                                              stream or None))

    def launch_batch_matmul_softmax(self, a_ptr: int, b_ptr: int, out_ptr: int, batch: int,
                                    m: int, n: int, k: int, stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_batch_matmul_softmax(self._h, a_ptr, b_ptr, out_ptr,
                                                            batch, m, n, k, stream or None))

    def launch_conv2d_group_norm_swish(self, x_ptr, w_ptr, bias_ptr, y_ptr, batch, in_c, in_h,
                                       in_w, out_c, kh, kw, stride_h, stride_w, pad_h, pad_w,
                                       dil_h, dil_w, groups, gamma_ptr, beta_ptr, gn_groups, eps,
                                       stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_conv2d_group_norm_swish(
            self._h, x_ptr, w_ptr, bias_ptr or None, y_ptr, batch, in_c, in_h, in_w, out_c, kh,
            kw, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w, groups, gamma_ptr, beta_ptr,
            gn_groups, C.c_float(eps), stream or None))

    def launch_group_norm_backward(self, dy_ptr, x_ptr, g_ptr, dx_ptr, dg_ptr, db_ptr, batch,
                                   channels, spatial, groups, eps, stream=0):
        _check(_lib.load().agpu_launch_group_norm_backward(
            self._h, dy_ptr, x_ptr, g_ptr, dx_ptr, dg_ptr, db_ptr, batch, channels, spatial,
            groups, C.c_float(eps), stream))

    def launch_group_norm(self, x_ptr, g_ptr, b_ptr, y_ptr, batch, channels, spatial, groups,
                          eps, swish=False, stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_group_norm(self._h, x_ptr, g_ptr, b_ptr, y_ptr, batch,
                                                  channels, spatial, groups, C.c_float(eps),
                                                  int(swish), stream or None))

    def launch_softmax(self, x_ptr: int, y_ptr: int, rows: int, cols: int,
                       stream: int = 0) -> None:
        _check(_lib.load().agpu_launch_softmax(self._h, x_ptr, y_ptr, rows, cols,
                                               stream or None))


class AdamW:
    """Mirror of the reference optimizer (src/optim.rs:53-138): lr, beta1 0.9,
    beta2 0.999, eps 1e-8, weight_decay 0.01; moment buffers created (zero) on
    the first step; each step updates every parameter buffer in place in one
    launch (agpu_adamw_step)."""

    def __init__(self, lr: float):
        self.lr, self.beta1, self.beta2, self.eps, self.weight_decay = lr, 0.9, 0.999, 1e-8, 0.01
        self.step_count = 0
        self.states: list[tuple[GpuBuffer, GpuBuffer]] = []

    def step(self, dev: "GpuDevice", params: list, grads: list) -> None:
        """Reference: `AdamW::step(dev, params, grads)` (src/optim.rs:82)."""
        if len(params) != len(grads):
            raise AnyGpuError(1, "params/grads length mismatch")
        self.step_count += 1
        while len(self.states) < len(params):
            n = params[len(self.states)].len
            self.states.append((dev.alloc(n), dev.alloc(n)))  # zero-filled
        k = len(params)
        arr = lambda bufs: (C.c_void_p * max(k, 1))(*[b.handle for b in bufs])
        _check(_lib.load().agpu_adamw_step(
            dev._h, arr(params), arr(grads), arr([s[0] for s in self.states[:k]]),
            arr([s[1] for s in self.states[:k]]), k, C.c_float(self.lr), C.c_float(self.beta1),
            C.c_float(self.beta2), C.c_float(self.eps), C.c_float(self.weight_decay),
            self.step_count))
