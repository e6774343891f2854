//! `GpuDevice` and `GpuBuffer` with the reference crate's names, argument
//! order and error behaviour (any-gpu `src/device.rs:12-145` and the
//! `impl GpuDevice` blocks of `src/ops/*.rs`), over libagpu's C ABI.  A
//! crate that did `use any_gpu::{GpuDevice, GpuBuffer}` compiles against this
//! one unchanged: ops take `&self` and `&GpuBuffer`s and return a new owned
//! `Result<GpuBuffer>`; size mismatches come back as `Err` (the C library
//! checks them where the reference's `ensure!` does, before any launch);
//! `upload` / `alloc` are infallible as in the reference and panic only if
//! device memory runs out; `read` blocks until the device stream drains.
//!
//! Beyond the reference's surface: the precision mode, the fused entry points
//! (`batch_matmul_softmax`, `group_norm_swish`, `conv2d_group_norm_swish`,
//! `gemm_ex`), the LLaMA-layer ops, and the multi-tensor AdamW step.

use std::ffi::CStr;
use std::fmt;
use std::os::raw::c_int;
use std::ptr;

use anyhow::Result;

use crate::ffi;

/// A failed C-ABI call: the `agpu_status` code and the library's message
/// (the text the reference's `anyhow::Error` would carry).
#[derive(Debug, Clone)]
pub struct AgpuError {
    pub status: i32,
    pub message: String,
}

impl fmt::Display for AgpuError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        let name = unsafe { CStr::from_ptr(ffi::agpu_status_string(self.status)) };
        write!(f, "{} ({}): {}", name.to_string_lossy(), self.status, self.message)
    }
}

impl std::error::Error for AgpuError {}

fn check(status: ffi::AgpuStatus) -> Result<()> {
    if status == ffi::AGPU_OK {
        return Ok(());
    }
    let message = unsafe { CStr::from_ptr(ffi::agpu_last_error_message()) }
        .to_string_lossy()
        .into_owned();
    Err(AgpuError { status, message }.into())
}

/// Arithmetic of the contractions (matmul, batch_matmul, sdpa, conv2d).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum Precision {
    /// tcgen05 kind::tf32 with fp32 accumulation (default).
    Tf32 = 0,
    /// error-corrected 3xTF32 on the tensor cores: fp32-level accuracy.
    Tf32x3 = 1,
    /// SIMT fp32 FFMA (the reference's arithmetic, slow).
    Ffma = 2,
}

/// GPU-resident f32 buffer (reference: `GpuBuffer`, src/device.rs:22-26).
/// Dropping it returns the memory to its device's pool; it keeps the device
/// alive until then, as the reference's buffer holds its wgpu device.
pub struct GpuBuffer {
    raw: *mut ffi::AgpuBuffer,
    pub len: usize,
}

// The C library is thread-safe and a buffer is plain device memory.
unsafe impl Send for GpuBuffer {}
unsafe impl Sync for GpuBuffer {}

impl GpuBuffer {
    fn from_raw(raw: *mut ffi::AgpuBuffer) -> Self {
        let len = unsafe { ffi::agpu_buffer_len(raw) } as usize;
        GpuBuffer { raw, len }
    }

    fn c(&self) -> *const ffi::AgpuBuffer {
        self.raw
    }

    /// Device address of the first element (for interop with other CUDA code).
    pub fn device_ptr(&self) -> *mut f32 {
        unsafe { ffi::agpu_buffer_device_ptr(self.raw) as *mut f32 }
    }
}

impl Drop for GpuBuffer {
    fn drop(&mut self) {
        unsafe {
            ffi::agpu_buffer_free(self.raw);
        }
    }
}

fn opt(b: Option<&GpuBuffer>) -> *const ffi::AgpuBuffer {
    b.map_or(ptr::null(), |b| b.c())
}

/// One CUDA B200 device, its stream and memory pool (reference: `GpuDevice`,
/// src/device.rs:12-20).
pub struct GpuDevice {
    raw: *mut ffi::AgpuDevice,
    pub adapter_name: String,
    pub backend: String,
}

unsafe impl Send for GpuDevice {}
unsafe impl Sync for GpuDevice {}

impl Drop for GpuDevice {
    fn drop(&mut self) {
        unsafe {
            ffi::agpu_device_destroy(self.raw);
        }
    }
}

impl GpuDevice {
    /// Reference: `GpuDevice::gpu()` (src/device.rs:31): the first GPU.
    pub fn gpu() -> Result<Self> {
        Self::with_ordinal(0)
    }

    /// The CUDA device `ordinal` (one process per GPU in a multi-GPU job).
    pub fn with_ordinal(ordinal: i32) -> Result<Self> {
        let mut raw = ptr::null_mut();
        check(unsafe { ffi::agpu_device_create(ordinal as c_int, &mut raw) })?;
        // owned from here on: an error below destroys the handle on drop
        let mut dev = GpuDevice { raw, adapter_name: String::new(), backend: "CUDA sm_100a".into() };
        let mut name = [0 as std::os::raw::c_char; 256];
        check(unsafe { ffi::agpu_device_name(dev.raw, name.as_mut_ptr(), name.len()) })?;
        dev.adapter_name = unsafe { CStr::from_ptr(name.as_ptr()) }.to_string_lossy().into_owned();
        Ok(dev)
    }

    fn out(&self, f: impl FnOnce(*mut *mut ffi::AgpuBuffer) -> ffi::AgpuStatus) -> Result<GpuBuffer> {
        let mut raw = ptr::null_mut();
        check(f(&mut raw))?;
        Ok(GpuBuffer::from_raw(raw))
    }

    // ---------------------------------------------------------- plumbing --
    pub fn synchronize(&self) -> Result<()> {
        check(unsafe { ffi::agpu_synchronize(self.raw) })
    }

    pub fn set_precision(&self, p: Precision) -> Result<()> {
        check(unsafe { ffi::agpu_set_precision(self.raw, p as c_int) })
    }

    /// Run `f` with the contractions it enqueues from this thread in
    /// precision `p`, leaving the device's own setting untouched.
    pub fn with_precision<T>(p: Precision, f: impl FnOnce() -> T) -> Result<T> {
        let prev = unsafe { ffi::agpu_get_thread_precision() };
        check(unsafe { ffi::agpu_set_thread_precision(p as c_int) })?;
        let r = f();
        unsafe {
            ffi::agpu_set_thread_precision(prev);
        }
        Ok(r)
    }

    /// Number of this library's kernels launched on the device so far.
    pub fn launch_count(&self) -> u64 {
        unsafe { ffi::agpu_device_launch_count(self.raw) }
    }

    // ------------------------------------------------------------ buffers --
    /// Reference: `upload(&[f32]) -> GpuBuffer` (src/device.rs:80).
    pub fn upload(&self, data: &[f32]) -> GpuBuffer {
        self.out(|o| unsafe { ffi::agpu_upload(self.raw, data.as_ptr(), data.len() as u64, o) })
            .expect("agpu_upload")
    }

    /// Reference: `alloc(n) -> GpuBuffer` (src/device.rs:97), zero-filled.
    pub fn alloc(&self, n: usize) -> GpuBuffer {
        self.out(|o| unsafe { ffi::agpu_alloc(self.raw, n as u64, o) }).expect("agpu_alloc")
    }

    /// Reference: `read(&GpuBuffer) -> Result<Vec<f32>>` (src/device.rs:115).
    pub fn read(&self, buf: &GpuBuffer) -> Result<Vec<f32>> {
        let mut v = vec![0f32; buf.len];
        check(unsafe { ffi::agpu_read(self.raw, buf.c(), v.as_mut_ptr(), v.len() as u64) })?;
        Ok(v)
    }

    /// Overwrite a buffer from host memory (stream-ordered).
    pub fn write(&self, buf: &GpuBuffer, data: &[f32]) -> Result<()> {
        check(unsafe { ffi::agpu_write(self.raw, buf.raw, data.as_ptr(), data.len() as u64) })
    }

    // ------------------------------------------------------- contractions --
    /// Reference: src/ops/conv.rs:416 — argument order (m, n, k).
    pub fn matmul(&self, a: &GpuBuffer, b: &GpuBuffer, m: u32, n: u32, k: u32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_matmul(self.raw, a.c(), b.c(), m, n, k, o) })
    }

    /// Reference: src/ops/conv.rs:426.
    pub fn batch_matmul(
        &self, a: &GpuBuffer, b: &GpuBuffer, batch: u32, m: u32, n: u32, k: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_batch_matmul(self.raw, a.c(), b.c(), batch, m, n, k, o) })
    }

    /// batch_matmul then a row softmax of the product, one call.
    pub fn batch_matmul_softmax(
        &self, a: &GpuBuffer, b: &GpuBuffer, batch: u32, m: u32, n: u32, k: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_batch_matmul_softmax(self.raw, a.c(), b.c(), batch, m, n, k, o)
        })
    }

    /// C[b] = op(A[b]) op(B[b]) with optionally transposed operands (the
    /// GEMMs of the autograd matmul backward, src/autograd.rs:357-366).
    pub fn gemm(
        &self, a: &GpuBuffer, b: &GpuBuffer, batch: u32, m: u32, n: u32, k: u32,
        trans_a: bool, trans_b: bool,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_gemm(self.raw, a.c(), b.c(), batch, m, n, k, trans_a as c_int,
                           trans_b as c_int, o)
        })
    }

    /// gemm with a fused epilogue: act(op(A) op(B) + bias[col] + resid),
    /// act 0 none, 1 swish, 2 relu, 3 SwiGLU over 32-column gate/up blocks.
    pub fn gemm_ex(
        &self, a: &GpuBuffer, b: &GpuBuffer, bias: Option<&GpuBuffer>,
        resid: Option<&GpuBuffer>, batch: u32, m: u32, n: u32, k: u32, trans_a: bool,
        trans_b: bool, act: i32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_gemm_ex(self.raw, a.c(), b.c(), opt(bias), opt(resid), batch, m, n, k,
                              trans_a as c_int, trans_b as c_int, act as c_int, o)
        })
    }

    // ---------------------------------------------------------- attention --
    /// Reference: src/ops/attention.rs:91.
    pub fn softmax(&self, input: &GpuBuffer, rows: u32, cols: u32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_softmax(self.raw, input.c(), rows, cols, o) })
    }

    /// Reference: src/ops/attention.rs:149 — one fused kernel here.
    pub fn scaled_dot_product_attention(
        &self, q: &GpuBuffer, k: &GpuBuffer, v: &GpuBuffer, batch_heads: u32, seq_len: u32,
        d_k: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_scaled_dot_product_attention(self.raw, q.c(), k.c(), v.c(), batch_heads,
                                                   seq_len, d_k, o)
        })
    }

    /// Causal attention (query i attends keys j <= i); not in the reference.
    pub fn sdpa_causal(
        &self, q: &GpuBuffer, k: &GpuBuffer, v: &GpuBuffer, batch_heads: u32, seq_len: u32,
        d_k: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_sdpa_causal(self.raw, q.c(), k.c(), v.c(), batch_heads, seq_len, d_k, o)
        })
    }

    /// Reference: src/ops/attention.rs:172.
    pub fn mse_loss(&self, pred: &GpuBuffer, target: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_mse_loss(self.raw, pred.c(), target.c(), o) })
    }

    // --------------------------------------------------------------- conv --
    /// Reference: src/ops/conv.rs:437.
    #[allow(clippy::too_many_arguments)]
    pub fn conv2d(
        &self, input: &GpuBuffer, weight: &GpuBuffer, bias: Option<&GpuBuffer>, batch: u32,
        in_c: u32, in_h: u32, in_w: u32, out_c: u32, kh: u32, kw: u32, stride: (u32, u32),
        padding: (u32, u32), dilation: (u32, u32), groups: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_conv2d(self.raw, input.c(), weight.c(), opt(bias), batch, in_c, in_h, in_w,
                             out_c, kh, kw, stride.0, stride.1, padding.0, padding.1, dilation.0,
                             dilation.1, groups, o)
        })
    }

    /// conv2d -> group_norm -> swish (the UNet block) in one call.
    #[allow(clippy::too_many_arguments)]
    pub fn conv2d_group_norm_swish(
        &self, input: &GpuBuffer, weight: &GpuBuffer, bias: Option<&GpuBuffer>, batch: u32,
        in_c: u32, in_h: u32, in_w: u32, out_c: u32, kh: u32, kw: u32, stride: (u32, u32),
        padding: (u32, u32), dilation: (u32, u32), groups: u32, gamma: &GpuBuffer,
        beta: &GpuBuffer, gn_groups: u32, eps: f32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_conv2d_group_norm_swish(self.raw, input.c(), weight.c(), opt(bias), batch,
                                              in_c, in_h, in_w, out_c, kh, kw, stride.0,
                                              stride.1, padding.0, padding.1, dilation.0,
                                              dilation.1, groups, gamma.c(), beta.c(), gn_groups,
                                              eps, o)
        })
    }

    /// Reference: src/ops/conv.rs:484.
    #[allow(clippy::too_many_arguments)]
    pub fn conv_transpose2d(
        &self, input: &GpuBuffer, weight: &GpuBuffer, bias: Option<&GpuBuffer>, batch: u32,
        in_c: u32, in_h: u32, in_w: u32, out_c: u32, kh: u32, kw: u32, stride: (u32, u32),
        padding: (u32, u32), output_padding: (u32, u32), dilation: (u32, u32), groups: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_conv_transpose2d(self.raw, input.c(), weight.c(), opt(bias), batch, in_c,
                                       in_h, in_w, out_c, kh, kw, stride.0, stride.1, padding.0,
                                       padding.1, output_padding.0, output_padding.1,
                                       dilation.0, dilation.1, groups, o)
        })
    }

    /// Reference: src/ops/conv.rs:529 (crate-private there, used by the
    /// autograd conv backward).
    #[allow(clippy::too_many_arguments)]
    pub fn conv2d_grad_weight(
        &self, input: &GpuBuffer, grad_out: &GpuBuffer, batch: u32, in_c: u32, in_h: u32,
        in_w: u32, out_c: u32, out_h: u32, out_w: u32, kh: u32, kw: u32, stride_h: u32,
        stride_w: u32, pad_h: u32, pad_w: u32, dil_h: u32, dil_w: u32, groups: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_conv2d_grad_weight(self.raw, input.c(), grad_out.c(), batch, in_c, in_h,
                                         in_w, out_c, out_h, out_w, kh, kw, stride_h, stride_w,
                                         pad_h, pad_w, dil_h, dil_w, groups, o)
        })
    }

    /// Reference: src/ops/conv.rs:552.
    pub fn conv2d_grad_bias(
        &self, grad_out: &GpuBuffer, batch: u32, out_c: u32, out_h: u32, out_w: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_conv2d_grad_bias(self.raw, grad_out.c(), batch, out_c, out_h, out_w, o)
        })
    }

    // --------------------------------------------------------- group norm --
    /// Reference: src/ops/norm.rs:210.
    #[allow(clippy::too_many_arguments)]
    pub fn group_norm(
        &self, input: &GpuBuffer, gamma: &GpuBuffer, beta: &GpuBuffer, batch: u32,
        channels: u32, spatial: u32, groups: u32, eps: f32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_group_norm(self.raw, input.c(), gamma.c(), beta.c(), batch, channels,
                                 spatial, groups, eps, o)
        })
    }

    /// group_norm followed by swish in one pass.
    #[allow(clippy::too_many_arguments)]
    pub fn group_norm_swish(
        &self, input: &GpuBuffer, gamma: &GpuBuffer, beta: &GpuBuffer, batch: u32,
        channels: u32, spatial: u32, groups: u32, eps: f32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_group_norm_swish(self.raw, input.c(), gamma.c(), beta.c(), batch, channels,
                                       spatial, groups, eps, o)
        })
    }

    /// Reference: src/ops/norm.rs:282 — (d_input, d_gamma, d_beta).
    #[allow(clippy::too_many_arguments)]
    pub fn group_norm_backward(
        &self, grad_out: &GpuBuffer, input: &GpuBuffer, gamma: &GpuBuffer, batch: u32,
        channels: u32, spatial: u32, groups: u32, eps: f32,
    ) -> Result<(GpuBuffer, GpuBuffer, GpuBuffer)> {
        let (mut dx, mut dg, mut db) = (ptr::null_mut(), ptr::null_mut(), ptr::null_mut());
        check(unsafe {
            ffi::agpu_group_norm_backward(self.raw, grad_out.c(), input.c(), gamma.c(), batch,
                                          channels, spatial, groups, eps, &mut dx, &mut dg,
                                          &mut db)
        })?;
        Ok((GpuBuffer::from_raw(dx), GpuBuffer::from_raw(dg), GpuBuffer::from_raw(db)))
    }

    // -------------------------------------------------------- elementwise --
    /// Reference: src/ops/elementwise.rs:188-250.
    pub fn add(&self, a: &GpuBuffer, b: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_add(self.raw, a.c(), b.c(), o) })
    }
    pub fn sub(&self, a: &GpuBuffer, b: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_sub(self.raw, a.c(), b.c(), o) })
    }
    pub fn mul(&self, a: &GpuBuffer, b: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_mul(self.raw, a.c(), b.c(), o) })
    }
    pub fn relu(&self, a: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_relu(self.raw, a.c(), o) })
    }
    pub fn sigmoid(&self, a: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_sigmoid(self.raw, a.c(), o) })
    }
    pub fn swish(&self, a: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_swish(self.raw, a.c(), o) })
    }
    pub fn tanh_act(&self, a: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_tanh_act(self.raw, a.c(), o) })
    }
    pub fn scale(&self, a: &GpuBuffer, s: f32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_scale(self.raw, a.c(), s, o) })
    }
    pub fn relu_backward(&self, grad_out: &GpuBuffer, input: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_relu_backward(self.raw, grad_out.c(), input.c(), o) })
    }
    pub fn sigmoid_backward(&self, grad_out: &GpuBuffer, output: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_sigmoid_backward(self.raw, grad_out.c(), output.c(), o) })
    }
    pub fn swish_backward(&self, grad_out: &GpuBuffer, input: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_swish_backward(self.raw, grad_out.c(), input.c(), o) })
    }
    pub fn tanh_backward(&self, grad_out: &GpuBuffer, output: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_tanh_backward(self.raw, grad_out.c(), output.c(), o) })
    }

    // --------------------------------------------------------- tensor ops --
    /// Reference: src/ops/tensor_ops.rs:251.
    pub fn transpose(
        &self, a: &GpuBuffer, outer_size: u32, d0: u32, d1: u32, inner: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_transpose(self.raw, a.c(), outer_size, d0, d1, inner, o) })
    }
    /// Reference: src/ops/tensor_ops.rs:229.
    pub fn concat(
        &self, a: &GpuBuffer, b: &GpuBuffer, outer_size: u32, a_inner: u32, b_inner: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_concat(self.raw, a.c(), b.c(), outer_size, a_inner, b_inner, o)
        })
    }
    /// Reference: src/ops/tensor_ops.rs:275.
    pub fn slice_per_block(
        &self, src: &GpuBuffer, outer: u32, slice_size: u32, slice_offset: u32, combined: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_slice_per_block(self.raw, src.c(), outer, slice_size, slice_offset,
                                      combined, o)
        })
    }
    /// Reference: src/ops/tensor_ops.rs:298.
    pub fn add_broadcast(&self, a: &GpuBuffer, b: &GpuBuffer, outer: u32, inner: u32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_add_broadcast(self.raw, a.c(), b.c(), outer, inner, o) })
    }
    /// Reference: src/ops/tensor_ops.rs:318.
    pub fn sum_inner(&self, src: &GpuBuffer, outer: u32, inner: u32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_sum_inner(self.raw, src.c(), outer, inner, o) })
    }
    /// Reference: src/ops/tensor_ops.rs:336.
    pub fn add_per_col(&self, a: &GpuBuffer, b: &GpuBuffer, rows: u32, cols: u32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_add_per_col(self.raw, a.c(), b.c(), rows, cols, o) })
    }
    /// Reference: src/ops/tensor_ops.rs:356.
    pub fn sum_rows(&self, src: &GpuBuffer, rows: u32, cols: u32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_sum_rows(self.raw, src.c(), rows, cols, o) })
    }
    /// Reference: src/ops/upsample.rs:94.
    #[allow(clippy::too_many_arguments)]
    pub fn upsample_nearest2d(
        &self, input: &GpuBuffer, batch: u32, channels: u32, in_h: u32, in_w: u32, scale_h: u32,
        scale_w: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_upsample_nearest2d(self.raw, input.c(), batch, channels, in_h, in_w, scale_h,
                                         scale_w, o)
        })
    }
    /// Reference: src/ops/upsample.rs:116.
    #[allow(clippy::too_many_arguments)]
    pub fn upsample_nearest2d_backward(
        &self, grad_out: &GpuBuffer, batch: u32, channels: u32, in_h: u32, in_w: u32,
        scale_h: u32, scale_w: u32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe {
            ffi::agpu_upsample_nearest2d_backward(self.raw, grad_out.c(), batch, channels, in_h,
                                                  in_w, scale_h, scale_w, o)
        })
    }

    // ---------------------------------------------------- LLaMA-layer ops --
    pub fn rmsnorm(&self, x: &GpuBuffer, w: &GpuBuffer, rows: u32, cols: u32, eps: f32) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_rmsnorm(self.raw, x.c(), w.c(), rows, cols, eps, o) })
    }
    pub fn rope(
        &self, x: &GpuBuffer, batch: u32, seq: u32, heads: u32, dim: u32, base: f32,
    ) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_rope(self.raw, x.c(), batch, seq, heads, dim, base, o) })
    }
    pub fn swish_mul(&self, gate: &GpuBuffer, up: &GpuBuffer) -> Result<GpuBuffer> {
        self.out(|o| unsafe { ffi::agpu_swish_mul(self.raw, gate.c(), up.c(), o) })
    }

    // -------------------------------------------------------------- AdamW --
    /// One AdamW step over many tensors in one launch (the reference's
    /// `AdamW::step`, src/optim.rs:82-138); params, m and v are updated in
    /// place; `step` counts from 1.
    #[allow(clippy::too_many_arguments)]
    pub fn adamw_step(
        &self, params: &[&GpuBuffer], grads: &[&GpuBuffer], m: &[&GpuBuffer], v: &[&GpuBuffer],
        lr: f32, beta1: f32, beta2: f32, eps: f32, weight_decay: f32, step: u32,
    ) -> Result<()> {
        let n = params.len();
        if grads.len() != n || m.len() != n || v.len() != n {
            return Err(AgpuError {
                status: ffi::AGPU_ERR_SHAPE,
                message: "adamw_step: params, grads, m and v differ in count".to_string(),
            }
            .into());
        }
        let p: Vec<*mut ffi::AgpuBuffer> = params.iter().map(|b| b.raw).collect();
        let g: Vec<*const ffi::AgpuBuffer> = grads.iter().map(|b| b.c()).collect();
        let mm: Vec<*mut ffi::AgpuBuffer> = m.iter().map(|b| b.raw).collect();
        let vv: Vec<*mut ffi::AgpuBuffer> = v.iter().map(|b| b.raw).collect();
        check(unsafe {
            ffi::agpu_adamw_step(self.raw, p.as_ptr(), g.as_ptr(), mm.as_ptr(), vv.as_ptr(),
                                 n as u32, lr, beta1, beta2, eps, weight_decay, step)
        })
    }
}
