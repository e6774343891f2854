//! Raw bindings of `include/agpu.h`, the C ABI of libagpu.so (one
//! declaration per exported function, in the header's order, same names,
//! argument order and C types).  `device.rs` wraps them in the reference
//! crate's `GpuDevice` / `GpuBuffer` API.
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_int, c_uint, c_void};

/// `agpu_status`: 0 = ok; see `AgpuError` in device.rs for the others.
pub type AgpuStatus = c_int;
pub const AGPU_OK: AgpuStatus = 0;
pub const AGPU_ERR_SHAPE: AgpuStatus = 1;
pub const AGPU_ERR_INVALID: AgpuStatus = 2;
pub const AGPU_ERR_CUDA: AgpuStatus = 3;
pub const AGPU_ERR_OOM: AgpuStatus = 4;
pub const AGPU_ERR_NO_DEVICE: AgpuStatus = 5;
pub const AGPU_ERR_TIMEOUT: AgpuStatus = 6;
pub const AGPU_ERR_UNSUPPORTED: AgpuStatus = 7;

/// `AGPU_SELFTEST_WAIT_CODE`: the status code agpu_selftest_wait_timeout records.
pub const AGPU_SELFTEST_WAIT_CODE: u32 = 0x7e57;

/// `AGPU_WAIT_FLAGS_CODE`: the status code an expired agpu_wait_flags records.
pub const AGPU_WAIT_FLAGS_CODE: u32 = 0x5157;

/// `agpu_precision`.
pub const AGPU_PREC_TF32: c_int = 0;
pub const AGPU_PREC_TF32X3: c_int = 1;
pub const AGPU_PREC_FFMA: c_int = 2;

/// Opaque `agpu_device`.
#[repr(C)]
pub struct AgpuDevice {
    _private: [u8; 0],
}

/// Opaque `agpu_buffer`.
#[repr(C)]
pub struct AgpuBuffer {
    _private: [u8; 0],
}

/// `agpu_ipc_handle`: a CUDA IPC handle of memory or of an event, as bytes.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct AgpuIpcHandle {
    pub bytes: [u8; 64],
}

/// `agpu_attn_layout`: element strides of one attention operand.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct AgpuAttnLayout {
    pub seq_stride: u64,
    pub head_stride: u64,
    pub batch_stride: u64,
}

/// `agpu_adamw_tensor`: one parameter tensor of a multi-tensor AdamW launch.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct AgpuAdamwTensor {
    pub param: *mut f32,
    pub grad: *const f32,
    pub m: *mut f32,
    pub v: *mut f32,
    pub n: u64,
}

#[link(name = "agpu")]
extern "C" {
    pub fn agpu_last_error_message() -> *const c_char;
    pub fn agpu_status_string(s: AgpuStatus) -> *const c_char;
    pub fn agpu_device_create(ordinal: c_int, out: *mut *mut AgpuDevice) -> AgpuStatus;
    pub fn agpu_device_destroy(dev: *mut AgpuDevice) -> AgpuStatus;
    pub fn agpu_device_name(
        dev: *const AgpuDevice,
        buf: *mut c_char,
        buf_len: usize,
    ) -> AgpuStatus;
    pub fn agpu_device_sm_count(dev: *const AgpuDevice, out: *mut c_int) -> AgpuStatus;
    pub fn agpu_device_ordinal(dev: *const AgpuDevice, out: *mut c_int) -> AgpuStatus;
    pub fn agpu_device_stream(dev: *const AgpuDevice) -> *mut c_void;
    pub fn agpu_synchronize(dev: *mut AgpuDevice) -> AgpuStatus;
    pub fn agpu_set_precision(dev: *mut AgpuDevice, p: c_int) -> AgpuStatus;
    pub fn agpu_get_precision(dev: *const AgpuDevice, p: *mut c_int) -> AgpuStatus;
    pub fn agpu_set_thread_precision(mode: c_int) -> AgpuStatus;
    pub fn agpu_get_thread_precision() -> c_int;
    pub fn agpu_device_launch_count(dev: *const AgpuDevice) -> u64;
    pub fn agpu_upload(
        dev: *mut AgpuDevice,
        host: *const f32,
        n: u64,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_alloc(dev: *mut AgpuDevice, n: u64, out: *mut *mut AgpuBuffer) -> AgpuStatus;
    pub fn agpu_read(
        dev: *mut AgpuDevice,
        buf: *const AgpuBuffer,
        host: *mut f32,
        n: u64,
    ) -> AgpuStatus;
    pub fn agpu_write(
        dev: *mut AgpuDevice,
        buf: *mut AgpuBuffer,
        host: *const f32,
        n: u64,
    ) -> AgpuStatus;
    pub fn agpu_write_async(
        dev: *mut AgpuDevice,
        buf: *mut AgpuBuffer,
        offset: u64,
        host: *const f32,
        n: u64,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_read_async(
        dev: *mut AgpuDevice,
        buf: *const AgpuBuffer,
        offset: u64,
        host: *mut f32,
        n: u64,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_buffer_free(buf: *mut AgpuBuffer) -> AgpuStatus;
    pub fn agpu_buffer_len(buf: *const AgpuBuffer) -> u64;
    pub fn agpu_buffer_device_ptr(buf: *const AgpuBuffer) -> *mut c_void;
    pub fn agpu_matmul(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        m: u32,
        n: u32,
        k: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_batch_matmul(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_batch_matmul_softmax(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_gemm(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        trans_a: c_int,
        trans_b: c_int,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_gemm_ex(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        bias: *const AgpuBuffer,
        resid: *const AgpuBuffer,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        trans_a: c_int,
        trans_b: c_int,
        act: c_int,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_softmax(
        dev: *mut AgpuDevice,
        x: *const AgpuBuffer,
        rows: u32,
        cols: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_conv2d(
        dev: *mut AgpuDevice,
        input: *const AgpuBuffer,
        weight: *const AgpuBuffer,
        bias: *const AgpuBuffer,
        batch: u32,
        in_c: u32,
        in_h: u32,
        in_w: u32,
        out_c: u32,
        kh: u32,
        kw: u32,
        stride_h: u32,
        stride_w: u32,
        pad_h: u32,
        pad_w: u32,
        dil_h: u32,
        dil_w: u32,
        groups: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_conv2d_group_norm_swish(
        dev: *mut AgpuDevice,
        input: *const AgpuBuffer,
        weight: *const AgpuBuffer,
        bias: *const AgpuBuffer,
        batch: u32,
        in_c: u32,
        in_h: u32,
        in_w: u32,
        out_c: u32,
        kh: u32,
        kw: u32,
        sh: u32,
        sw: u32,
        ph: u32,
        pw: u32,
        dh: u32,
        dw: u32,
        groups: u32,
        gamma: *const AgpuBuffer,
        beta: *const AgpuBuffer,
        gn_groups: u32,
        eps: f32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_conv_transpose2d(
        dev: *mut AgpuDevice,
        input: *const AgpuBuffer,
        weight: *const AgpuBuffer,
        bias: *const AgpuBuffer,
        batch: u32,
        in_c: u32,
        in_h: u32,
        in_w: u32,
        out_c: u32,
        kh: u32,
        kw: u32,
        stride_h: u32,
        stride_w: u32,
        pad_h: u32,
        pad_w: u32,
        out_pad_h: u32,
        out_pad_w: u32,
        dil_h: u32,
        dil_w: u32,
        groups: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_conv2d_grad_weight(
        dev: *mut AgpuDevice,
        input: *const AgpuBuffer,
        grad_out: *const AgpuBuffer,
        batch: u32,
        in_c: u32,
        in_h: u32,
        in_w: u32,
        out_c: u32,
        out_h: u32,
        out_w: u32,
        kh: u32,
        kw: u32,
        stride_h: u32,
        stride_w: u32,
        pad_h: u32,
        pad_w: u32,
        dil_h: u32,
        dil_w: u32,
        groups: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_conv2d_grad_bias(
        dev: *mut AgpuDevice,
        grad_out: *const AgpuBuffer,
        batch: u32,
        out_c: u32,
        out_h: u32,
        out_w: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_group_norm(
        dev: *mut AgpuDevice,
        x: *const AgpuBuffer,
        gamma: *const AgpuBuffer,
        beta: *const AgpuBuffer,
        batch: u32,
        channels: u32,
        spatial: u32,
        groups: u32,
        eps: f32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_group_norm_swish(
        dev: *mut AgpuDevice,
        x: *const AgpuBuffer,
        gamma: *const AgpuBuffer,
        beta: *const AgpuBuffer,
        batch: u32,
        channels: u32,
        spatial: u32,
        groups: u32,
        eps: f32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_group_norm_backward(
        dev: *mut AgpuDevice,
        grad_out: *const AgpuBuffer,
        input: *const AgpuBuffer,
        gamma: *const AgpuBuffer,
        batch: u32,
        channels: u32,
        spatial: u32,
        groups: u32,
        eps: f32,
        d_input: *mut *mut AgpuBuffer,
        d_gamma: *mut *mut AgpuBuffer,
        d_beta: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_scaled_dot_product_attention(
        dev: *mut AgpuDevice,
        q: *const AgpuBuffer,
        k: *const AgpuBuffer,
        v: *const AgpuBuffer,
        batch_heads: u32,
        seq_len: u32,
        d_k: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_sdpa_causal(
        dev: *mut AgpuDevice,
        q: *const AgpuBuffer,
        k: *const AgpuBuffer,
        v: *const AgpuBuffer,
        batch_heads: u32,
        seq_len: u32,
        d_k: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_sdpa_backward(
        dev: *mut AgpuDevice,
        q: *const AgpuBuffer,
        k: *const AgpuBuffer,
        v: *const AgpuBuffer,
        grad_out: *const AgpuBuffer,
        batch_heads: u32,
        seq_len: u32,
        d_k: u32,
        causal: c_int,
        d_q: *mut *mut AgpuBuffer,
        d_k_out: *mut *mut AgpuBuffer,
        d_v: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_rmsnorm(
        dev: *mut AgpuDevice,
        x: *const AgpuBuffer,
        w: *const AgpuBuffer,
        rows: u32,
        cols: u32,
        eps: f32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_rope(
        dev: *mut AgpuDevice,
        x: *const AgpuBuffer,
        batch: u32,
        seq: u32,
        heads: u32,
        dim: u32,
        base: f32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_swish_mul(
        dev: *mut AgpuDevice,
        gate: *const AgpuBuffer,
        up: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_add(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_sub(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_mul(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_relu(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_sigmoid(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_swish(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_tanh_act(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_scale(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        s: f32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_relu_backward(
        dev: *mut AgpuDevice,
        grad_out: *const AgpuBuffer,
        input: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_sigmoid_backward(
        dev: *mut AgpuDevice,
        grad_out: *const AgpuBuffer,
        output: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_swish_backward(
        dev: *mut AgpuDevice,
        grad_out: *const AgpuBuffer,
        input: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_tanh_backward(
        dev: *mut AgpuDevice,
        grad_out: *const AgpuBuffer,
        output: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_transpose(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        outer: u32,
        d0: u32,
        d1: u32,
        inner: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_add_per_col(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        rows: u32,
        cols: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_add_broadcast(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        outer: u32,
        inner: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_sum_inner(
        dev: *mut AgpuDevice,
        src: *const AgpuBuffer,
        outer: u32,
        inner: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_sum_rows(
        dev: *mut AgpuDevice,
        src: *const AgpuBuffer,
        rows: u32,
        cols: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_concat(
        dev: *mut AgpuDevice,
        a: *const AgpuBuffer,
        b: *const AgpuBuffer,
        outer: u32,
        a_inner: u32,
        b_inner: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_slice_per_block(
        dev: *mut AgpuDevice,
        src: *const AgpuBuffer,
        outer: u32,
        slice_size: u32,
        slice_offset: u32,
        combined: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_upsample_nearest2d(
        dev: *mut AgpuDevice,
        input: *const AgpuBuffer,
        batch: u32,
        channels: u32,
        in_h: u32,
        in_w: u32,
        scale_h: u32,
        scale_w: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_upsample_nearest2d_backward(
        dev: *mut AgpuDevice,
        grad_out: *const AgpuBuffer,
        batch: u32,
        channels: u32,
        in_h: u32,
        in_w: u32,
        scale_h: u32,
        scale_w: u32,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_mse_loss(
        dev: *mut AgpuDevice,
        pred: *const AgpuBuffer,
        target: *const AgpuBuffer,
        out: *mut *mut AgpuBuffer,
    ) -> AgpuStatus;
    pub fn agpu_adamw_step(
        dev: *mut AgpuDevice,
        params: *const *mut AgpuBuffer,
        grads: *const *const AgpuBuffer,
        m: *const *mut AgpuBuffer,
        v: *const *mut AgpuBuffer,
        count: u32,
        lr: f32,
        beta1: f32,
        beta2: f32,
        eps: f32,
        weight_decay: f32,
        step: u32,
    ) -> AgpuStatus;
    pub fn agpu_launch_adamw(
        dev: *mut AgpuDevice,
        tensors: *const AgpuAdamwTensor,
        count: u32,
        lr: f32,
        beta1: f32,
        beta2: f32,
        eps: f32,
        weight_decay: f32,
        step: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_batch_matmul(
        dev: *mut AgpuDevice,
        a: *const f32,
        b: *const f32,
        c: *mut f32,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_batch_matmul_softmax(
        dev: *mut AgpuDevice,
        a: *const f32,
        b: *const f32,
        out: *mut f32,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_gemm(
        dev: *mut AgpuDevice,
        a: *const f32,
        b: *const f32,
        c: *mut f32,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        trans_a: c_int,
        trans_b: c_int,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_conv2d(
        dev: *mut AgpuDevice,
        input: *const f32,
        weight: *const f32,
        bias: *const f32,
        out: *mut f32,
        batch: u32,
        in_c: u32,
        in_h: u32,
        in_w: u32,
        out_c: u32,
        kh: u32,
        kw: u32,
        stride_h: u32,
        stride_w: u32,
        pad_h: u32,
        pad_w: u32,
        dil_h: u32,
        dil_w: u32,
        groups: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_conv2d_group_norm_swish(
        dev: *mut AgpuDevice,
        input: *const f32,
        weight: *const f32,
        bias: *const f32,
        out: *mut f32,
        batch: u32,
        in_c: u32,
        in_h: u32,
        in_w: u32,
        out_c: u32,
        kh: u32,
        kw: u32,
        sh: u32,
        sw: u32,
        ph: u32,
        pw: u32,
        dh: u32,
        dw: u32,
        groups: u32,
        gamma: *const f32,
        beta: *const f32,
        gn_groups: u32,
        eps: f32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_group_norm(
        dev: *mut AgpuDevice,
        x: *const f32,
        gamma: *const f32,
        beta: *const f32,
        y: *mut f32,
        batch: u32,
        channels: u32,
        spatial: u32,
        groups: u32,
        eps: f32,
        apply_swish: c_int,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_group_norm_backward(
        dev: *mut AgpuDevice,
        grad_out: *const f32,
        input: *const f32,
        gamma: *const f32,
        d_input: *mut f32,
        d_gamma: *mut f32,
        d_beta: *mut f32,
        batch: u32,
        channels: u32,
        spatial: u32,
        groups: u32,
        eps: f32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_sdpa(
        dev: *mut AgpuDevice,
        q: *const f32,
        k: *const f32,
        v: *const f32,
        out: *mut f32,
        batch_heads: u32,
        seq_len: u32,
        d_k: u32,
        causal: c_int,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_sdpa_backward(
        dev: *mut AgpuDevice,
        q: *const f32,
        k: *const f32,
        v: *const f32,
        grad_out: *const f32,
        d_q: *mut f32,
        d_k: *mut f32,
        d_v: *mut f32,
        batch_heads: u32,
        seq_len: u32,
        d_k_dim: u32,
        causal: c_int,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_gemm_ex(
        dev: *mut AgpuDevice,
        a: *const f32,
        b: *const f32,
        c: *mut f32,
        batch: u32,
        m: u32,
        n: u32,
        k: u32,
        trans_a: c_int,
        trans_b: c_int,
        bias: *const f32,
        resid: *const f32,
        act: c_int,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_sdpa_strided(
        dev: *mut AgpuDevice,
        q: *const f32,
        k: *const f32,
        v: *const f32,
        out: *mut f32,
        batch: u32,
        heads: u32,
        seq_len: u32,
        d_k: u32,
        q_layout: *const AgpuAttnLayout,
        k_layout: *const AgpuAttnLayout,
        v_layout: *const AgpuAttnLayout,
        out_layout: *const AgpuAttnLayout,
        causal: c_int,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_rmsnorm(
        dev: *mut AgpuDevice,
        x: *const f32,
        w: *const f32,
        y: *mut f32,
        rows: u64,
        cols: u32,
        eps: f32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_rope(
        dev: *mut AgpuDevice,
        x: *const f32,
        y: *mut f32,
        batch: u32,
        seq: u32,
        heads: u32,
        dim: u32,
        row_stride: u64,
        base: f32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_swish_mul(
        dev: *mut AgpuDevice,
        gate: *const f32,
        up: *const f32,
        out: *mut f32,
        rows: u64,
        cols: u32,
        gate_stride: u64,
        up_stride: u64,
        out_stride: u64,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_launch_softmax(
        dev: *mut AgpuDevice,
        x: *const f32,
        y: *mut f32,
        rows: u64,
        cols: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_group_norm_noalloc(
        x: *const f32,
        gamma: *const f32,
        beta: *const f32,
        y: *mut f32,
        batch: u32,
        channels: u32,
        spatial: u32,
        groups: u32,
        eps: f32,
        apply_swish: c_int,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_ipc_export(
        dev: *mut AgpuDevice,
        dptr: *const c_void,
        handle: *mut AgpuIpcHandle,
        offset: *mut u64,
    ) -> AgpuStatus;
    pub fn agpu_ipc_import(
        dev: *mut AgpuDevice,
        handle: *const AgpuIpcHandle,
        base: *mut *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_ipc_close(dev: *mut AgpuDevice, base: *mut c_void) -> AgpuStatus;
    pub fn agpu_ipc_event_create(
        dev: *mut AgpuDevice,
        event: *mut *mut c_void,
        handle: *mut AgpuIpcHandle,
    ) -> AgpuStatus;
    pub fn agpu_ipc_event_import(
        dev: *mut AgpuDevice,
        handle: *const AgpuIpcHandle,
        event: *mut *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_event_destroy(dev: *mut AgpuDevice, event: *mut c_void) -> AgpuStatus;
    pub fn agpu_event_record(
        dev: *mut AgpuDevice,
        event: *mut c_void,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_stream_wait_event(
        dev: *mut AgpuDevice,
        stream: *mut c_void,
        event: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_copy_async(
        dev: *mut AgpuDevice,
        dst: *mut c_void,
        src: *const c_void,
        bytes: u64,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_signal_peers(
        dev: *mut AgpuDevice,
        peer_flags: *const *mut c_uint,
        count: u32,
        value: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_wait_flags(
        dev: *mut AgpuDevice,
        flags: *const c_uint,
        count: u32,
        target: u32,
        limit_us: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
    pub fn agpu_selftest_wait_timeout(
        dev: *mut AgpuDevice,
        limit_us: u32,
        stream: *mut c_void,
    ) -> AgpuStatus;
}
