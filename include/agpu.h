/*
 * agpu.h -- C ABI of the B200-native dense-op library that replaces the
 * hot path of any-gpu's `GpuDevice` (reference crate `any_gpu`, Rust + WGSL).
 *
 * Every entry point is plain C: opaque handles, raw pointers, 64-bit sizes,
 * an `agpu_status` return code.  No CUDA, torch or C++ types cross it, so a
 * Rust `extern "C"` block, ctypes, JNI or cgo can bind it unchanged.
 *
 * Two layers:
 *   1. Buffer layer (mirrors `GpuDevice`): ops take `agpu_buffer*` inputs and
 *      return a freshly allocated output buffer owned by the caller, exactly
 *      like the reference's `fn op(&self, ...) -> Result<GpuBuffer>`.
 *      Size mismatches return AGPU_ERR_SHAPE before anything is launched,
 *      where the reference returns `Err` from `ensure!`.
 *   2. Launch layer (`agpu_launch_*`): the same kernels on caller-owned
 *      device memory and a caller-chosen CUDA stream (passed as `void*`),
 *      for frameworks that manage their own memory (torch, NCCL buffers).
 *
 * Ordering: every op of a device is enqueued on that device's stream in call
 * order; `agpu_read` and `agpu_synchronize` block until the stream drains.
 * Inputs are only read; outputs never alias inputs.
 * All element counts are 64-bit, so no `u32` wraparound at BH*S*S >= 2^32.
 *
 * Kernel-choice switches, read once per process from the environment (all
 * on by default; results stay within the documented tolerances either way):
 *   AGPU_GEMM_PAIR=0      TF32 GEMMs on single-CTA 128-row tiles, not CTA pairs
 *   AGPU_GEMM_SPLITK=0    no cluster split-K for GEMMs with few tiles
 *                         (=256: split-K on 256 x 256 tiles only, not 256 x 128)
 *   AGPU_GEMM_WIDE=0|2    never / always 256 x 512 pair tiles (default: estimate)
 *   AGPU_GEMM_CHUNKED=0   MN-major operands by one TMA box per 32 columns
 *                         (bit-identical output)
 *   AGPU_SDPA_PAIR=0      attention on single CTAs for every sequence length
 *   AGPU_CONV_WIDE=0      conv2d on 256 x 160 tiles instead of 256 x 320
 *   AGPU_CONV_OVERLAP=0   conv2d staging and conv in one stream (no halves)
 *   AGPU_BMM_SOFTMAX_PIECES=N  at most N pieces (1, 2, 4, 8) in the fused
 *                         batch_matmul + softmax pipeline
 *   AGPU_X3_SEG=N         3xTF32 on CTA pairs: K-blocks (of 32) per accumulator
 *                         segment (default 16; 0 = none: faster, less accurate)
 *   AGPU_SDPA_BWD_FUSED=0 attention backward with the two row passes over the
 *                         [heads, S, S] matrices instead of the forward rerun
 *                         and the GEMM epilogues that form P and dS
 *   AGPU_GEMM_TMA_STORE=0 GEMM outputs by the warp-transposing float4 store
 *                         instead of TMA bulk tensor stores (bit-identical)
 */
#ifndef AGPU_H
#define AGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define AGPU_API __attribute__((visibility("default")))
#else
#define AGPU_API
#endif

typedef enum agpu_status {
  AGPU_OK = 0,
  AGPU_ERR_SHAPE = 1,       /* buffer length / dimension mismatch (reference: ensure!) */
  AGPU_ERR_INVALID = 2,     /* null handle, zero dimension, bad enum value            */
  AGPU_ERR_CUDA = 3,        /* CUDA runtime / launch error                             */
  AGPU_ERR_OOM = 4,         /* device memory pool exhausted                            */
  AGPU_ERR_NO_DEVICE = 5,   /* no CUDA device with that ordinal                        */
  AGPU_ERR_TIMEOUT = 6,     /* a bounded device-side wait expired; results invalid     */
  AGPU_ERR_UNSUPPORTED = 7  /* shape/option combination this build does not handle     */
} agpu_status;

/* Arithmetic used by the contractions (matmul, batch_matmul, sdpa, conv2d). */
typedef enum agpu_precision {
  AGPU_PREC_TF32 = 0,   /* tcgen05 kind::tf32, fp32 accumulate (default)            */
  AGPU_PREC_TF32X3 = 1, /* error-corrected 3xTF32 on tcgen05: fp32-level accuracy   */
  AGPU_PREC_FFMA = 2    /* SIMT fp32 FFMA (exact fp32 products, slow)               */
} agpu_precision;

typedef struct agpu_device agpu_device;
typedef struct agpu_buffer agpu_buffer;

/* ---------------------------------------------------------------- errors -- */
/* Message of the last failing call on this thread ("" if none).
 * Replaces the anyhow::Error text of the reference. */
AGPU_API const char* agpu_last_error_message(void);
AGPU_API const char* agpu_status_string(agpu_status s);

/* ---------------------------------------------------------------- device -- */
/* Replaces GpuDevice::gpu() (src/device.rs:31-78): binds CUDA device
 * `ordinal`, creates its stream and a stream-ordered memory pool. */
AGPU_API agpu_status agpu_device_create(int ordinal, agpu_device** out);
/* Releases the handle.  Buffers still alive keep the device's stream and
 * memory valid until they are freed (like GpuBuffer holding its device). */
AGPU_API agpu_status agpu_device_destroy(agpu_device* dev);
/* Replaces the `adapter_name` / `backend` fields (src/device.rs:15-16). */
AGPU_API agpu_status agpu_device_name(const agpu_device* dev, char* buf, size_t buf_len);
AGPU_API agpu_status agpu_device_sm_count(const agpu_device* dev, int* out);
AGPU_API agpu_status agpu_device_ordinal(const agpu_device* dev, int* out);
/* The device's CUDA stream as an opaque cudaStream_t. */
AGPU_API void* agpu_device_stream(const agpu_device* dev);
AGPU_API agpu_status agpu_synchronize(agpu_device* dev);
/* Device-wide default arithmetic of the contractions (initially TF32). */
AGPU_API agpu_status agpu_set_precision(agpu_device* dev, agpu_precision p);
AGPU_API agpu_status agpu_get_precision(const agpu_device* dev, agpu_precision* p);
/* Per-call precision without touching the shared device: every contraction
 * this host thread enqueues after the call, on any device, uses `mode`
 * (an agpu_precision) until the thread sets -1 again, which returns it to
 * each device's own setting.  Other threads are unaffected.  No counterpart
 * in the reference (its shaders have one arithmetic). */
AGPU_API agpu_status agpu_set_thread_precision(int mode);
AGPU_API int agpu_get_thread_precision(void);
/* Number of this library's kernels launched on `dev` since creation. */
AGPU_API uint64_t agpu_device_launch_count(const agpu_device* dev);

/* --------------------------------------------------------------- buffers -- */
/* Replaces GpuDevice::upload (src/device.rs:80-94): H2D copy of n f32. */
AGPU_API agpu_status agpu_upload(agpu_device* dev, const float* host, uint64_t n,
                                 agpu_buffer** out);
/* Replaces GpuDevice::alloc (src/device.rs:97-112).  Zero-filled, as the
 * reference's wgpu buffers are (the fill is ordered on the device stream). */
AGPU_API agpu_status agpu_alloc(agpu_device* dev, uint64_t n, agpu_buffer** out);
/* Replaces GpuDevice::read (src/device.rs:115-145): blocking D2H of the
 * whole buffer; `n` must equal the buffer length. */
AGPU_API agpu_status agpu_read(agpu_device* dev, const agpu_buffer* buf, float* host,
                               uint64_t n);
/* Stream-ordered H2D into an existing buffer (no new allocation). */
AGPU_API agpu_status agpu_write(agpu_device* dev, agpu_buffer* buf, const float* host,
                                uint64_t n);
/* Stream-ordered partial copies, for hosts that overlap PCIe transfers in
 * both directions with compute on other streams (the reference's upload and
 * read are synchronous).  Copies `n` floats between `host` and elements
 * [offset, offset + n) of `buf` on `stream` (NULL = the device stream) and
 * returns without waiting; `host` must stay valid and unchanged until the
 * stream reaches the copy (page-locked memory makes the copy asynchronous).
 * offset + n > buffer length -> AGPU_ERR_SHAPE.  Expired device waits are
 * reported by the next agpu_read / agpu_synchronize. */
AGPU_API agpu_status agpu_write_async(agpu_device* dev, agpu_buffer* buf, uint64_t offset,
                                      const float* host, uint64_t n, void* stream);
AGPU_API agpu_status agpu_read_async(agpu_device* dev, const agpu_buffer* buf, uint64_t offset,
                                     float* host, uint64_t n, void* stream);
/* Replaces Drop for GpuBuffer: returns memory to the device pool, ordered
 * on the device stream.  Work that uses the buffer on another stream
 * (agpu_read_async / agpu_write_async / a launch-layer call given its
 * address) must have been reached by that stream first: synchronise the
 * stream, or make the device stream wait on it, before freeing. */
AGPU_API agpu_status agpu_buffer_free(agpu_buffer* buf);
/* GpuBuffer::len (src/device.rs:25). */
AGPU_API uint64_t agpu_buffer_len(const agpu_buffer* buf);
/* Device address of the buffer's first element (for interop). */
AGPU_API void* agpu_buffer_device_ptr(const agpu_buffer* buf);

/* ------------------------------------------------------ contractions ------ */
/* GpuDevice::matmul(a, b, m, n, k) (src/ops/conv.rs:416-423).
 * C[m,n] = A[m,k] * B[k,n], row-major.  Argument order is the code's (m,n,k). */
AGPU_API agpu_status agpu_matmul(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                                 uint32_t m, uint32_t n, uint32_t k, agpu_buffer** out);
/* GpuDevice::batch_matmul (src/ops/conv.rs:426-433). C[b] = A[b] * B[b]. */
AGPU_API agpu_status agpu_batch_matmul(agpu_device* dev, const agpu_buffer* a,
                                       const agpu_buffer* b, uint32_t batch, uint32_t m,
                                       uint32_t n, uint32_t k, agpu_buffer** out);

/* batch_matmul followed by a row softmax over the last dim of the result (the
 * batch_matmul + softmax workload), in one call and one output buffer: the
 * softmax runs in place on the product.  Same shape checks as batch_matmul.
 * A large batch runs in pieces whose softmaxes overlap the next pieces'
 * GEMMs (see agpu_launch_batch_matmul_softmax). */
AGPU_API agpu_status agpu_batch_matmul_softmax(agpu_device* dev, const agpu_buffer* a,
                                               const agpu_buffer* b, uint32_t batch, uint32_t m,
                                               uint32_t n, uint32_t k, agpu_buffer** out);

/* General (batched) GEMM with optional transposed operands, the kernels the
 * reference's autograd backward reaches through transpose + matmul
 * (src/autograd.rs:357-366): dA = dC * B^T (trans_b), dB = A^T * dC (trans_a).
 * trans_a = 0: A stored [batch, m, k]; 1: A stored [batch, k, m].
 * trans_b = 0: B stored [batch, k, n]; 1: B stored [batch, n, k].
 * C is always [batch, m, n] row-major. */
AGPU_API agpu_status agpu_gemm(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                               uint32_t batch, uint32_t m, uint32_t n, uint32_t k, int trans_a,
                               int trans_b, agpu_buffer** out);

/* gemm with a fused epilogue: C = act(op(A) op(B) + bias[col] + resid), act
 * 0 = none, 1 = swish, 2 = relu; bias ([n]) and resid ([batch, m, n]) may be
 * NULL.  The bias term is the reference's Linear bias add_per_col
 * (src/ops/tensor_ops.rs:336-352) and swish its activation
 * (src/ops/elementwise.rs:77-89), applied while the tile is in registers.
 * act 3 = SwiGLU: B's n columns come in 32-column blocks, gate block j =
 * columns [64j, 64j+32) and up block j = [64j+32, 64j+64); C is
 * [batch, m, n/2] with C[.., 32j+i] = swish(gate_i) * up_i; n % 64 == 0 and
 * no bias or residual, else AGPU_ERR_SHAPE. */
AGPU_API agpu_status agpu_gemm_ex(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                                  const agpu_buffer* bias, const agpu_buffer* resid,
                                  uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                                  int trans_a, int trans_b, int act, agpu_buffer** out);

/* ----------------------------------------------------------- attention ---- */
/* GpuDevice::softmax (src/ops/attention.rs:91-145): row softmax of [rows, cols]. */
AGPU_API agpu_status agpu_softmax(agpu_device* dev, const agpu_buffer* x, uint32_t rows,
                                  uint32_t cols, agpu_buffer** out);

/* ------------------------------------------------------------- conv2d ----- */
/* GpuDevice::conv2d (src/ops/conv.rs:437-480): input [batch, in_c, in_h, in_w],
 * weight [out_c, in_c/groups, kh, kw], bias [out_c] or NULL (zeros), NCHW.
 * out [batch, out_c, out_h, out_w], out = (in + 2*pad - dil*(k-1) - 1)/stride + 1.
 * The reference's (stride, padding, dilation) tuples are passed as (h, w) pairs. */
AGPU_API agpu_status agpu_conv2d(agpu_device* dev, const agpu_buffer* input,
                                 const agpu_buffer* weight, const agpu_buffer* bias,
                                 uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w,
                                 uint32_t out_c, uint32_t kh, uint32_t kw, uint32_t stride_h,
                                 uint32_t stride_w, uint32_t pad_h, uint32_t pad_w,
                                 uint32_t dil_h, uint32_t dil_w, uint32_t groups,
                                 agpu_buffer** out);
/* conv2d -> group_norm -> swish (the UNet block) in one call:
 * out = swish(group_norm(conv2d(input, weight, bias, ...), gamma, beta,
 * gn_groups, eps)).  Arguments and shape checks as agpu_conv2d and
 * agpu_group_norm_swish (out_c % gn_groups != 0 -> AGPU_ERR_SHAPE).  With
 * several images the batch runs in two halves on two streams and the group
 * norm of one half overlaps the conv of the other. */
AGPU_API agpu_status agpu_conv2d_group_norm_swish(
    agpu_device* dev, const agpu_buffer* input, const agpu_buffer* weight,
    const agpu_buffer* bias, uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w,
    uint32_t out_c, uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ph, uint32_t pw,
    uint32_t dh, uint32_t dw, uint32_t groups, const agpu_buffer* gamma, const agpu_buffer* beta,
    uint32_t gn_groups, float eps, agpu_buffer** out);
/* GpuDevice::conv_transpose2d (src/ops/conv.rs:484-530): weight
 * [in_c, out_c/groups, kh, kw]; out = (in-1)*stride - 2*pad + dil*(k-1) + out_pad + 1. */
AGPU_API agpu_status agpu_conv_transpose2d(agpu_device* dev, const agpu_buffer* input,
                                           const agpu_buffer* weight, const agpu_buffer* bias,
                                           uint32_t batch, uint32_t in_c, uint32_t in_h,
                                           uint32_t in_w, uint32_t out_c, uint32_t kh, uint32_t kw,
                                           uint32_t stride_h, uint32_t stride_w, uint32_t pad_h,
                                           uint32_t pad_w, uint32_t out_pad_h, uint32_t out_pad_w,
                                           uint32_t dil_h, uint32_t dil_w, uint32_t groups,
                                           agpu_buffer** out);
/* GpuDevice::conv2d_grad_weight (src/ops/conv.rs:531-549, used by the autograd
 * conv backward src/autograd.rs:376-427): dW [out_c, in_c/groups, kh, kw]. */
AGPU_API agpu_status agpu_conv2d_grad_weight(agpu_device* dev, const agpu_buffer* input,
                                             const agpu_buffer* grad_out, uint32_t batch,
                                             uint32_t in_c, uint32_t in_h, uint32_t in_w,
                                             uint32_t out_c, uint32_t out_h, uint32_t out_w,
                                             uint32_t kh, uint32_t kw, uint32_t stride_h,
                                             uint32_t stride_w, uint32_t pad_h, uint32_t pad_w,
                                             uint32_t dil_h, uint32_t dil_w, uint32_t groups,
                                             agpu_buffer** out);
/* GpuDevice::conv2d_grad_bias (src/ops/conv.rs:551-563): db [out_c]. */
AGPU_API agpu_status agpu_conv2d_grad_bias(agpu_device* dev, const agpu_buffer* grad_out,
                                           uint32_t batch, uint32_t out_c, uint32_t out_h,
                                           uint32_t out_w, agpu_buffer** out);

/* ------------------------------------------------------------ group norm -- */
/* GpuDevice::group_norm (src/ops/norm.rs:210-278): x [batch, channels, spatial]
 * in `groups` groups of channels/groups channels; y = (x-mean)/sqrt(var+eps) *
 * gamma[c] + beta[c].  channels % groups != 0 -> AGPU_ERR_SHAPE. */
AGPU_API agpu_status agpu_group_norm(agpu_device* dev, const agpu_buffer* x,
                                     const agpu_buffer* gamma, const agpu_buffer* beta,
                                     uint32_t batch, uint32_t channels, uint32_t spatial,
                                     uint32_t groups, float eps, agpu_buffer** out);
/* group_norm followed by swish in one pass (the UNet block's GN -> swish,
 * src/ops/norm.rs:210 then src/ops/elementwise.rs:211). */
AGPU_API agpu_status agpu_group_norm_swish(agpu_device* dev, const agpu_buffer* x,
                                           const agpu_buffer* gamma, const agpu_buffer* beta,
                                           uint32_t batch, uint32_t channels, uint32_t spatial,
                                           uint32_t groups, float eps, agpu_buffer** out);

/* GpuDevice::group_norm_backward (src/ops/norm.rs:282-438): gradients of
 * group_norm with respect to its input, gamma and beta, statistics recomputed
 * from `input`.  d_input [batch, channels, spatial], d_gamma and d_beta
 * [channels] are new buffers.  Size mismatches and channels % groups != 0
 * -> AGPU_ERR_SHAPE (src/ops/norm.rs:291-294). */
AGPU_API agpu_status agpu_group_norm_backward(agpu_device* dev, const agpu_buffer* grad_out,
                                              const agpu_buffer* input, const agpu_buffer* gamma,
                                              uint32_t batch, uint32_t channels,
                                              uint32_t spatial, uint32_t groups, float eps,
                                              agpu_buffer** d_input, agpu_buffer** d_gamma,
                                              agpu_buffer** d_beta);

/* ------------------------------------------------------------- sdpa ------- */
/* GpuDevice::scaled_dot_product_attention (src/ops/attention.rs:149-169):
 * softmax(Q K^T / sqrt(d_k)) V per head, non-causal; Q, K, V, out are
 * [batch_heads, seq_len, d_k].  One fused kernel: no [bh, S, S] scores in HBM. */
AGPU_API agpu_status agpu_scaled_dot_product_attention(agpu_device* dev, const agpu_buffer* q,
                                                       const agpu_buffer* k,
                                                       const agpu_buffer* v, uint32_t batch_heads,
                                                       uint32_t seq_len, uint32_t d_k,
                                                       agpu_buffer** out);
/* Causal variant (query i attends keys j <= i).  No counterpart in the
 * reference; the LLaMA-style layer of the benchmark configs uses it. */
AGPU_API agpu_status agpu_sdpa_causal(agpu_device* dev, const agpu_buffer* q,
                                      const agpu_buffer* k, const agpu_buffer* v,
                                      uint32_t batch_heads, uint32_t seq_len, uint32_t d_k,
                                      agpu_buffer** out);

/* Gradients of attention: dQ, dK, dV (new buffers, [batch_heads, seq_len,
 * d_k]) from dO = grad_out, for the non-causal (causal = 0) or causal
 * forward.  No counterpart in the reference (its tape has no attention
 * node); the result is its SDPA composition (src/ops/attention.rs:149-169)
 * differentiated with its own matmul rule (src/autograd.rs:357-366), the
 * scale rule and the softmax Jacobian: P = softmax(Q K^T / sqrt(d_k)) is
 * recomputed, dV = P^T dO, dS = P o (dO V^T - rowsum(P o dO V^T)) / sqrt(d_k),
 * dQ = dS K, dK = dS^T Q.  The products run on the tensor-core GEMMs in the
 * current precision mode.  In TF32 with seq_len >= 256 and d_k 64 or 128 the
 * forward is rerun for each row's log-sum-exp and O, P is formed in the
 * S product's epilogue and dS in the dP product's, in place: pool scratch of
 * min(batch_heads, 2^30 / seq_len^2) x seq_len^2 floats plus O; otherwise P
 * and dS take twice that.  Shape checks as the forward. */
AGPU_API agpu_status agpu_sdpa_backward(agpu_device* dev, const agpu_buffer* q,
                                        const agpu_buffer* k, const agpu_buffer* v,
                                        const agpu_buffer* grad_out, uint32_t batch_heads,
                                        uint32_t seq_len, uint32_t d_k, int causal,
                                        agpu_buffer** d_q, agpu_buffer** d_k_out,
                                        agpu_buffer** d_v);

/* ------------------------------------------------- LLaMA-layer ops -------- */
/* No counterparts in the reference (its ops have no RMSNorm or RoPE); they
 * complete the decoder layer of the benchmark configs from the ops above. */
/* RMSNorm over rows of `cols`: y = x / sqrt(mean(x^2) + eps) * w[col]. */
AGPU_API agpu_status agpu_rmsnorm(agpu_device* dev, const agpu_buffer* x, const agpu_buffer* w,
                                  uint32_t rows, uint32_t cols, float eps, agpu_buffer** out);
/* Rotary embedding (rotate-half) of x [batch, seq, heads, dim], position =
 * seq index, angle = pos * base^(-2i/dim). */
AGPU_API agpu_status agpu_rope(agpu_device* dev, const agpu_buffer* x, uint32_t batch,
                               uint32_t seq, uint32_t heads, uint32_t dim, float base,
                               agpu_buffer** out);
/* SwiGLU product swish(gate) * up, one pass (the reference composes
 * swish, src/ops/elementwise.rs:211, and mul, :198). Equal lengths. */
AGPU_API agpu_status agpu_swish_mul(agpu_device* dev, const agpu_buffer* gate,
                                    const agpu_buffer* up, agpu_buffer** out);

/* --------------------------------------------------------- elementwise ---- */
/* src/ops/elementwise.rs:188-250.  Binary ops require equal lengths. */
AGPU_API agpu_status agpu_add(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                              agpu_buffer** out);
AGPU_API agpu_status agpu_sub(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                              agpu_buffer** out);
AGPU_API agpu_status agpu_mul(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                              agpu_buffer** out);
AGPU_API agpu_status agpu_relu(agpu_device* dev, const agpu_buffer* a, agpu_buffer** out);
AGPU_API agpu_status agpu_sigmoid(agpu_device* dev, const agpu_buffer* a, agpu_buffer** out);
AGPU_API agpu_status agpu_swish(agpu_device* dev, const agpu_buffer* a, agpu_buffer** out);
AGPU_API agpu_status agpu_tanh_act(agpu_device* dev, const agpu_buffer* a, agpu_buffer** out);
AGPU_API agpu_status agpu_scale(agpu_device* dev, const agpu_buffer* a, float s,
                                agpu_buffer** out);
/* Activation backward (src/ops/elementwise.rs:229-250). */
AGPU_API agpu_status agpu_relu_backward(agpu_device* dev, const agpu_buffer* grad_out,
                                        const agpu_buffer* input, agpu_buffer** out);
AGPU_API agpu_status agpu_sigmoid_backward(agpu_device* dev, const agpu_buffer* grad_out,
                                           const agpu_buffer* output, agpu_buffer** out);
AGPU_API agpu_status agpu_swish_backward(agpu_device* dev, const agpu_buffer* grad_out,
                                         const agpu_buffer* input, agpu_buffer** out);
AGPU_API agpu_status agpu_tanh_backward(agpu_device* dev, const agpu_buffer* grad_out,
                                        const agpu_buffer* output, agpu_buffer** out);

/* ----------------------------------------------------------- tensor ops --- */
/* GpuDevice::transpose (src/ops/tensor_ops.rs:251-269): [outer,d0,d1,inner] ->
 * [outer,d1,d0,inner]. */
AGPU_API agpu_status agpu_transpose(agpu_device* dev, const agpu_buffer* a, uint32_t outer,
                                    uint32_t d0, uint32_t d1, uint32_t inner,
                                    agpu_buffer** out);
/* GpuDevice::add_per_col (src/ops/tensor_ops.rs:336-352): out[r,c] = a[r,c] + b[c]. */
AGPU_API agpu_status agpu_add_per_col(agpu_device* dev, const agpu_buffer* a,
                                      const agpu_buffer* b, uint32_t rows, uint32_t cols,
                                      agpu_buffer** out);
/* GpuDevice::add_broadcast (src/ops/tensor_ops.rs:298-315): out[o,i] = a[o,i] + b[o]. */
AGPU_API agpu_status agpu_add_broadcast(agpu_device* dev, const agpu_buffer* a,
                                        const agpu_buffer* b, uint32_t outer, uint32_t inner,
                                        agpu_buffer** out);
/* GpuDevice::sum_inner (src/ops/tensor_ops.rs:318-333, the AddBroadcast backward):
 * out[o] = sum_i src[o,i]. */
AGPU_API agpu_status agpu_sum_inner(agpu_device* dev, const agpu_buffer* src, uint32_t outer,
                                    uint32_t inner, agpu_buffer** out);
/* GpuDevice::sum_rows (src/ops/tensor_ops.rs:356-372, the AddPerCol backward):
 * out[c] = sum_r src[r,c]. */
AGPU_API agpu_status agpu_sum_rows(agpu_device* dev, const agpu_buffer* src, uint32_t rows,
                                   uint32_t cols, agpu_buffer** out);
/* GpuDevice::concat (src/ops/tensor_ops.rs:229-245): [outer,a_inner] ++ [outer,b_inner]
 * -> [outer, a_inner+b_inner]. */
AGPU_API agpu_status agpu_concat(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                                 uint32_t outer, uint32_t a_inner, uint32_t b_inner,
                                 agpu_buffer** out);
/* GpuDevice::slice_per_block (src/ops/tensor_ops.rs:274-294, the Concat backward):
 * [outer, combined] -> [outer, slice_size] from column slice_offset;
 * slice_offset + slice_size > combined -> AGPU_ERR_SHAPE. */
AGPU_API agpu_status agpu_slice_per_block(agpu_device* dev, const agpu_buffer* src,
                                          uint32_t outer, uint32_t slice_size,
                                          uint32_t slice_offset, uint32_t combined,
                                          agpu_buffer** out);
/* GpuDevice::upsample_nearest2d (src/ops/upsample.rs:94-113): NCHW [N,C,H,W] ->
 * [N,C,H*scale_h,W*scale_w]. */
AGPU_API agpu_status agpu_upsample_nearest2d(agpu_device* dev, const agpu_buffer* input,
                                             uint32_t batch, uint32_t channels, uint32_t in_h,
                                             uint32_t in_w, uint32_t scale_h, uint32_t scale_w,
                                             agpu_buffer** out);
/* GpuDevice::upsample_nearest2d_backward (src/ops/upsample.rs:116-137): each input pixel
 * sums its scale_h x scale_w output block. */
AGPU_API agpu_status agpu_upsample_nearest2d_backward(agpu_device* dev,
                                                      const agpu_buffer* grad_out,
                                                      uint32_t batch, uint32_t channels,
                                                      uint32_t in_h, uint32_t in_w,
                                                      uint32_t scale_h, uint32_t scale_w,
                                                      agpu_buffer** out);
/* GpuDevice::mse_loss (src/ops/attention.rs:171-182): 1-element mean((pred-target)^2);
 * pred.len != target.len -> AGPU_ERR_SHAPE. */
AGPU_API agpu_status agpu_mse_loss(agpu_device* dev, const agpu_buffer* pred,
                                   const agpu_buffer* target, agpu_buffer** out);

/* ---------------------------------------------------------------- AdamW -- */
/* One AdamW step (the reference's AdamW::step, src/optim.rs:82-138, and its
 * shader :22-51) for `count` parameter tensors in one launch:
 *   m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2
 *   p = p (1 - lr wd) - lr (m / (1 - b1^t)) / (sqrt(v / (1 - b2^t)) + eps)
 * with t = `step` (>= 1; the reference increments its counter before the
 * update).  params, m, v are updated in place; m and v start at zero.  A
 * param/grad/m/v length mismatch -> AGPU_ERR_SHAPE (src/optim.rs:95). */
AGPU_API agpu_status agpu_adamw_step(agpu_device* dev, agpu_buffer* const* params,
                                     const agpu_buffer* const* grads, agpu_buffer* const* m,
                                     agpu_buffer* const* v, uint32_t count, float lr,
                                     float beta1, float beta2, float eps, float weight_decay,
                                     uint32_t step);
/* The same on caller-owned device memory: a host array of tensors. */
typedef struct agpu_adamw_tensor {
  float* param;
  const float* grad;
  float* m;
  float* v;
  uint64_t n;
} agpu_adamw_tensor;
AGPU_API agpu_status agpu_launch_adamw(agpu_device* dev, const agpu_adamw_tensor* tensors,
                                       uint32_t count, float lr, float beta1, float beta2,
                                       float eps, float weight_decay, uint32_t step,
                                       void* stream);

/* ------------------------------------------------ launch layer (raw ptrs) -- */
/* Same kernels on caller-owned device memory; `stream` is a cudaStream_t
 * (NULL = the device's own stream).  No allocation happens in these calls
 * unless stated.  Shapes are validated; pointers are trusted. */
AGPU_API agpu_status agpu_launch_batch_matmul(agpu_device* dev, const float* a, const float* b,
                                              float* c, uint32_t batch, uint32_t m, uint32_t n,
                                              uint32_t k, void* stream);
/* Launch-layer agpu_batch_matmul_softmax: out = softmax(A * B) row-wise, on
 * `stream`; the GEMM writes `out` and the softmax runs on it in place.  With
 * a large batch the pieces' GEMMs run back to back on `stream` and each
 * piece's softmax on a second stream beside the next GEMM; `stream` waits
 * for all of it before the call's later work. */
AGPU_API agpu_status agpu_launch_batch_matmul_softmax(agpu_device* dev, const float* a,
                                                     const float* b, float* out, uint32_t batch,
                                                     uint32_t m, uint32_t n, uint32_t k,
                                                     void* stream);
AGPU_API agpu_status agpu_launch_gemm(agpu_device* dev, const float* a, const float* b, float* c,
                                      uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                                      int trans_a, int trans_b, void* stream);
AGPU_API agpu_status agpu_launch_conv2d(agpu_device* dev, const float* input, const float* weight,
                                        const float* bias, float* out, uint32_t batch,
                                        uint32_t in_c, uint32_t in_h, uint32_t in_w,
                                        uint32_t out_c, uint32_t kh, uint32_t kw,
                                        uint32_t stride_h, uint32_t stride_w, uint32_t pad_h,
                                        uint32_t pad_w, uint32_t dil_h, uint32_t dil_w,
                                        uint32_t groups, void* stream);
/* Launch-layer agpu_conv2d_group_norm_swish (caller memory, caller stream). */
AGPU_API agpu_status agpu_launch_conv2d_group_norm_swish(
    agpu_device* dev, const float* input, const float* weight, const float* bias, float* out,
    uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w, uint32_t out_c, uint32_t kh,
    uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ph, uint32_t pw, uint32_t dh, uint32_t dw,
    uint32_t groups, const float* gamma, const float* beta, uint32_t gn_groups, float eps,
    void* stream);
AGPU_API agpu_status agpu_launch_group_norm(agpu_device* dev, const float* x, const float* gamma,
                                            const float* beta, float* y, uint32_t batch,
                                            uint32_t channels, uint32_t spatial, uint32_t groups,
                                            float eps, int apply_swish, void* stream);
AGPU_API agpu_status agpu_launch_group_norm_backward(agpu_device* dev, const float* grad_out,
                                                     const float* input, const float* gamma,
                                                     float* d_input, float* d_gamma,
                                                     float* d_beta, uint32_t batch,
                                                     uint32_t channels, uint32_t spatial,
                                                     uint32_t groups, float eps, void* stream);
AGPU_API agpu_status agpu_launch_sdpa(agpu_device* dev, const float* q, const float* k,
                                      const float* v, float* out, uint32_t batch_heads,
                                      uint32_t seq_len, uint32_t d_k, int causal, void* stream);
AGPU_API agpu_status agpu_launch_sdpa_backward(agpu_device* dev, const float* q,
                                               const float* k, const float* v,
                                               const float* grad_out, float* d_q, float* d_k,
                                               float* d_v, uint32_t batch_heads, uint32_t seq_len,
                                               uint32_t d_k_dim, int causal, void* stream);
AGPU_API agpu_status agpu_launch_gemm_ex(agpu_device* dev, const float* a, const float* b,
                                         float* c, uint32_t batch, uint32_t m, uint32_t n,
                                         uint32_t k, int trans_a, int trans_b, const float* bias,
                                         const float* resid, int act, void* stream);
/* Element strides of one attention operand laid out as [batch, seq, heads, d]
 * in any order (d contiguous): e.g. contiguous [bh, s, d] is
 * {d, s*d, bh*s*d} with heads = bh, batch = 1; the Q part of a packed
 * [batch, seq, 3, heads, d] projection is {3*heads*d, d, seq*3*heads*d}. */
typedef struct agpu_attn_layout {
  uint64_t seq_stride, head_stride, batch_stride;
} agpu_attn_layout;
AGPU_API agpu_status agpu_launch_sdpa_strided(agpu_device* dev, const float* q, const float* k,
                                              const float* v, float* out, uint32_t batch,
                                              uint32_t heads, uint32_t seq_len, uint32_t d_k,
                                              const agpu_attn_layout* q_layout,
                                              const agpu_attn_layout* k_layout,
                                              const agpu_attn_layout* v_layout,
                                              const agpu_attn_layout* out_layout, int causal,
                                              void* stream);
AGPU_API agpu_status agpu_launch_rmsnorm(agpu_device* dev, const float* x, const float* w,
                                         float* y, uint64_t rows, uint32_t cols, float eps,
                                         void* stream);
/* rows of x / y are row_stride elements apart (in place allowed), heads
 * `dim` apart inside a row. */
AGPU_API agpu_status agpu_launch_rope(agpu_device* dev, const float* x, float* y, uint32_t batch,
                                      uint32_t seq, uint32_t heads, uint32_t dim,
                                      uint64_t row_stride, float base, void* stream);
AGPU_API agpu_status agpu_launch_swish_mul(agpu_device* dev, const float* gate, const float* up,
                                           float* out, uint64_t rows, uint32_t cols,
                                           uint64_t gate_stride, uint64_t up_stride,
                                           uint64_t out_stride, void* stream);
AGPU_API agpu_status agpu_launch_softmax(agpu_device* dev, const float* x, float* y,
                                         uint64_t rows, uint32_t cols, void* stream);

/* ------------------------------------------- allocation-free group norm -- */
/* No counterpart in the reference.  Group norm (same math as agpu_group_norm,
 * swish fused when apply_swish != 0) for callers that may not allocate
 * device memory themselves -- a process that owns all device memory through
 * its own arena and cap, a foreign host that passes only device pointers and
 * a stream, a latency-critical loop that cannot pay for an allocation's
 * implicit synchronisation.  It allocates nothing: its scratch (per-chunk
 * partial statistics) lives in a fixed 512 KiB array inside the library,
 * held by every GPU that loads the library until exit.
 * Inputs and output are caller-owned device pointers on the current CUDA
 * device; `stream` is a cudaStream_t (NULL = the default stream).
 * Limit: batch*groups*ceil((channels/groups)*spatial/8192) <= 65536 and
 * batch*groups <= 65535, else AGPU_ERR_UNSUPPORTED (nothing launched).
 * The first call on a device sets that device up (looks up the array's
 * address); make it before any stream capture.  All calls share the array:
 * calls that overlap on the GPU race, so order them on one stream. */
AGPU_API agpu_status agpu_group_norm_noalloc(const float* x, const float* gamma,
                                             const float* beta, float* y, uint32_t batch,
                                             uint32_t channels, uint32_t spatial,
                                             uint32_t groups, float eps, int apply_swish,
                                             void* stream);

/* ------------------------------------------- peer memory (multi-GPU) ----- */
/* No counterpart in the reference (it has no multi-GPU code).  For sharded
 * jobs with one process per GPU of a node: a rank shares its output buffer
 * and an event with its peers through CUDA IPC, then pushes each finished
 * part of its results into every peer's copy of the buffer with
 * agpu_copy_async (copy engines over NVLink, no SMs), records its event after
 * the pushes, and -- once every rank has issued its record (a host barrier)
 * -- makes its stream wait on every peer's event.  Handles are plain bytes,
 * exchanged by the caller (e.g. over torch.distributed or a socket). */
typedef struct agpu_ipc_handle {
  unsigned char bytes[64];
} agpu_ipc_handle;
/* Handle of the allocation holding `dptr` (memory from cudaMalloc, torch's
 * default allocator included; pool memory cannot be shared ->
 * AGPU_ERR_UNSUPPORTED) and dptr's byte offset inside it. */
AGPU_API agpu_status agpu_ipc_export(agpu_device* dev, const void* dptr, agpu_ipc_handle* handle,
                                     uint64_t* offset);
/* Map a peer's allocation into this process; *base + offset is the peer's
 * dptr.  agpu_ipc_close unmaps it (every copy into it must be complete). */
AGPU_API agpu_status agpu_ipc_import(agpu_device* dev, const agpu_ipc_handle* handle,
                                     void** base);
AGPU_API agpu_status agpu_ipc_close(agpu_device* dev, void* base);
/* An interprocess event (no timing) and its handle; a peer's copy from
 * agpu_ipc_event_import.  Both are released with agpu_event_destroy. */
AGPU_API agpu_status agpu_ipc_event_create(agpu_device* dev, void** event,
                                           agpu_ipc_handle* handle);
AGPU_API agpu_status agpu_ipc_event_import(agpu_device* dev, const agpu_ipc_handle* handle,
                                           void** event);
AGPU_API agpu_status agpu_event_destroy(agpu_device* dev, void* event);
/* cudaEventRecord / cudaStreamWaitEvent (stream NULL = the device stream). */
AGPU_API agpu_status agpu_event_record(agpu_device* dev, void* event, void* stream);
AGPU_API agpu_status agpu_stream_wait_event(agpu_device* dev, void* stream, void* event);
/* Stream-ordered device-to-device copy of `bytes` (either side may be a
 * peer's memory from agpu_ipc_import). */
AGPU_API agpu_status agpu_copy_async(agpu_device* dev, void* dst, const void* src, uint64_t bytes,
                                     void* stream);

/* Completion without events or host barriers: agpu_signal_peers stores
 * `value` into each of `count` (<= 16) flag words in peers' memory (mapped
 * with agpu_ipc_import) on `stream`, after all earlier work of that stream
 * (a system-scope release); agpu_wait_flags makes `stream` wait until each
 * of `count` (<= 32) local flag words is >= `target` (serial-number compare),
 * spinning one warp for at most `limit_us` (1 us - 10 s) -- on expiry it
 * records AGPU_WAIT_FLAGS_CODE in the device status word, reported as
 * AGPU_ERR_TIMEOUT by the next agpu_synchronize / agpu_read, and returns. */
#define AGPU_WAIT_FLAGS_CODE 0x5157u
AGPU_API agpu_status agpu_signal_peers(agpu_device* dev, unsigned int* const* peer_flags,
                                       uint32_t count, uint32_t value, void* stream);
AGPU_API agpu_status agpu_wait_flags(agpu_device* dev, const unsigned int* flags,
                                     uint32_t count, uint32_t target, uint32_t limit_us,
                                     void* stream);

/* ---------------------------------------------------- failure self-test -- */
/* No counterpart in the reference.  Exercises the failure path of the
 * bounded device-side waits without faulting or hanging anything: launches
 * one warp on `stream` (NULL = the device stream) that waits on an mbarrier
 * no thread arrives on, gives up after `limit_us` microseconds (1..1e6),
 * records AGPU_SELFTEST_WAIT_CODE in the device status word and returns.
 * The next agpu_synchronize / agpu_read on the device stream then returns
 * AGPU_ERR_TIMEOUT (the message names the code) and clears the word; the
 * device stays usable.  Every pipeline wait of the contraction kernels
 * expires the same way, after 2 s. */
#define AGPU_SELFTEST_WAIT_CODE 0x7e57u
AGPU_API agpu_status agpu_selftest_wait_timeout(agpu_device* dev, uint32_t limit_us,
                                                void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AGPU_H */
