// Internal runtime state shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/agpu.h"

struct agpu_device {
  int ordinal = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  // second stream for work a launcher forks off and joins back (created on
  // first use, under `mu`)
  cudaStream_t aux = nullptr;
  // this device's own stream-ordered pool (cudaMemPoolCreate), so that its
  // release threshold and cached blocks touch no other user of the device
  cudaMemPool_t pool = nullptr;
  // device-wide default arithmetic of the contractions; read once per call
  // through effective_precision(), which a thread-scoped override shadows
  std::atomic<int> precision{AGPU_PREC_TF32};
  char name[256] = {0};
  // Device-side status word written by kernels whose bounded waits expire.
  unsigned int* d_status = nullptr;
  std::atomic<uint64_t> launches{0};
  // One reference held by the handle returned from agpu_device_create, one
  // per live buffer: buffers may outlive agpu_device_destroy (their memory
  // goes back to the pool when they are freed), and the stream and status
  // word are released with the last reference.
  std::atomic<int64_t> refs{1};
  std::mutex mu;  // guards descriptor caches and pool growth
};

struct agpu_buffer {
  float* dptr = nullptr;
  uint64_t len = 0;
  agpu_device* dev = nullptr;
};

namespace agpu {

// Per-thread last error message (agpu_last_error_message).
void set_error(const char* fmt, ...);
agpu_status fail(agpu_status s, const char* fmt, ...);

// Check a CUDA call; on failure record the message and return AGPU_ERR_CUDA
// (or AGPU_ERR_OOM for allocation failures).
agpu_status cuda_status(cudaError_t e, const char* what);

#define AGPU_CUDA(expr)                                             \
  do {                                                              \
    cudaError_t e__ = (expr);                                       \
    if (e__ != cudaSuccess) return ::agpu::cuda_status(e__, #expr); \
  } while (0)

#define AGPU_TRY(expr)                     \
  do {                                     \
    agpu_status s__ = (expr);              \
    if (s__ != AGPU_OK) return s__;        \
  } while (0)

// Stream-ordered allocation from the device pool; sets OOM on failure.
agpu_status pool_alloc(agpu_device* dev, size_t bytes, void** out, cudaStream_t s);
void pool_free(agpu_device* dev, void* p, cudaStream_t s);

// Drop one reference to `dev`; the last one releases the stream.
void device_release(agpu_device* dev);

// The device's auxiliary stream (created on first use), or nullptr on error.
cudaStream_t aux_stream(agpu_device* dev);

// Allocate an output buffer of n floats on the device stream.
agpu_status new_buffer(agpu_device* dev, uint64_t n, agpu_buffer** out);

// Precision set by agpu_set_thread_precision for calls made from this host
// thread (-1: none, use the device's).
extern thread_local int g_thread_precision;

// The arithmetic a contraction enqueued now from this thread uses: the
// thread's override if set, else the device's setting.  Each launcher reads
// it once, so one call never mixes modes.
inline agpu_precision effective_precision(const agpu_device* dev) {
  const int t = g_thread_precision;
  return static_cast<agpu_precision>(t >= 0 ? t : dev->precision.load(std::memory_order_relaxed));
}

inline cudaStream_t pick_stream(agpu_device* dev, void* s) {
  return s ? static_cast<cudaStream_t>(s) : dev->stream;
}

// After a launch: record it and turn launch errors into a status.
agpu_status after_launch(agpu_device* dev, const char* kernel, int n_launches = 1);
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per kernel and device
// (a driver call on every launch otherwise; the value never changes).
template <auto Kernel>
cudaError_t set_smem_once(const agpu_device* dev, int bytes) {
  static std::atomic<uint64_t> done{0};
  const uint64_t bit = 1ull << (dev->ordinal & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Read back and clear the device status word (non-zero = a bounded wait expired).
agpu_status check_device_status(agpu_device* dev);

inline uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

// ----------------------------------------------------------- op launchers --
// Implemented in the kernel translation units; all validate nothing (the
// C-ABI layer validates) and enqueue on `s`.
agpu_status launch_gemm(agpu_device* dev, const float* a, const float* b, float* c,
                        uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                        bool a_trans, bool b_trans, cudaStream_t s);
// Fused GEMM epilogue: C = act(A*B + bias[col] + resid[batch, row, col]).
struct GemmEpilogue {
  const float* bias = nullptr;   // [n] or null
  const float* resid = nullptr;  // [batch, m, n] or null (may alias nothing but C's shape)
  int act = 0;                   // 0 none, 1 swish, 2 relu
  // Row-vector modes for the attention backward (C = A B^T with no bias,
  // resid or act; only on the TF32 CTA-pair kernel -- launch_gemm_ex returns
  // AGPU_ERR_UNSUPPORTED, launching nothing, where that kernel does not run
  // the GEMM whole):
  //   mode 1: C = 2^(A*B * scale - rowvec[batch, row]), 0 where col > row if causal
  //   mode 2: C = C o (A*B - rowvec[batch, row]) * scale  (C read, then overwritten)
  int mode = 0;
  const float* rowvec = nullptr;  // [batch, m]
  float scale = 1.0f;
  bool causal = false;
};
// Whether launch_gemm_ex would run a row-vector mode for this shape.
bool gemm_rowvec_mode_ok(agpu_device* dev, const float* a, const float* b, const float* c,
                         uint32_t batch, uint32_t m, uint32_t n, uint32_t k);
agpu_status launch_gemm_ex(agpu_device* dev, const float* a, const float* b, float* c,
                           uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool a_trans,
                           bool b_trans, const GemmEpilogue& ep, cudaStream_t s);
agpu_status launch_softmax(agpu_device* dev, const float* x, float* y, uint64_t rows,
                           uint32_t cols, cudaStream_t s);

agpu_status launch_group_norm(agpu_device* dev, const float* x, const float* gamma,
                              const float* beta, float* y, uint32_t batch, uint32_t channels,
                              uint32_t spatial, uint32_t groups, float eps, bool swish,
                              cudaStream_t s);
agpu_status launch_group_norm_backward(agpu_device* dev, const float* dy, const float* x,
                                       const float* gamma, float* dx, float* dgamma,
                                       float* dbeta, uint32_t batch, uint32_t channels,
                                       uint32_t spatial, uint32_t groups, float eps,
                                       cudaStream_t s);
agpu_status launch_adamw(agpu_device* dev, const agpu_adamw_tensor* tensors, uint32_t count,
                         float lr, float beta1, float beta2, float eps, float weight_decay,
                         uint32_t step, cudaStream_t s);

agpu_status launch_rmsnorm(agpu_device* dev, const float* x, const float* w, float* y,
                           uint64_t rows, uint32_t cols, float eps, cudaStream_t s);
agpu_status launch_rope(agpu_device* dev, const float* x, float* y, uint32_t batch, uint32_t seq,
                        uint32_t heads, uint32_t dim, uint64_t row_stride, float base,
                        cudaStream_t s);
agpu_status launch_swish_mul(agpu_device* dev, const float* gate, const float* up, float* out,
                             uint64_t rows, uint32_t cols, uint64_t gs, uint64_t us, uint64_t os,
                             cudaStream_t s);
agpu_status launch_attention_strided(agpu_device* dev, const float* q, const float* k,
                                     const float* v, float* o, uint32_t B, uint32_t H,
                                     uint32_t s, uint32_t d, const long long (&qs)[3],
                                     const long long (&ks)[3], const long long (&vs)[3],
                                     const long long (&os)[3], bool causal, cudaStream_t st);
agpu_status launch_attention(agpu_device* dev, const float* q, const float* k, const float* v,
                             float* o, uint32_t bh, uint32_t s, uint32_t d, bool causal,
                             cudaStream_t st);
// The forward on CTA pairs writing each row's log-sum-exp of its base-2
// scores (P = 2^(q.k / sqrt(d) * log2 e - lse)) to lse [bh, s];
// AGPU_ERR_UNSUPPORTED, launching nothing, where the pair kernel does not run.
agpu_status launch_attention_lse(agpu_device* dev, const float* q, const float* k,
                                 const float* v, float* o, float* lse, uint32_t bh, uint32_t s,
                                 uint32_t d, bool causal, cudaStream_t st);
// dQ, dK, dV of attention from dO (recomputes P; tensor-core GEMMs; scratch
// from the device pool).
agpu_status launch_attention_backward(agpu_device* dev, const float* q, const float* k,
                                      const float* v, const float* dout, float* dq, float* dk,
                                      float* dv, uint32_t bh, uint32_t s, uint32_t d,
                                      bool causal, cudaStream_t st);

// conv2d geometry (NCHW); ho/wo already computed.
struct ConvParams {
  int n, cin, h, w, cout, kh, kw, sh, sw, ph, pw, dh, dw, groups, ho, wo;
};
agpu_status launch_conv2d(agpu_device* dev, const ConvParams& p, const float* x, const float* w,
                          const float* bias, float* y, cudaStream_t s);
// conv2d followed by group_norm (+ swish) of its output, in place.
struct GnEpilogue {
  const float* gamma;
  const float* beta;
  uint32_t groups;
  float eps;
  bool swish;
};
agpu_status launch_conv2d_gn(agpu_device* dev, const ConvParams& p, const float* x,
                             const float* w, const float* bias, float* y, const GnEpilogue& gn,
                             cudaStream_t s);
agpu_status launch_conv_transpose2d(agpu_device* dev, const ConvParams& p, const float* x,
                                    const float* w, const float* bias, float* y, cudaStream_t s);
agpu_status launch_conv2d_grad_weight(agpu_device* dev, const ConvParams& p, const float* x,
                                      const float* gy, float* gw, cudaStream_t s);
agpu_status launch_conv2d_grad_bias(agpu_device* dev, const float* gy, float* gb, int n, int cout,
                                    long long hw, cudaStream_t s);

enum class Unary : int { Relu = 0, Sigmoid, Swish, Tanh, Scale };
enum class Binary : int {
  Add = 0, Sub, Mul, ReluBwd, SigmoidBwd, SwishBwd, TanhBwd
};
agpu_status launch_unary(agpu_device* dev, Unary op, const float* a, float* out, uint64_t n,
                         float s, cudaStream_t st);
agpu_status launch_binary(agpu_device* dev, Binary op, const float* a, const float* b,
                          float* out, uint64_t n, cudaStream_t st);
agpu_status launch_transpose(agpu_device* dev, const float* a, float* out, uint64_t outer,
                             uint64_t d0, uint64_t d1, uint64_t inner, cudaStream_t st);
agpu_status launch_add_per_col(agpu_device* dev, const float* a, const float* b, float* out,
                               uint64_t rows, uint64_t cols, cudaStream_t st);
agpu_status launch_add_broadcast(agpu_device* dev, const float* a, const float* b, float* out,
                                 uint64_t outer, uint64_t inner, cudaStream_t s);
agpu_status launch_sum_inner(agpu_device* dev, const float* src, float* out, uint64_t outer,
                             uint64_t inner, cudaStream_t s);
agpu_status launch_sum_rows(agpu_device* dev, const float* src, float* out, uint64_t rows,
                            uint64_t cols, cudaStream_t s);
agpu_status launch_concat(agpu_device* dev, const float* a, const float* b, float* out,
                          uint64_t outer, uint64_t ai, uint64_t bi, cudaStream_t s);
agpu_status launch_slice_per_block(agpu_device* dev, const float* src, float* dst, uint64_t outer,
                                   uint64_t size, uint64_t offset, uint64_t combined,
                                   cudaStream_t s);
agpu_status launch_upsample_nearest2d(agpu_device* dev, const float* in, float* out,
                                      uint64_t planes, uint32_t in_h, uint32_t in_w, uint32_t sh,
                                      uint32_t sw, cudaStream_t s);
agpu_status launch_upsample_nearest2d_backward(agpu_device* dev, const float* go, float* gi,
                                               uint64_t planes, uint32_t in_h, uint32_t in_w,
                                               uint32_t sh, uint32_t sw, cudaStream_t s);
agpu_status launch_mse_loss(agpu_device* dev, const float* pred, const float* target, float* out,
                            uint64_t n, cudaStream_t s);

}  // namespace agpu
