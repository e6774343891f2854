// C-ABI op entry points (buffer layer and launch layer).
//
// Each buffer-layer function mirrors one `pub fn` of the reference's
// `impl GpuDevice`: the same argument order and meaning, the same size
// checks (returned as AGPU_ERR_SHAPE where the reference's `ensure!` returns
// Err), a freshly allocated output buffer owned by the caller.
#include "agpu_internal.cuh"

using namespace agpu;

namespace {

#define CHECK_DEV(dev, fn)                                                 \
  do {                                                                     \
    if (!(dev)) return fail(AGPU_ERR_INVALID, fn ": NULL device");         \
    if (cudaSetDevice((dev)->ordinal) != cudaSuccess)                      \
      return fail(AGPU_ERR_CUDA, fn ": cannot select device %d", (dev)->ordinal); \
  } while (0)

#define CHECK_BUF(b, fn, name)                                             \
  do {                                                                     \
    if (!(b)) return fail(AGPU_ERR_INVALID, fn ": " name " is NULL");      \
  } while (0)

#define CHECK_OUT(o, fn)                                                   \
  do {                                                                     \
    if (!(o)) return fail(AGPU_ERR_INVALID, fn ": out is NULL");           \
    *(o) = nullptr;                                                        \
  } while (0)

#define CHECK_LEN(b, want, fn, name)                                                      \
  do {                                                                                    \
    if ((b)->len != (uint64_t)(want))                                                     \
      return fail(AGPU_ERR_SHAPE, fn ": " name " has %llu elems, expected %llu",          \
                  (unsigned long long)(b)->len, (unsigned long long)(want));              \
  } while (0)

// Allocate `n` floats, run `launch`, free the output again if it failed.
template <typename F>
agpu_status with_output(agpu_device* dev, uint64_t n, agpu_buffer** out, F&& launch) {
  agpu_buffer* o = nullptr;
  AGPU_TRY(new_buffer(dev, n, &o));
  agpu_status s = launch(o->dptr);
  if (s != AGPU_OK) {
    agpu_buffer_free(o);
    return s;
  }
  *out = o;
  return AGPU_OK;
}

agpu_status unary(agpu_device* dev, const agpu_buffer* a, agpu_buffer** out, Unary op, float s,
                  const char* fn) {
  if (!dev) return fail(AGPU_ERR_INVALID, "%s: NULL device", fn);
  if (!a) return fail(AGPU_ERR_INVALID, "%s: input is NULL", fn);
  if (!out) return fail(AGPU_ERR_INVALID, "%s: out is NULL", fn);
  *out = nullptr;
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  return with_output(dev, a->len, out, [&](float* o) {
    return launch_unary(dev, op, a->dptr, o, a->len, s, dev->stream);
  });
}

agpu_status binary(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                   agpu_buffer** out, Binary op, const char* fn) {
  if (!dev) return fail(AGPU_ERR_INVALID, "%s: NULL device", fn);
  if (!a || !b) return fail(AGPU_ERR_INVALID, "%s: input is NULL", fn);
  if (!out) return fail(AGPU_ERR_INVALID, "%s: out is NULL", fn);
  *out = nullptr;
  // src/ops/elementwise.rs:189,194,199,231,237,243,249
  if (a->len != b->len)
    return fail(AGPU_ERR_SHAPE, "%s: length mismatch (%llu vs %llu)", fn,
                (unsigned long long)a->len, (unsigned long long)b->len);
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  return with_output(dev, a->len, out, [&](float* o) {
    return launch_binary(dev, op, a->dptr, b->dptr, o, a->len, dev->stream);
  });
}

}  // namespace

extern "C" {

// ------------------------------------------------------------ contractions --
agpu_status agpu_matmul(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b, uint32_t m,
                        uint32_t n, uint32_t k, agpu_buffer** out) {
  CHECK_DEV(dev, "matmul");
  CHECK_BUF(a, "matmul", "A");
  CHECK_BUF(b, "matmul", "B");
  CHECK_OUT(out, "matmul");
  // src/ops/conv.rs:417-418
  CHECK_LEN(a, (uint64_t)m * k, "matmul", "A");
  CHECK_LEN(b, (uint64_t)k * n, "matmul", "B");
  return with_output(dev, (uint64_t)m * n, out, [&](float* c) {
    return launch_gemm(dev, a->dptr, b->dptr, c, 1, m, n, k, false, false, dev->stream);
  });
}

agpu_status agpu_batch_matmul(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                              uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                              agpu_buffer** out) {
  CHECK_DEV(dev, "batch_matmul");
  CHECK_BUF(a, "batch_matmul", "A");
  CHECK_BUF(b, "batch_matmul", "B");
  CHECK_OUT(out, "batch_matmul");
  // src/ops/conv.rs:427-428
  CHECK_LEN(a, (uint64_t)batch * m * k, "batch_matmul", "A");
  CHECK_LEN(b, (uint64_t)batch * k * n, "batch_matmul", "B");
  return with_output(dev, (uint64_t)batch * m * n, out, [&](float* c) {
    return launch_gemm(dev, a->dptr, b->dptr, c, batch, m, n, k, false, false, dev->stream);
  });
}

agpu_status agpu_gemm(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                      uint32_t batch, uint32_t m, uint32_t n, uint32_t k, int trans_a, int trans_b,
                      agpu_buffer** out) {
  CHECK_DEV(dev, "gemm");
  CHECK_BUF(a, "gemm", "A");
  CHECK_BUF(b, "gemm", "B");
  CHECK_OUT(out, "gemm");
  CHECK_LEN(a, (uint64_t)batch * m * k, "gemm", "A");
  CHECK_LEN(b, (uint64_t)batch * k * n, "gemm", "B");
  return with_output(dev, (uint64_t)batch * m * n, out, [&](float* c) {
    return launch_gemm(dev, a->dptr, b->dptr, c, batch, m, n, k, trans_a != 0, trans_b != 0,
                       dev->stream);
  });
}

// --------------------------------------------------------------- softmax --
agpu_status agpu_softmax(agpu_device* dev, const agpu_buffer* x, uint32_t rows, uint32_t cols,
                         agpu_buffer** out) {
  CHECK_DEV(dev, "softmax");
  CHECK_BUF(x, "softmax", "input");
  CHECK_OUT(out, "softmax");
  // src/ops/attention.rs:92
  CHECK_LEN(x, (uint64_t)rows * cols, "softmax", "input");
  return with_output(dev, (uint64_t)rows * cols, out, [&](float* y) {
    return launch_softmax(dev, x->dptr, y, rows, cols, dev->stream);
  });
}

// ------------------------------------------------------------ group norm --
static agpu_status group_norm_impl(agpu_device* dev, const agpu_buffer* x,
                                   const agpu_buffer* gamma, const agpu_buffer* beta,
                                   uint32_t batch, uint32_t channels, uint32_t spatial,
                                   uint32_t groups, float eps, bool swish, agpu_buffer** out,
                                   const char* fn) {
  if (!dev) return fail(AGPU_ERR_INVALID, "%s: NULL device", fn);
  if (!x || !gamma || !beta) return fail(AGPU_ERR_INVALID, "%s: input is NULL", fn);
  if (!out) return fail(AGPU_ERR_INVALID, "%s: out is NULL", fn);
  *out = nullptr;
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  // src/ops/norm.rs:218-221
  const uint64_t total = (uint64_t)batch * channels * spatial;
  if (x->len != total)
    return fail(AGPU_ERR_SHAPE, "%s: input has %llu elems, expected %llu", fn,
                (unsigned long long)x->len, (unsigned long long)total);
  if (gamma->len != channels || beta->len != channels)
    return fail(AGPU_ERR_SHAPE, "%s: gamma/beta must have %u elems", fn, channels);
  if (groups == 0 || channels % groups != 0)
    return fail(AGPU_ERR_SHAPE, "%s: channels must be divisible by groups", fn);
  return with_output(dev, total, out, [&](float* y) {
    return launch_group_norm(dev, x->dptr, gamma->dptr, beta->dptr, y, batch, channels, spatial,
                             groups, eps, swish, dev->stream);
  });
}

extern "C" agpu_status agpu_group_norm(agpu_device* dev, const agpu_buffer* x,
                                       const agpu_buffer* gamma, const agpu_buffer* beta,
                                       uint32_t batch, uint32_t channels, uint32_t spatial,
                                       uint32_t groups, float eps, agpu_buffer** out) {
  return group_norm_impl(dev, x, gamma, beta, batch, channels, spatial, groups, eps, false, out,
                         "group_norm");
}

extern "C" agpu_status agpu_group_norm_swish(agpu_device* dev, const agpu_buffer* x,
                                             const agpu_buffer* gamma, const agpu_buffer* beta,
                                             uint32_t batch, uint32_t channels, uint32_t spatial,
                                             uint32_t groups, float eps, agpu_buffer** out) {
  return group_norm_impl(dev, x, gamma, beta, batch, channels, spatial, groups, eps, true, out,
                         "group_norm_swish");
}

// ----------------------------------------------------------- elementwise --
agpu_status agpu_add(agpu_device* d, const agpu_buffer* a, const agpu_buffer* b, agpu_buffer** o) {
  return binary(d, a, b, o, Binary::Add, "add");
}
agpu_status agpu_sub(agpu_device* d, const agpu_buffer* a, const agpu_buffer* b, agpu_buffer** o) {
  return binary(d, a, b, o, Binary::Sub, "sub");
}
agpu_status agpu_mul(agpu_device* d, const agpu_buffer* a, const agpu_buffer* b, agpu_buffer** o) {
  return binary(d, a, b, o, Binary::Mul, "mul");
}
agpu_status agpu_relu(agpu_device* d, const agpu_buffer* a, agpu_buffer** o) {
  return unary(d, a, o, Unary::Relu, 0.f, "relu");
}
agpu_status agpu_sigmoid(agpu_device* d, const agpu_buffer* a, agpu_buffer** o) {
  return unary(d, a, o, Unary::Sigmoid, 0.f, "sigmoid");
}
agpu_status agpu_swish(agpu_device* d, const agpu_buffer* a, agpu_buffer** o) {
  return unary(d, a, o, Unary::Swish, 0.f, "swish");
}
agpu_status agpu_tanh_act(agpu_device* d, const agpu_buffer* a, agpu_buffer** o) {
  return unary(d, a, o, Unary::Tanh, 0.f, "tanh_act");
}
agpu_status agpu_scale(agpu_device* d, const agpu_buffer* a, float s, agpu_buffer** o) {
  return unary(d, a, o, Unary::Scale, s, "scale");
}
agpu_status agpu_relu_backward(agpu_device* d, const agpu_buffer* g, const agpu_buffer* x,
                               agpu_buffer** o) {
  return binary(d, g, x, o, Binary::ReluBwd, "relu_backward");
}
agpu_status agpu_sigmoid_backward(agpu_device* d, const agpu_buffer* g, const agpu_buffer* y,
                                  agpu_buffer** o) {
  return binary(d, g, y, o, Binary::SigmoidBwd, "sigmoid_backward");
}
agpu_status agpu_swish_backward(agpu_device* d, const agpu_buffer* g, const agpu_buffer* x,
                                agpu_buffer** o) {
  return binary(d, g, x, o, Binary::SwishBwd, "swish_backward");
}
agpu_status agpu_tanh_backward(agpu_device* d, const agpu_buffer* g, const agpu_buffer* y,
                               agpu_buffer** o) {
  return binary(d, g, y, o, Binary::TanhBwd, "tanh_backward");
}

// ------------------------------------------------------------ tensor ops --
agpu_status agpu_transpose(agpu_device* dev, const agpu_buffer* a, uint32_t outer, uint32_t d0,
                           uint32_t d1, uint32_t inner, agpu_buffer** out) {
  CHECK_DEV(dev, "transpose");
  CHECK_BUF(a, "transpose", "input");
  CHECK_OUT(out, "transpose");
  const uint64_t total = (uint64_t)outer * d0 * d1 * inner;
  // src/ops/tensor_ops.rs:257
  CHECK_LEN(a, total, "transpose", "input");
  return with_output(dev, total, out, [&](float* o) {
    return launch_transpose(dev, a->dptr, o, outer, d0, d1, inner, dev->stream);
  });
}

agpu_status agpu_add_per_col(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                             uint32_t rows, uint32_t cols, agpu_buffer** out) {
  CHECK_DEV(dev, "add_per_col");
  CHECK_BUF(a, "add_per_col", "A");
  CHECK_BUF(b, "add_per_col", "bias");
  CHECK_OUT(out, "add_per_col");
  // src/ops/tensor_ops.rs:341-342
  CHECK_LEN(a, (uint64_t)rows * cols, "add_per_col", "A");
  CHECK_LEN(b, cols, "add_per_col", "bias");
  return with_output(dev, (uint64_t)rows * cols, out, [&](float* o) {
    return launch_add_per_col(dev, a->dptr, b->dptr, o, rows, cols, dev->stream);
  });
}

// ----------------------------------------------------------- launch layer --
agpu_status agpu_launch_batch_matmul(agpu_device* dev, const float* a, const float* b, float* c,
                                     uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                                     void* stream) {
  CHECK_DEV(dev, "launch_batch_matmul");
  if ((!a || !b || !c) && (uint64_t)batch * m * n)
    return fail(AGPU_ERR_INVALID, "launch_batch_matmul: NULL pointer");
  return launch_gemm(dev, a, b, c, batch, m, n, k, false, false, pick_stream(dev, stream));
}

agpu_status agpu_launch_gemm(agpu_device* dev, const float* a, const float* b, float* c,
                             uint32_t batch, uint32_t m, uint32_t n, uint32_t k, int trans_a,
                             int trans_b, void* stream) {
  CHECK_DEV(dev, "launch_gemm");
  if ((!a || !b || !c) && (uint64_t)batch * m * n)
    return fail(AGPU_ERR_INVALID, "launch_gemm: NULL pointer");
  return launch_gemm(dev, a, b, c, batch, m, n, k, trans_a != 0, trans_b != 0,
                     pick_stream(dev, stream));
}

agpu_status agpu_launch_group_norm(agpu_device* dev, const float* x, const float* gamma,
                                   const float* beta, float* y, uint32_t batch, uint32_t channels,
                                   uint32_t spatial, uint32_t groups, float eps, int apply_swish,
                                   void* stream) {
  CHECK_DEV(dev, "launch_group_norm");
  if (groups == 0 || channels % groups != 0)
    return fail(AGPU_ERR_SHAPE, "launch_group_norm: channels must be divisible by groups");
  return launch_group_norm(dev, x, gamma, beta, y, batch, channels, spatial, groups, eps,
                           apply_swish != 0, pick_stream(dev, stream));
}

agpu_status agpu_launch_softmax(agpu_device* dev, const float* x, float* y, uint64_t rows,
                                uint32_t cols, void* stream) {
  CHECK_DEV(dev, "launch_softmax");
  if ((!x || !y) && rows * cols) return fail(AGPU_ERR_INVALID, "launch_softmax: NULL pointer");
  return launch_softmax(dev, x, y, rows, cols, pick_stream(dev, stream));
}

}  // extern "C"
