// C-ABI op entry points (buffer layer and launch layer).
//
// Each buffer-layer function mirrors one `pub fn` of the reference's
// `impl GpuDevice`: the same argument order and meaning, the same size
// checks (returned as AGPU_ERR_SHAPE where the reference's `ensure!` returns
// Err), a freshly allocated output buffer owned by the caller.
#include <cstdlib>
#include <vector>

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

// C = batch_matmul(A, B), then the row softmax of C in place (each row is
// read completely before any of it is written).  When the batch splits into
// pieces that each still fill the SMs (up to 8), the GEMMs run back to back on
// the caller's stream and each piece's softmax on the device's auxiliary
// stream as soon as its GEMM is done: the softmax (HBM-bound) runs beside
// the next GEMM (tensor-bound), no GEMM ever waits for a softmax, and only
// the last piece's softmax is exposed.
static agpu_status bmm_softmax(agpu_device* dev, const float* a, const float* b, float* c,
                               uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                               cudaStream_t s) {
  const uint64_t tiles_item = ceil_div(m, 256) * ceil_div(n, 256);
  static const uint32_t max_pieces = [] {
    const char* e = getenv("AGPU_BMM_SOFTMAX_PIECES");
    return e ? (uint32_t)atoi(e) : 8u;
  }();
  uint32_t pieces = 1;
  for (uint32_t p : {8u, 4u, 2u})
    if (p <= max_pieces && batch >= p &&
        (uint64_t)(batch / p) * tiles_item >= (uint64_t)dev->sm_count) {
      pieces = p;
      break;
    }
  cudaStream_t s2 = pieces > 1 ? aux_stream(dev) : nullptr;
  if (!s2) {
    AGPU_TRY(launch_gemm(dev, a, b, c, batch, m, n, k, false, false, s));
    return launch_softmax(dev, c, c, (uint64_t)batch * m, n, s);
  }
  cudaEvent_t ev = nullptr;
  if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess)
    return cuda_status(cudaGetLastError(), "batch_matmul_softmax: event create");
  agpu_status st = AGPU_OK;
  cudaError_t e = cudaSuccess;
  uint32_t b0 = 0;
  for (uint32_t i = 0; i < pieces && st == AGPU_OK && e == cudaSuccess; ++i) {
    const uint32_t nb = (uint32_t)((uint64_t)batch * (i + 1) / pieces) - b0;
    float* ci = c + (uint64_t)b0 * m * n;
    st = launch_gemm(dev, a + (uint64_t)b0 * m * k, b + (uint64_t)b0 * k * n, ci, nb, m, n, k,
                     false, false, s);
    // each wait takes the event's latest record: this piece's GEMM
    if (st == AGPU_OK) e = cudaEventRecord(ev, s);
    if (st == AGPU_OK && e == cudaSuccess) e = cudaStreamWaitEvent(s2, ev, 0);
    if (st == AGPU_OK && e == cudaSuccess)
      st = launch_softmax(dev, ci, ci, (uint64_t)nb * m, n, s2);
    b0 += nb;
  }
  // join in every case, so that nothing on s2 outlives the call's stream order
  const cudaError_t ej = cudaEventRecord(ev, s2);
  const cudaError_t ew = ej == cudaSuccess ? cudaStreamWaitEvent(s, ev, 0) : ej;
  cudaEventDestroy(ev);
  if (e == cudaSuccess) e = ew;
  if (e != cudaSuccess && st == AGPU_OK) st = cuda_status(e, "batch_matmul_softmax: fork/join");
  return st;
}

agpu_status agpu_batch_matmul_softmax(agpu_device* dev, const agpu_buffer* a,
                                      const agpu_buffer* b, uint32_t batch, uint32_t m,
                                      uint32_t n, uint32_t k, agpu_buffer** out) {
  CHECK_DEV(dev, "batch_matmul_softmax");
  CHECK_BUF(a, "batch_matmul_softmax", "A");
  CHECK_BUF(b, "batch_matmul_softmax", "B");
  CHECK_OUT(out, "batch_matmul_softmax");
  // src/ops/conv.rs:427-428
  CHECK_LEN(a, (uint64_t)batch * m * k, "batch_matmul_softmax", "A");
  CHECK_LEN(b, (uint64_t)batch * k * n, "batch_matmul_softmax", "B");
  return with_output(dev, (uint64_t)batch * m * n, out, [&](float* c) {
    return bmm_softmax(dev, a->dptr, b->dptr, c, batch, m, n, k, dev->stream);
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

// --------------------------------------------------------------- conv2d --
static agpu_status conv_geometry(uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w,
                                 uint32_t out_c, uint32_t kh, uint32_t kw, uint32_t sh,
                                 uint32_t sw, uint32_t ph, uint32_t pw, uint32_t dh, uint32_t dw,
                                 uint32_t groups, ConvParams* p, const char* fn) {
  if (groups == 0 || in_c % groups || out_c % groups)
    return fail(AGPU_ERR_SHAPE, "%s: channels (%u in, %u out) not divisible by groups %u", fn,
                in_c, out_c, groups);
  if (sh == 0 || sw == 0 || dh == 0 || dw == 0 || kh == 0 || kw == 0)
    return fail(AGPU_ERR_INVALID, "%s: zero stride, dilation or kernel size", fn);
  const long long eh = (long long)in_h + 2LL * ph - (long long)dh * (kh - 1) - 1;
  const long long ew = (long long)in_w + 2LL * pw - (long long)dw * (kw - 1) - 1;
  if (eh < 0 || ew < 0)
    return fail(AGPU_ERR_SHAPE, "%s: kernel larger than the padded input", fn);
  *p = ConvParams{(int)batch, (int)in_c, (int)in_h, (int)in_w, (int)out_c, (int)kh, (int)kw,
                  (int)sh, (int)sw, (int)ph, (int)pw, (int)dh, (int)dw, (int)groups,
                  (int)(eh / sh + 1), (int)(ew / sw + 1)};
  return AGPU_OK;
}

extern "C" agpu_status agpu_conv2d(agpu_device* dev, const agpu_buffer* input,
                                   const agpu_buffer* weight, const agpu_buffer* bias,
                                   uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w,
                                   uint32_t out_c, uint32_t kh, uint32_t kw, uint32_t sh,
                                   uint32_t sw, uint32_t ph, uint32_t pw, uint32_t dh, uint32_t dw,
                                   uint32_t groups, agpu_buffer** out) {
  CHECK_DEV(dev, "conv2d");
  CHECK_BUF(input, "conv2d", "input");
  CHECK_BUF(weight, "conv2d", "weight");
  CHECK_OUT(out, "conv2d");
  ConvParams p;
  AGPU_TRY(conv_geometry(batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, dh, dw, groups,
                         &p, "conv2d"));
  // src/ops/conv.rs:450-458
  CHECK_LEN(input, (uint64_t)batch * in_c * in_h * in_w, "conv2d", "input");
  CHECK_LEN(weight, (uint64_t)out_c * (in_c / groups) * kh * kw, "conv2d", "weight");
  if (bias) CHECK_LEN(bias, out_c, "conv2d", "bias");
  return with_output(dev, (uint64_t)batch * out_c * p.ho * p.wo, out, [&](float* y) {
    return launch_conv2d(dev, p, input->dptr, weight->dptr, bias ? bias->dptr : nullptr, y,
                         dev->stream);
  });
}

// conv2d -> group_norm -> swish (the UNet block) in one call; the same
// checks as agpu_conv2d and agpu_group_norm_swish.
extern "C" agpu_status agpu_conv2d_group_norm_swish(
    agpu_device* dev, const agpu_buffer* input, const agpu_buffer* weight,
    const agpu_buffer* bias, uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w,
    uint32_t out_c, uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ph, uint32_t pw,
    uint32_t dh, uint32_t dw, uint32_t groups, const agpu_buffer* gamma, const agpu_buffer* beta,
    uint32_t gn_groups, float eps, agpu_buffer** out) {
  CHECK_DEV(dev, "conv2d_group_norm_swish");
  CHECK_BUF(input, "conv2d_group_norm_swish", "input");
  CHECK_BUF(weight, "conv2d_group_norm_swish", "weight");
  CHECK_BUF(gamma, "conv2d_group_norm_swish", "gamma");
  CHECK_BUF(beta, "conv2d_group_norm_swish", "beta");
  CHECK_OUT(out, "conv2d_group_norm_swish");
  ConvParams p;
  AGPU_TRY(conv_geometry(batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, dh, dw, groups,
                         &p, "conv2d_group_norm_swish"));
  CHECK_LEN(input, (uint64_t)batch * in_c * in_h * in_w, "conv2d_group_norm_swish", "input");
  CHECK_LEN(weight, (uint64_t)out_c * (in_c / groups) * kh * kw, "conv2d_group_norm_swish",
            "weight");
  if (bias) CHECK_LEN(bias, out_c, "conv2d_group_norm_swish", "bias");
  if (gn_groups == 0 || out_c % gn_groups != 0)  // src/ops/norm.rs:218-221
    return fail(AGPU_ERR_SHAPE, "conv2d_group_norm_swish: channels must be divisible by groups");
  CHECK_LEN(gamma, out_c, "conv2d_group_norm_swish", "gamma");
  CHECK_LEN(beta, out_c, "conv2d_group_norm_swish", "beta");
  const GnEpilogue gn{gamma->dptr, beta->dptr, gn_groups, eps, true};
  return with_output(dev, (uint64_t)batch * out_c * p.ho * p.wo, out, [&](float* y) {
    return launch_conv2d_gn(dev, p, input->dptr, weight->dptr, bias ? bias->dptr : nullptr, y, gn,
                            dev->stream);
  });
}

extern "C" agpu_status agpu_conv_transpose2d(
    agpu_device* dev, const agpu_buffer* input, const agpu_buffer* weight,
    const agpu_buffer* bias, uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w,
    uint32_t out_c, uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ph, uint32_t pw,
    uint32_t oph, uint32_t opw, uint32_t dh, uint32_t dw, uint32_t groups, agpu_buffer** out) {
  CHECK_DEV(dev, "conv_transpose2d");
  CHECK_BUF(input, "conv_transpose2d", "input");
  CHECK_BUF(weight, "conv_transpose2d", "weight");
  CHECK_OUT(out, "conv_transpose2d");
  if (groups == 0 || in_c % groups || out_c % groups || sh == 0 || sw == 0)
    return fail(AGPU_ERR_SHAPE, "conv_transpose2d: bad groups or stride");
  // output size: src/ops/conv.rs:498-499
  const long long oh = ((long long)in_h - 1) * sh - 2LL * ph + (long long)dh * (kh - 1) + oph + 1;
  const long long ow = ((long long)in_w - 1) * sw - 2LL * pw + (long long)dw * (kw - 1) + opw + 1;
  if (oh <= 0 || ow <= 0) return fail(AGPU_ERR_SHAPE, "conv_transpose2d: empty output");
  // src/ops/conv.rs:502-510
  CHECK_LEN(input, (uint64_t)batch * in_c * in_h * in_w, "conv_transpose2d", "input");
  CHECK_LEN(weight, (uint64_t)in_c * (out_c / groups) * kh * kw, "conv_transpose2d", "weight");
  if (bias) CHECK_LEN(bias, out_c, "conv_transpose2d", "bias");
  ConvParams p{(int)batch, (int)in_c, (int)in_h, (int)in_w, (int)out_c, (int)kh, (int)kw,
               (int)sh, (int)sw, (int)ph, (int)pw, (int)dh, (int)dw, (int)groups, (int)oh,
               (int)ow};
  return with_output(dev, (uint64_t)batch * out_c * oh * ow, out, [&](float* y) {
    return launch_conv_transpose2d(dev, p, input->dptr, weight->dptr, bias ? bias->dptr : nullptr,
                                   y, dev->stream);
  });
}

extern "C" agpu_status agpu_conv2d_grad_weight(
    agpu_device* dev, const agpu_buffer* input, const agpu_buffer* grad_out, uint32_t batch,
    uint32_t in_c, uint32_t in_h, uint32_t in_w, uint32_t out_c, uint32_t out_h, uint32_t out_w,
    uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ph, uint32_t pw, uint32_t dh,
    uint32_t dw, uint32_t groups, agpu_buffer** out) {
  CHECK_DEV(dev, "conv2d_grad_weight");
  CHECK_BUF(input, "conv2d_grad_weight", "input");
  CHECK_BUF(grad_out, "conv2d_grad_weight", "grad_out");
  CHECK_OUT(out, "conv2d_grad_weight");
  if (groups == 0 || in_c % groups || out_c % groups)
    return fail(AGPU_ERR_SHAPE, "conv2d_grad_weight: channels not divisible by groups");
  CHECK_LEN(input, (uint64_t)batch * in_c * in_h * in_w, "conv2d_grad_weight", "input");
  CHECK_LEN(grad_out, (uint64_t)batch * out_c * out_h * out_w, "conv2d_grad_weight", "grad_out");
  ConvParams p{(int)batch, (int)in_c, (int)in_h, (int)in_w, (int)out_c, (int)kh, (int)kw,
               (int)sh, (int)sw, (int)ph, (int)pw, (int)dh, (int)dw, (int)groups, (int)out_h,
               (int)out_w};
  return with_output(dev, (uint64_t)out_c * (in_c / groups) * kh * kw, out, [&](float* gw) {
    return launch_conv2d_grad_weight(dev, p, input->dptr, grad_out->dptr, gw, dev->stream);
  });
}

extern "C" agpu_status agpu_conv2d_grad_bias(agpu_device* dev, const agpu_buffer* grad_out,
                                             uint32_t batch, uint32_t out_c, uint32_t out_h,
                                             uint32_t out_w, agpu_buffer** out) {
  CHECK_DEV(dev, "conv2d_grad_bias");
  CHECK_BUF(grad_out, "conv2d_grad_bias", "grad_out");
  CHECK_OUT(out, "conv2d_grad_bias");
  CHECK_LEN(grad_out, (uint64_t)batch * out_c * out_h * out_w, "conv2d_grad_bias", "grad_out");
  return with_output(dev, out_c, out, [&](float* gb) {
    return launch_conv2d_grad_bias(dev, grad_out->dptr, gb, (int)batch, (int)out_c,
                                   (long long)out_h * out_w, dev->stream);
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

extern "C" agpu_status agpu_group_norm_backward(agpu_device* dev, const agpu_buffer* grad_out,
                                                const agpu_buffer* input,
                                                const agpu_buffer* gamma, uint32_t batch,
                                                uint32_t channels, uint32_t spatial,
                                                uint32_t groups, float eps,
                                                agpu_buffer** d_input, agpu_buffer** d_gamma,
                                                agpu_buffer** d_beta) {
  const char* fn = "group_norm_backward";
  if (!dev) return fail(AGPU_ERR_INVALID, "%s: NULL device", fn);
  if (!grad_out || !input || !gamma) return fail(AGPU_ERR_INVALID, "%s: input is NULL", fn);
  if (!d_input || !d_gamma || !d_beta) return fail(AGPU_ERR_INVALID, "%s: out is NULL", fn);
  *d_input = *d_gamma = *d_beta = nullptr;
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  // src/ops/norm.rs:291-294
  const uint64_t total = (uint64_t)batch * channels * spatial;
  if (input->len != total || grad_out->len != total)
    return fail(AGPU_ERR_SHAPE, "%s: input/grad_out must have %llu elems (got %llu, %llu)", fn,
                (unsigned long long)total, (unsigned long long)input->len,
                (unsigned long long)grad_out->len);
  if (gamma->len != channels)
    return fail(AGPU_ERR_SHAPE, "%s: gamma must have %u elems", fn, channels);
  if (groups == 0 || channels % groups != 0)
    return fail(AGPU_ERR_SHAPE, "%s: channels must be divisible by groups", fn);
  agpu_buffer *di = nullptr, *dg = nullptr, *db = nullptr;
  agpu_status st = new_buffer(dev, total, &di);
  if (st == AGPU_OK) st = new_buffer(dev, channels, &dg);
  if (st == AGPU_OK) st = new_buffer(dev, channels, &db);
  if (st == AGPU_OK)
    st = launch_group_norm_backward(dev, grad_out->dptr, input->dptr, gamma->dptr, di->dptr,
                                    dg->dptr, db->dptr, batch, channels, spatial, groups, eps,
                                    dev->stream);
  if (st != AGPU_OK) {
    if (di) agpu_buffer_free(di);
    if (dg) agpu_buffer_free(dg);
    if (db) agpu_buffer_free(db);
    return st;
  }
  *d_input = di;
  *d_gamma = dg;
  *d_beta = db;
  return AGPU_OK;
}

// ----------------------------------------------------------------- AdamW --
extern "C" agpu_status agpu_adamw_step(agpu_device* dev, agpu_buffer* const* params,
                                       const agpu_buffer* const* grads, agpu_buffer* const* m,
                                       agpu_buffer* const* v, uint32_t count, float lr,
                                       float beta1, float beta2, float eps, float weight_decay,
                                       uint32_t step) {
  CHECK_DEV(dev, "adamw_step");
  if (count && (!params || !grads || !m || !v))
    return fail(AGPU_ERR_INVALID, "adamw_step: NULL array");
  std::vector<agpu_adamw_tensor> t(count);
  for (uint32_t i = 0; i < count; ++i) {
    if (!params[i] || !grads[i] || !m[i] || !v[i])
      return fail(AGPU_ERR_INVALID, "adamw_step: NULL buffer at index %u", i);
    // src/optim.rs:95
    if (params[i]->len != grads[i]->len || m[i]->len != params[i]->len ||
        v[i]->len != params[i]->len)
      return fail(AGPU_ERR_SHAPE, "adamw_step: param/grad size mismatch at index %u", i);
    t[i] = agpu_adamw_tensor{params[i]->dptr, grads[i]->dptr, m[i]->dptr, v[i]->dptr,
                             params[i]->len};
  }
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  return launch_adamw(dev, t.data(), count, lr, beta1, beta2, eps, weight_decay, step,
                      dev->stream);
}

// --------------------------------------------------------- gemm epilogue --
extern "C" agpu_status agpu_gemm_ex(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                                    const agpu_buffer* bias, const agpu_buffer* resid,
                                    uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                                    int trans_a, int trans_b, int act, agpu_buffer** out) {
  CHECK_DEV(dev, "gemm_ex");
  CHECK_BUF(a, "gemm_ex", "A");
  CHECK_BUF(b, "gemm_ex", "B");
  CHECK_OUT(out, "gemm_ex");
  CHECK_LEN(a, (uint64_t)batch * m * k, "gemm_ex", "A");
  CHECK_LEN(b, (uint64_t)batch * k * n, "gemm_ex", "B");
  if (bias) CHECK_LEN(bias, n, "gemm_ex", "bias");
  if (resid) CHECK_LEN(resid, (uint64_t)batch * m * n, "gemm_ex", "resid");
  if (act < 0 || act > 3) return fail(AGPU_ERR_INVALID, "gemm_ex: unknown activation %d", act);
  if (act == 3 && (n % 64 != 0 || bias || resid))
    return fail(AGPU_ERR_SHAPE, "gemm_ex: SwiGLU needs n %% 64 == 0 and no bias or residual");
  GemmEpilogue ep;
  ep.bias = bias ? bias->dptr : nullptr;
  ep.resid = resid ? resid->dptr : nullptr;
  ep.act = act;
  const uint64_t cn = act == 3 ? n / 2 : n;
  return with_output(dev, (uint64_t)batch * m * cn, out, [&](float* c) {
    return launch_gemm_ex(dev, a->dptr, b->dptr, c, batch, m, n, k, trans_a != 0, trans_b != 0,
                          ep, dev->stream);
  });
}

// ------------------------------------------------------- LLaMA-layer ops --
extern "C" agpu_status agpu_rmsnorm(agpu_device* dev, const agpu_buffer* x, const agpu_buffer* w,
                                    uint32_t rows, uint32_t cols, float eps, agpu_buffer** out) {
  CHECK_DEV(dev, "rmsnorm");
  CHECK_BUF(x, "rmsnorm", "input");
  CHECK_BUF(w, "rmsnorm", "weight");
  CHECK_OUT(out, "rmsnorm");
  CHECK_LEN(x, (uint64_t)rows * cols, "rmsnorm", "input");
  CHECK_LEN(w, cols, "rmsnorm", "weight");
  return with_output(dev, (uint64_t)rows * cols, out, [&](float* y) {
    return launch_rmsnorm(dev, x->dptr, w->dptr, y, rows, cols, eps, dev->stream);
  });
}

extern "C" agpu_status agpu_rope(agpu_device* dev, const agpu_buffer* x, uint32_t batch,
                                 uint32_t seq, uint32_t heads, uint32_t dim, float base,
                                 agpu_buffer** out) {
  CHECK_DEV(dev, "rope");
  CHECK_BUF(x, "rope", "input");
  CHECK_OUT(out, "rope");
  const uint64_t n = (uint64_t)batch * seq * heads * dim;
  CHECK_LEN(x, n, "rope", "input");
  if (dim % 2) return fail(AGPU_ERR_SHAPE, "rope: head dim %u is odd", dim);
  return with_output(dev, n, out, [&](float* y) {
    return launch_rope(dev, x->dptr, y, batch, seq, heads, dim, (uint64_t)heads * dim, base,
                       dev->stream);
  });
}

extern "C" agpu_status agpu_swish_mul(agpu_device* dev, const agpu_buffer* gate,
                                      const agpu_buffer* up, agpu_buffer** out) {
  CHECK_DEV(dev, "swish_mul");
  CHECK_BUF(gate, "swish_mul", "gate");
  CHECK_BUF(up, "swish_mul", "up");
  CHECK_OUT(out, "swish_mul");
  if (gate->len != up->len)
    return fail(AGPU_ERR_SHAPE, "swish_mul: length mismatch (%llu vs %llu)",
                (unsigned long long)gate->len, (unsigned long long)up->len);
  return with_output(dev, gate->len, out, [&](float* o) {
    return launch_swish_mul(dev, gate->dptr, up->dptr, o, 1, (uint32_t)gate->len, gate->len,
                            up->len, gate->len, dev->stream);
  });
}

// ------------------------------------------------------------------ sdpa --
static agpu_status sdpa_impl(agpu_device* dev, const agpu_buffer* q, const agpu_buffer* k,
                             const agpu_buffer* v, uint32_t bh, uint32_t s, uint32_t d,
                             bool causal, agpu_buffer** out, const char* fn) {
  if (!dev) return fail(AGPU_ERR_INVALID, "%s: NULL device", fn);
  if (!q || !k || !v) return fail(AGPU_ERR_INVALID, "%s: input is NULL", fn);
  if (!out) return fail(AGPU_ERR_INVALID, "%s: out is NULL", fn);
  *out = nullptr;
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  // the reference's transpose/batch_matmul checks (src/ops/tensor_ops.rs:257,
  // src/ops/conv.rs:427-428) require each of Q, K, V to hold bh*s*d elements
  const uint64_t n = (uint64_t)bh * s * d;
  if (q->len != n || k->len != n || v->len != n)
    return fail(AGPU_ERR_SHAPE, "%s: Q/K/V have %llu/%llu/%llu elems, expected %llu", fn,
                (unsigned long long)q->len, (unsigned long long)k->len,
                (unsigned long long)v->len, (unsigned long long)n);
  return with_output(dev, n, out, [&](float* o) {
    return launch_attention(dev, q->dptr, k->dptr, v->dptr, o, bh, s, d, causal, dev->stream);
  });
}

extern "C" agpu_status agpu_scaled_dot_product_attention(agpu_device* dev, const agpu_buffer* q,
                                                         const agpu_buffer* k,
                                                         const agpu_buffer* v, uint32_t bh,
                                                         uint32_t s, uint32_t d,
                                                         agpu_buffer** out) {
  return sdpa_impl(dev, q, k, v, bh, s, d, false, out, "scaled_dot_product_attention");
}

extern "C" agpu_status agpu_sdpa_causal(agpu_device* dev, const agpu_buffer* q,
                                        const agpu_buffer* k, const agpu_buffer* v, uint32_t bh,
                                        uint32_t s, uint32_t d, agpu_buffer** out) {
  return sdpa_impl(dev, q, k, v, bh, s, d, true, out, "sdpa_causal");
}

extern "C" agpu_status agpu_sdpa_backward(agpu_device* dev, const agpu_buffer* q,
                                          const agpu_buffer* k, const agpu_buffer* v,
                                          const agpu_buffer* grad_out, uint32_t bh, uint32_t s,
                                          uint32_t d, int causal, agpu_buffer** d_q,
                                          agpu_buffer** d_k, agpu_buffer** d_v) {
  const char* fn = "sdpa_backward";
  if (!dev) return fail(AGPU_ERR_INVALID, "%s: NULL device", fn);
  if (!q || !k || !v || !grad_out) return fail(AGPU_ERR_INVALID, "%s: input is NULL", fn);
  if (!d_q || !d_k || !d_v) return fail(AGPU_ERR_INVALID, "%s: out is NULL", fn);
  *d_q = *d_k = *d_v = nullptr;
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  // the forward's checks (each of Q, K, V holds bh*s*d elements), and dO has
  // the output's shape
  const uint64_t n = (uint64_t)bh * s * d;
  if (q->len != n || k->len != n || v->len != n || grad_out->len != n)
    return fail(AGPU_ERR_SHAPE, "%s: Q/K/V/dO have %llu/%llu/%llu/%llu elems, expected %llu", fn,
                (unsigned long long)q->len, (unsigned long long)k->len,
                (unsigned long long)v->len, (unsigned long long)grad_out->len,
                (unsigned long long)n);
  agpu_buffer *dq = nullptr, *dk = nullptr, *dv = nullptr;
  agpu_status st = new_buffer(dev, n, &dq);
  if (st == AGPU_OK) st = new_buffer(dev, n, &dk);
  if (st == AGPU_OK) st = new_buffer(dev, n, &dv);
  if (st == AGPU_OK)
    st = launch_attention_backward(dev, q->dptr, k->dptr, v->dptr, grad_out->dptr, dq->dptr,
                                   dk->dptr, dv->dptr, bh, s, d, causal != 0, dev->stream);
  if (st != AGPU_OK) {
    agpu_buffer_free(dq);
    agpu_buffer_free(dk);
    agpu_buffer_free(dv);
    return st;
  }
  *d_q = dq;
  *d_k = dk;
  *d_v = dv;
  return AGPU_OK;
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

agpu_status agpu_add_broadcast(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                               uint32_t outer, uint32_t inner, agpu_buffer** out) {
  CHECK_DEV(dev, "add_broadcast");
  CHECK_BUF(a, "add_broadcast", "A");
  CHECK_BUF(b, "add_broadcast", "B");
  CHECK_OUT(out, "add_broadcast");
  // src/ops/tensor_ops.rs:303-304
  CHECK_LEN(a, (uint64_t)outer * inner, "add_broadcast", "A");
  CHECK_LEN(b, outer, "add_broadcast", "B");
  return with_output(dev, (uint64_t)outer * inner, out, [&](float* o) {
    return launch_add_broadcast(dev, a->dptr, b->dptr, o, outer, inner, dev->stream);
  });
}

agpu_status agpu_sum_inner(agpu_device* dev, const agpu_buffer* src, uint32_t outer,
                           uint32_t inner, agpu_buffer** out) {
  CHECK_DEV(dev, "sum_inner");
  CHECK_BUF(src, "sum_inner", "src");
  CHECK_OUT(out, "sum_inner");
  CHECK_LEN(src, (uint64_t)outer * inner, "sum_inner", "src");  // src/ops/tensor_ops.rs:323
  return with_output(dev, outer, out, [&](float* o) {
    return launch_sum_inner(dev, src->dptr, o, outer, inner, dev->stream);
  });
}

agpu_status agpu_sum_rows(agpu_device* dev, const agpu_buffer* src, uint32_t rows, uint32_t cols,
                          agpu_buffer** out) {
  CHECK_DEV(dev, "sum_rows");
  CHECK_BUF(src, "sum_rows", "src");
  CHECK_OUT(out, "sum_rows");
  CHECK_LEN(src, (uint64_t)rows * cols, "sum_rows", "src");  // src/ops/tensor_ops.rs:361
  return with_output(dev, cols, out, [&](float* o) {
    return launch_sum_rows(dev, src->dptr, o, rows, cols, dev->stream);
  });
}

agpu_status agpu_concat(agpu_device* dev, const agpu_buffer* a, const agpu_buffer* b,
                        uint32_t outer, uint32_t a_inner, uint32_t b_inner, agpu_buffer** out) {
  CHECK_DEV(dev, "concat");
  CHECK_BUF(a, "concat", "A");
  CHECK_BUF(b, "concat", "B");
  CHECK_OUT(out, "concat");
  // src/ops/tensor_ops.rs:234-235
  CHECK_LEN(a, (uint64_t)outer * a_inner, "concat", "A");
  CHECK_LEN(b, (uint64_t)outer * b_inner, "concat", "B");
  const uint64_t total = (uint64_t)outer * ((uint64_t)a_inner + b_inner);
  return with_output(dev, total, out, [&](float* o) {
    return launch_concat(dev, a->dptr, b->dptr, o, outer, a_inner, b_inner, dev->stream);
  });
}

agpu_status agpu_slice_per_block(agpu_device* dev, const agpu_buffer* src, uint32_t outer,
                                 uint32_t slice_size, uint32_t slice_offset, uint32_t combined,
                                 agpu_buffer** out) {
  CHECK_DEV(dev, "slice_per_block");
  CHECK_BUF(src, "slice_per_block", "src");
  CHECK_OUT(out, "slice_per_block");
  // src/ops/tensor_ops.rs:280-281
  CHECK_LEN(src, (uint64_t)outer * combined, "slice_per_block", "src");
  if ((uint64_t)slice_offset + slice_size > combined)
    return fail(AGPU_ERR_SHAPE, "slice_per_block: offset %u + size %u > combined %u",
                slice_offset, slice_size, combined);
  return with_output(dev, (uint64_t)outer * slice_size, out, [&](float* o) {
    return launch_slice_per_block(dev, src->dptr, o, outer, slice_size, slice_offset, combined,
                                  dev->stream);
  });
}

agpu_status agpu_upsample_nearest2d(agpu_device* dev, const agpu_buffer* input, uint32_t batch,
                                    uint32_t channels, uint32_t in_h, uint32_t in_w,
                                    uint32_t scale_h, uint32_t scale_w, agpu_buffer** out) {
  CHECK_DEV(dev, "upsample_nearest2d");
  CHECK_BUF(input, "upsample_nearest2d", "input");
  CHECK_OUT(out, "upsample_nearest2d");
  const uint64_t planes = (uint64_t)batch * channels;
  CHECK_LEN(input, planes * in_h * in_w, "upsample_nearest2d", "input");  // upsample.rs:101
  const uint64_t total = planes * in_h * scale_h * in_w * scale_w;
  return with_output(dev, total, out, [&](float* o) {
    return launch_upsample_nearest2d(dev, input->dptr, o, planes, in_h, in_w, scale_h, scale_w,
                                     dev->stream);
  });
}

agpu_status agpu_upsample_nearest2d_backward(agpu_device* dev, const agpu_buffer* grad_out,
                                             uint32_t batch, uint32_t channels, uint32_t in_h,
                                             uint32_t in_w, uint32_t scale_h, uint32_t scale_w,
                                             agpu_buffer** out) {
  CHECK_DEV(dev, "upsample_nearest2d_backward");
  CHECK_BUF(grad_out, "upsample_nearest2d_backward", "grad_out");
  CHECK_OUT(out, "upsample_nearest2d_backward");
  const uint64_t planes = (uint64_t)batch * channels;
  // src/ops/upsample.rs:124
  CHECK_LEN(grad_out, planes * in_h * scale_h * in_w * scale_w, "upsample_nearest2d_backward",
            "grad_out");
  return with_output(dev, planes * in_h * in_w, out, [&](float* o) {
    return launch_upsample_nearest2d_backward(dev, grad_out->dptr, o, planes, in_h, in_w,
                                              scale_h, scale_w, dev->stream);
  });
}

agpu_status agpu_mse_loss(agpu_device* dev, const agpu_buffer* pred, const agpu_buffer* target,
                          agpu_buffer** out) {
  CHECK_DEV(dev, "mse_loss");
  CHECK_BUF(pred, "mse_loss", "pred");
  CHECK_BUF(target, "mse_loss", "target");
  CHECK_OUT(out, "mse_loss");
  CHECK_LEN(target, pred->len, "mse_loss", "target");  // src/ops/attention.rs:173
  return with_output(dev, 1, out, [&](float* o) {
    return launch_mse_loss(dev, pred->dptr, target->dptr, o, pred->len, dev->stream);
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

agpu_status agpu_launch_conv2d(agpu_device* dev, const float* input, const float* weight,
                               const float* bias, float* out, uint32_t batch, uint32_t in_c,
                               uint32_t in_h, uint32_t in_w, uint32_t out_c, uint32_t kh,
                               uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ph, uint32_t pw,
                               uint32_t dh, uint32_t dw, uint32_t groups, void* stream) {
  CHECK_DEV(dev, "launch_conv2d");
  ConvParams p;
  AGPU_TRY(conv_geometry(batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, dh, dw, groups,
                         &p, "launch_conv2d"));
  return launch_conv2d(dev, p, input, weight, bias, out, pick_stream(dev, stream));
}

agpu_status agpu_launch_batch_matmul_softmax(agpu_device* dev, const float* a, const float* b,
                                             float* out, uint32_t batch, uint32_t m, uint32_t n,
                                             uint32_t k, void* stream) {
  CHECK_DEV(dev, "launch_batch_matmul_softmax");
  if ((!a || !b || !out) && (uint64_t)batch * m * n)
    return fail(AGPU_ERR_INVALID, "launch_batch_matmul_softmax: NULL pointer");
  if ((uint64_t)batch * m * n == 0) return AGPU_OK;
  return bmm_softmax(dev, a, b, out, batch, m, n, k, pick_stream(dev, stream));
}

agpu_status agpu_launch_conv2d_group_norm_swish(
    agpu_device* dev, const float* input, const float* weight, const float* bias, float* out,
    uint32_t batch, uint32_t in_c, uint32_t in_h, uint32_t in_w, uint32_t out_c, uint32_t kh,
    uint32_t kw, uint32_t sh, uint32_t sw, uint32_t ph, uint32_t pw, uint32_t dh, uint32_t dw,
    uint32_t groups, const float* gamma, const float* beta, uint32_t gn_groups, float eps,
    void* stream) {
  CHECK_DEV(dev, "launch_conv2d_group_norm_swish");
  ConvParams p;
  AGPU_TRY(conv_geometry(batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, dh, dw, groups,
                         &p, "launch_conv2d_group_norm_swish"));
  if (gn_groups == 0 || out_c % gn_groups != 0)
    return fail(AGPU_ERR_SHAPE,
                "launch_conv2d_group_norm_swish: channels must be divisible by groups");
  const GnEpilogue gn{gamma, beta, gn_groups, eps, true};
  return launch_conv2d_gn(dev, p, input, weight, bias, out, gn, pick_stream(dev, stream));
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

agpu_status agpu_launch_group_norm_backward(agpu_device* dev, const float* grad_out,
                                            const float* input, const float* gamma,
                                            float* d_input, float* d_gamma, float* d_beta,
                                            uint32_t batch, uint32_t channels, uint32_t spatial,
                                            uint32_t groups, float eps, void* stream) {
  CHECK_DEV(dev, "launch_group_norm_backward");
  if (groups == 0 || channels % groups != 0)
    return fail(AGPU_ERR_SHAPE, "launch_group_norm_backward: channels must be divisible by groups");
  return launch_group_norm_backward(dev, grad_out, input, gamma, d_input, d_gamma, d_beta, batch,
                                    channels, spatial, groups, eps, pick_stream(dev, stream));
}

agpu_status agpu_launch_adamw(agpu_device* dev, const agpu_adamw_tensor* tensors,
                              uint32_t count, float lr, float beta1, float beta2, float eps,
                              float weight_decay, uint32_t step, void* stream) {
  CHECK_DEV(dev, "launch_adamw");
  if (count && !tensors) return fail(AGPU_ERR_INVALID, "launch_adamw: NULL tensor array");
  return launch_adamw(dev, tensors, count, lr, beta1, beta2, eps, weight_decay, step,
                      pick_stream(dev, stream));
}

agpu_status agpu_launch_sdpa(agpu_device* dev, const float* q, const float* k, const float* v,
                             float* out, uint32_t bh, uint32_t s, uint32_t d, int causal,
                             void* stream) {
  CHECK_DEV(dev, "launch_sdpa");
  return launch_attention(dev, q, k, v, out, bh, s, d, causal != 0, pick_stream(dev, stream));
}

agpu_status agpu_launch_sdpa_backward(agpu_device* dev, const float* q, const float* k,
                                      const float* v, const float* grad_out, float* d_q,
                                      float* d_k, float* d_v, uint32_t bh, uint32_t s, uint32_t d,
                                      int causal, void* stream) {
  CHECK_DEV(dev, "launch_sdpa_backward");
  if ((!q || !k || !v || !grad_out || !d_q || !d_k || !d_v) && (uint64_t)bh * s * d)
    return fail(AGPU_ERR_INVALID, "launch_sdpa_backward: NULL pointer");
  return launch_attention_backward(dev, q, k, v, grad_out, d_q, d_k, d_v, bh, s, d, causal != 0,
                                   pick_stream(dev, stream));
}

agpu_status agpu_launch_gemm_ex(agpu_device* dev, const float* a, const float* b, float* c,
                                uint32_t batch, uint32_t m, uint32_t n, uint32_t k, int trans_a,
                                int trans_b, const float* bias, const float* resid, int act,
                                void* stream) {
  CHECK_DEV(dev, "launch_gemm_ex");
  if ((!a || !b || !c) && (uint64_t)batch * m * n)
    return fail(AGPU_ERR_INVALID, "launch_gemm_ex: NULL pointer");
  if (act < 0 || act > 3) return fail(AGPU_ERR_INVALID, "launch_gemm_ex: unknown activation");
  if (act == 3 && (n % 64 != 0 || bias || resid))
    return fail(AGPU_ERR_SHAPE, "launch_gemm_ex: SwiGLU needs n %% 64 == 0 and no bias or residual");
  GemmEpilogue ep;
  ep.bias = bias;
  ep.resid = resid;
  ep.act = act;
  return launch_gemm_ex(dev, a, b, c, batch, m, n, k, trans_a != 0, trans_b != 0, ep,
                        pick_stream(dev, stream));
}

agpu_status agpu_launch_sdpa_strided(agpu_device* dev, const float* q, const float* k,
                                     const float* v, float* out, uint32_t batch, uint32_t heads,
                                     uint32_t seq, uint32_t d, const agpu_attn_layout* ql,
                                     const agpu_attn_layout* kl, const agpu_attn_layout* vl,
                                     const agpu_attn_layout* ol, int causal, void* stream) {
  CHECK_DEV(dev, "launch_sdpa_strided");
  if (!ql || !kl || !vl || !ol) return fail(AGPU_ERR_INVALID, "launch_sdpa_strided: NULL layout");
  auto cv = [](const agpu_attn_layout* l, long long (&s)[3]) {
    s[0] = (long long)l->seq_stride;
    s[1] = (long long)l->head_stride;
    s[2] = (long long)l->batch_stride;
  };
  long long qs[3], ks[3], vs[3], os[3];
  cv(ql, qs); cv(kl, ks); cv(vl, vs); cv(ol, os);
  return launch_attention_strided(dev, q, k, v, out, batch, heads, seq, d, qs, ks, vs, os,
                                  causal != 0, pick_stream(dev, stream));
}

agpu_status agpu_launch_rmsnorm(agpu_device* dev, const float* x, const float* w, float* y,
                                uint64_t rows, uint32_t cols, float eps, void* stream) {
  CHECK_DEV(dev, "launch_rmsnorm");
  return launch_rmsnorm(dev, x, w, y, rows, cols, eps, pick_stream(dev, stream));
}

agpu_status agpu_launch_rope(agpu_device* dev, const float* x, float* y, uint32_t batch,
                             uint32_t seq, uint32_t heads, uint32_t dim, uint64_t row_stride,
                             float base, void* stream) {
  CHECK_DEV(dev, "launch_rope");
  if (row_stride < (uint64_t)heads * dim)
    return fail(AGPU_ERR_SHAPE, "launch_rope: row stride smaller than heads * dim");
  return launch_rope(dev, x, y, batch, seq, heads, dim, row_stride, base,
                     pick_stream(dev, stream));
}

agpu_status agpu_launch_swish_mul(agpu_device* dev, const float* gate, const float* up,
                                  float* out, uint64_t rows, uint32_t cols, uint64_t gs,
                                  uint64_t us, uint64_t os, void* stream) {
  CHECK_DEV(dev, "launch_swish_mul");
  if (gs < cols || us < cols || os < cols)
    return fail(AGPU_ERR_SHAPE, "launch_swish_mul: row stride smaller than cols");
  return launch_swish_mul(dev, gate, up, out, rows, cols, gs, us, os, pick_stream(dev, stream));
}

agpu_status agpu_launch_softmax(agpu_device* dev, const float* x, float* y, uint64_t rows,
                                uint32_t cols, void* stream) {
  CHECK_DEV(dev, "launch_softmax");
  if ((!x || !y) && rows * cols) return fail(AGPU_ERR_INVALID, "launch_softmax: NULL pointer");
  return launch_softmax(dev, x, y, rows, cols, pick_stream(dev, stream));
}

}  // extern "C"
