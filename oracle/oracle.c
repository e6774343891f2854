/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference's
 * own CPU implementations of the dense-op hot path of any-gpu (Rust crate,
 * file:line cited per function), used by tests/ as the parity checker and by
 * bench.py's cpu_baseline / --impl reference leg as the timed CPU path.
 * Nothing in the product (libagpu.so, any_gpu/) links or calls this.
 *
 * Arithmetic matches the Rust code: f32 throughout, the same loop order, a
 * separate multiply and add per step (built with -ffp-contract=off, as rustc
 * does not fuse a*b+c), f32 exp/sqrt from libm.
 *
 * Where the reference's CPU helper is silent, the WGSL shader fixes the
 * semantics and is restated instead (dilation in conv2d, conv_transpose2d,
 * conv2d grad weight/bias, group_norm backward, transpose index map).
 * RMSNorm and RoPE have no reference implementation at all: they are the
 * standard formulas and their parity is unpinned.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <unistd.h>

/* ------------------------------------------------ parallel-for (pthreads) --
 * The *_mt variants split their outermost independent loop into contiguous
 * chunks, one per host thread; every output element is computed by exactly
 * the same sequential arithmetic as the single-thread function. */
int oracle_num_threads(void) {
  const char* env = getenv("ORACLE_THREADS");
  if (env && atoi(env) > 0) return atoi(env);
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

typedef void (*range_fn)(void* ctx, int64_t begin, int64_t end);
typedef struct { range_fn fn; void* ctx; int64_t begin, end; } range_job;

static void* range_thread(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->begin, j->end);
  return NULL;
}

static void parallel_for(int64_t n, range_fn fn, void* ctx) {
  int nt = oracle_num_threads();
  if (nt > n) nt = (int)n;
  if (nt <= 1) { fn(ctx, 0, n); return; }
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nt);
  range_job* jobs = (range_job*)malloc(sizeof(range_job) * nt);
  for (int t = 0; t < nt; ++t) {
    jobs[t].fn = fn; jobs[t].ctx = ctx;
    jobs[t].begin = n * t / nt; jobs[t].end = n * (t + 1) / nt;
    pthread_create(&th[t], NULL, range_thread, &jobs[t]);
  }
  for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
  free(th); free(jobs);
}

/* cpu_matmul: src/ops/conv.rs:575-585, examples/bench.rs:10-22 */
void oracle_matmul(const float* a, const float* b, float* out, int64_t m, int64_t n, int64_t k) {
  for (int64_t row = 0; row < m; ++row)
    for (int64_t col = 0; col < n; ++col) {
      float sum = 0.0f;
      for (int64_t i = 0; i < k; ++i) sum += a[row * k + i] * b[i * n + col];
      out[row * n + col] = sum;
    }
}

/* Same arithmetic per output element, rows split across host threads:
 * the multi-core variant of the timed CPU baseline. */
typedef struct { const float *a, *b; float* out; int64_t m, n, k; } mm_ctx;

static void mm_rows(void* p, int64_t r0, int64_t r1) {
  const mm_ctx* c = (const mm_ctx*)p;
  /* rows of all batches flattened: row index r covers batch r / m */
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t bat = r / c->m, row = r % c->m;
    const float* ar = c->a + bat * c->m * c->k + row * c->k;
    const float* bb = c->b + bat * c->k * c->n;
    float* o = c->out + bat * c->m * c->n + row * c->n;
    for (int64_t col = 0; col < c->n; ++col) {
      float sum = 0.0f;
      for (int64_t i = 0; i < c->k; ++i) sum += ar[i] * bb[i * c->n + col];
      o[col] = sum;
    }
  }
}

void oracle_matmul_mt(const float* a, const float* b, float* out, int64_t m, int64_t n,
                      int64_t k) {
  mm_ctx c = {a, b, out, m, n, k};
  parallel_for(m, mm_rows, &c);
}

/* batch loop of test_batch_matmul_vs_cpu: src/ops/conv.rs:850-861 */
void oracle_batch_matmul(const float* a, const float* b, float* out, int64_t batch, int64_t m,
                         int64_t n, int64_t k) {
  for (int64_t bat = 0; bat < batch; ++bat)
    oracle_matmul(a + bat * m * k, b + bat * k * n, out + bat * m * n, m, n, k);
}

void oracle_batch_matmul_mt(const float* a, const float* b, float* out, int64_t batch, int64_t m,
                            int64_t n, int64_t k) {
  mm_ctx c = {a, b, out, m, n, k};
  parallel_for(batch * m, mm_rows, &c);
}

/* cpu_softmax: src/ops/attention.rs:193-205.  max is a fold from -inf with
 * f32::max; the sum is the in-order iterator sum of exp(x - max). */
static void softmax_row(const float* row, float* out, int64_t cols) {
  float mx = -INFINITY;
  for (int64_t c = 0; c < cols; ++c) mx = fmaxf(mx, row[c]);
  float sum = 0.0f;
  for (int64_t c = 0; c < cols; ++c) sum += expf(row[c] - mx);
  for (int64_t c = 0; c < cols; ++c) out[c] = expf(row[c] - mx) / sum;
}

void oracle_softmax(const float* x, float* out, int64_t rows, int64_t cols) {
  for (int64_t r = 0; r < rows; ++r) softmax_row(x + r * cols, out + r * cols, cols);
}

typedef struct { const float* x; float* out; int64_t cols; } sm_ctx;

static void sm_rows(void* p, int64_t r0, int64_t r1) {
  const sm_ctx* c = (const sm_ctx*)p;
  for (int64_t r = r0; r < r1; ++r) softmax_row(c->x + r * c->cols, c->out + r * c->cols, c->cols);
}

void oracle_softmax_mt(const float* x, float* out, int64_t rows, int64_t cols) {
  sm_ctx c = {x, out, cols};
  parallel_for(rows, sm_rows, &c);
}

/* cpu_attention: src/ops/attention.rs:208-229, one head of [seq, dk]. */
static void attention_head(const float* q, const float* k, const float* v, float* out,
                           int64_t seq, int64_t dk, float* scores) {
  const float scale = 1.0f / sqrtf((float)dk);
  for (int64_t i = 0; i < seq; ++i)
    for (int64_t j = 0; j < seq; ++j) {
      float s = 0.0f;
      for (int64_t d = 0; d < dk; ++d) s += q[i * dk + d] * k[j * dk + d];
      scores[i * seq + j] = s * scale;
    }
  oracle_softmax(scores, scores, seq, seq);
  for (int64_t i = 0; i < seq; ++i)
    for (int64_t d = 0; d < dk; ++d) {
      float s = 0.0f;
      for (int64_t j = 0; j < seq; ++j) s += scores[i * seq + j] * v[j * dk + d];
      out[i * dk + d] = s;
    }
}

/* SDPA over batch_heads independent heads (the reference op's semantics,
 * src/ops/attention.rs:149-169), each head restated with cpu_attention. */
void oracle_attention(const float* q, const float* k, const float* v, float* out, int64_t bh,
                      int64_t seq, int64_t dk) {
  float* scores = (float*)malloc(sizeof(float) * seq * seq);
  for (int64_t h = 0; h < bh; ++h)
    attention_head(q + h * seq * dk, k + h * seq * dk, v + h * seq * dk, out + h * seq * dk, seq,
                   dk, scores);
  free(scores);
}

typedef struct { const float *q, *k, *v; float* out; int64_t seq, dk; } at_ctx;

static void at_heads(void* p, int64_t h0, int64_t h1) {
  const at_ctx* c = (const at_ctx*)p;
  const int64_t sz = c->seq * c->dk;
  float* scores = (float*)malloc(sizeof(float) * c->seq * c->seq);
  for (int64_t h = h0; h < h1; ++h)
    attention_head(c->q + h * sz, c->k + h * sz, c->v + h * sz, c->out + h * sz, c->seq, c->dk,
                   scores);
  free(scores);
}

void oracle_attention_mt(const float* q, const float* k, const float* v, float* out, int64_t bh,
                         int64_t seq, int64_t dk) {
  at_ctx c = {q, k, v, out, seq, dk};
  parallel_for(bh, at_heads, &c);
}

/* Causal variant (not in the reference; standard formula): position i only
 * attends to j <= i.  Parity unpinned. */
void oracle_attention_causal(const float* q, const float* k, const float* v, float* out,
                             int64_t bh, int64_t seq, int64_t dk) {
  float* scores = (float*)malloc(sizeof(float) * seq * seq);
  const float scale = 1.0f / sqrtf((float)dk);
  for (int64_t h = 0; h < bh; ++h) {
    const float* qh = q + h * seq * dk;
    const float* kh = k + h * seq * dk;
    const float* vh = v + h * seq * dk;
    float* oh = out + h * seq * dk;
    for (int64_t i = 0; i < seq; ++i) {
      for (int64_t j = 0; j <= i; ++j) {
        float s = 0.0f;
        for (int64_t d = 0; d < dk; ++d) s += qh[i * dk + d] * kh[j * dk + d];
        scores[j] = s * scale;
      }
      softmax_row(scores, scores, i + 1);
      for (int64_t d = 0; d < dk; ++d) {
        float s = 0.0f;
        for (int64_t j = 0; j <= i; ++j) s += scores[j] * vh[j * dk + d];
        oh[i * dk + d] = s;
      }
    }
  }
  free(scores);
}

/* conv2d output size with dilation: src/ops/conv.rs:447-448. */
int64_t oracle_conv_out(int64_t in, int64_t k, int64_t stride, int64_t pad, int64_t dil) {
  return (in + 2 * pad - dil * (k - 1) - 1) / stride + 1;
}

/* cpu_conv2d: src/ops/conv.rs:588-628, with the shader's dilation term
 * (src/ops/conv.rs:204-205) added; the CPU helper itself assumes dilation 1. */
typedef struct {
  const float *input, *weight, *bias;
  float* out;
  int64_t batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, dh, dw, groups;
} conv_ctx;

static void conv_range(void* p, int64_t j0, int64_t j1) {
  const conv_ctx* c = (const conv_ctx*)p;
  const float *input = c->input, *weight = c->weight, *bias = c->bias;
  float* out = c->out;
  const int64_t in_c = c->in_c, in_h = c->in_h, in_w = c->in_w, out_c = c->out_c;
  const int64_t kh = c->kh, kw = c->kw, sh = c->sh, sw = c->sw, ph = c->ph, pw = c->pw;
  const int64_t dh = c->dh, dw = c->dw;
  const int64_t out_h = oracle_conv_out(in_h, kh, sh, ph, dh);
  const int64_t out_w = oracle_conv_out(in_w, kw, sw, pw, dw);
  const int64_t group_in = in_c / c->groups, group_out = out_c / c->groups;
  for (int64_t j = j0; j < j1; ++j) {
    const int64_t n = j / out_c, oc = j % out_c;
    {
      const int64_t g = oc / group_out;
      for (int64_t oh = 0; oh < out_h; ++oh)
        for (int64_t ow = 0; ow < out_w; ++ow) {
          float sum = bias ? bias[oc] : 0.0f;
          for (int64_t ic = 0; ic < group_in; ++ic)
            for (int64_t kr = 0; kr < kh; ++kr)
              for (int64_t kc = 0; kc < kw; ++kc) {
                const int64_t ih = oh * sh + kr * dh - ph;
                const int64_t iw = ow * sw + kc * dw - pw;
                if (ih >= 0 && ih < in_h && iw >= 0 && iw < in_w) {
                  const int64_t in_idx =
                      n * in_c * in_h * in_w + (g * group_in + ic) * in_h * in_w + ih * in_w + iw;
                  const int64_t w_idx = oc * group_in * kh * kw + ic * kh * kw + kr * kw + kc;
                  sum += input[in_idx] * weight[w_idx];
                }
              }
          out[n * out_c * out_h * out_w + oc * out_h * out_w + oh * out_w + ow] = sum;
        }
    }
  }
}

static void conv2d_impl(const float* input, const float* weight, const float* bias, float* out,
                        int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w, int64_t out_c,
                        int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                        int64_t dh, int64_t dw, int64_t groups, int parallel) {
  conv_ctx c = {input, weight, bias, out, batch, in_c, in_h, in_w, out_c,
                kh, kw, sh, sw, ph, pw, dh, dw, groups};
  if (parallel) parallel_for(batch * out_c, conv_range, &c);
  else conv_range(&c, 0, batch * out_c);
}

void oracle_conv2d(const float* input, const float* weight, const float* bias, float* out,
                   int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w, int64_t out_c,
                   int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                   int64_t dh, int64_t dw, int64_t groups) {
  conv2d_impl(input, weight, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw,
              dh, dw, groups, 0);
}

void oracle_conv2d_mt(const float* input, const float* weight, const float* bias, float* out,
                      int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w, int64_t out_c,
                      int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                      int64_t dh, int64_t dw, int64_t groups) {
  conv2d_impl(input, weight, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw,
              dh, dw, groups, 1);
}

/* SHADER_CONV_TRANSPOSE2D semantics: src/ops/conv.rs:245-296, output size
 * src/ops/conv.rs:498-499.  Weight layout [in_c, out_c/groups, kh, kw]. */
void oracle_conv_transpose2d(const float* input, const float* weight, const float* bias,
                             float* out, int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w,
                             int64_t out_c, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                             int64_t ph, int64_t pw, int64_t oph, int64_t opw, int64_t dh,
                             int64_t dw, int64_t groups) {
  const int64_t out_h = (in_h - 1) * sh - 2 * ph + dh * (kh - 1) + oph + 1;
  const int64_t out_w = (in_w - 1) * sw - 2 * pw + dw * (kw - 1) + opw + 1;
  const int64_t group_in = in_c / groups, group_out = out_c / groups;
  for (int64_t n = 0; n < batch; ++n)
    for (int64_t oc = 0; oc < out_c; ++oc) {
      const int64_t g = oc / group_out, oc_local = oc % group_out;
      for (int64_t oh = 0; oh < out_h; ++oh)
        for (int64_t ow = 0; ow < out_w; ++ow) {
          float sum = bias ? bias[oc] : 0.0f;
          for (int64_t ic = 0; ic < group_in; ++ic)
            for (int64_t kr = 0; kr < kh; ++kr)
              for (int64_t kc = 0; kc < kw; ++kc) {
                const int64_t oh_off = oh + ph - kr * dh;
                const int64_t ow_off = ow + pw - kc * dw;
                if (oh_off < 0 || ow_off < 0) continue;  /* u32 wraparound in the shader */
                if (oh_off % sh != 0 || ow_off % sw != 0) continue;
                const int64_t ih = oh_off / sh, iw = ow_off / sw;
                if (ih < in_h && iw < in_w) {
                  const int64_t in_idx =
                      n * in_c * in_h * in_w + (g * group_in + ic) * in_h * in_w + ih * in_w + iw;
                  const int64_t w_idx = (g * group_in + ic) * group_out * kh * kw +
                                        oc_local * kh * kw + kr * kw + kc;
                  sum += input[in_idx] * weight[w_idx];
                }
              }
          out[n * out_c * out_h * out_w + oc * out_h * out_w + oh * out_w + ow] = sum;
        }
    }
}

/* SHADER_CONV2D_GRAD_WEIGHT: src/ops/conv.rs:337-385. */
void oracle_conv2d_grad_weight(const float* input, const float* grad_out, float* grad_w,
                               int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w,
                               int64_t out_c, int64_t out_h, int64_t out_w, int64_t kh,
                               int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                               int64_t dh, int64_t dw, int64_t groups) {
  const int64_t group_in = in_c / groups, group_out = out_c / groups;
  for (int64_t oc = 0; oc < out_c; ++oc)
    for (int64_t ic = 0; ic < group_in; ++ic)
      for (int64_t kr = 0; kr < kh; ++kr)
        for (int64_t kc = 0; kc < kw; ++kc) {
          const int64_t g = oc / group_out;
          float sum = 0.0f;
          for (int64_t n = 0; n < batch; ++n)
            for (int64_t oh = 0; oh < out_h; ++oh)
              for (int64_t ow = 0; ow < out_w; ++ow) {
                const int64_t ih = oh * sh + kr * dh - ph;
                const int64_t iw = ow * sw + kc * dw - pw;
                if (ih >= 0 && iw >= 0 && ih < in_h && iw < in_w) {
                  const int64_t in_idx =
                      n * in_c * in_h * in_w + (g * group_in + ic) * in_h * in_w + ih * in_w + iw;
                  const int64_t go_idx =
                      n * out_c * out_h * out_w + oc * out_h * out_w + oh * out_w + ow;
                  sum += grad_out[go_idx] * input[in_idx];
                }
              }
          grad_w[((oc * group_in + ic) * kh + kr) * kw + kc] = sum;
        }
}

/* SHADER_CONV2D_GRAD_BIAS: src/ops/conv.rs:390-410. */
void oracle_conv2d_grad_bias(const float* grad_out, float* grad_b, int64_t batch, int64_t out_c,
                             int64_t out_h, int64_t out_w) {
  for (int64_t oc = 0; oc < out_c; ++oc) {
    float sum = 0.0f;
    for (int64_t n = 0; n < batch; ++n)
      for (int64_t p = 0; p < out_h * out_w; ++p)
        sum += grad_out[n * out_c * out_h * out_w + oc * out_h * out_w + p];
    grad_b[oc] = sum;
  }
}

/* cpu_group_norm: src/ops/norm.rs:448-480 (E[x^2] - mean^2 variance). */
typedef struct {
  const float *input, *gamma, *beta;
  float* out;
  int64_t channels, spatial, groups;
  float eps;
} gn_ctx;

static void gn_range(void* p, int64_t j0, int64_t j1) {
  const gn_ctx* cx = (const gn_ctx*)p;
  const float *input = cx->input, *gamma = cx->gamma, *beta = cx->beta;
  float* out = cx->out;
  const int64_t channels = cx->channels, spatial = cx->spatial, groups = cx->groups;
  const float eps = cx->eps;
  const int64_t cpg = channels / groups;
  for (int64_t j = j0; j < j1; ++j) {
    const int64_t n = j / groups, g = j % groups;
    {
      float sum = 0.0f, sum_sq = 0.0f;
      const float count = (float)(cpg * spatial);
      for (int64_t c = 0; c < cpg; ++c) {
        const int64_t ch = g * cpg + c;
        for (int64_t s = 0; s < spatial; ++s) {
          const float v = input[n * channels * spatial + ch * spatial + s];
          sum += v;
          sum_sq += v * v;
        }
      }
      const float mean = sum / count;
      const float var = sum_sq / count - mean * mean;
      const float inv_std = 1.0f / sqrtf(var + eps);
      for (int64_t c = 0; c < cpg; ++c) {
        const int64_t ch = g * cpg + c;
        for (int64_t s = 0; s < spatial; ++s) {
          const int64_t idx = n * channels * spatial + ch * spatial + s;
          out[idx] = (input[idx] - mean) * inv_std * gamma[ch] + beta[ch];
        }
      }
    }
  }
}

static void group_norm_impl(const float* input, const float* gamma, const float* beta,
                            float* out, int64_t batch, int64_t channels, int64_t spatial,
                            int64_t groups, float eps, int parallel) {
  gn_ctx c = {input, gamma, beta, out, channels, spatial, groups, eps};
  if (parallel) parallel_for(batch * groups, gn_range, &c);
  else gn_range(&c, 0, batch * groups);
}

void oracle_group_norm(const float* input, const float* gamma, const float* beta, float* out,
                       int64_t batch, int64_t channels, int64_t spatial, int64_t groups,
                       float eps) {
  group_norm_impl(input, gamma, beta, out, batch, channels, spatial, groups, eps, 0);
}

void oracle_group_norm_mt(const float* input, const float* gamma, const float* beta, float* out,
                          int64_t batch, int64_t channels, int64_t spatial, int64_t groups,
                          float eps) {
  group_norm_impl(input, gamma, beta, out, batch, channels, spatial, groups, eps, 1);
}

/* group_norm_backward: SHADER_GN_STATS + BACK_SUMS/DINPUT/DAFFINE,
 * src/ops/norm.rs:22-56, 97-205. */
void oracle_group_norm_backward(const float* grad_out, const float* input, const float* gamma,
                                float* d_input, float* d_gamma, float* d_beta, int64_t batch,
                                int64_t channels, int64_t spatial, int64_t groups, float eps) {
  const int64_t cpg = channels / groups;
  const int64_t ng = batch * groups;
  float* stats = (float*)malloc(sizeof(float) * 2 * ng);
  float* sums = (float*)malloc(sizeof(float) * 2 * ng);
  for (int64_t idx = 0; idx < ng; ++idx) {
    const int64_t g = idx % groups, n = idx / groups;
    float sum = 0.0f, sum_sq = 0.0f;
    for (int64_t c = 0; c < cpg; ++c) {
      const int64_t base = n * channels * spatial + (g * cpg + c) * spatial;
      for (int64_t s = 0; s < spatial; ++s) {
        const float v = input[base + s];
        sum += v;
        sum_sq += v * v;
      }
    }
    const float count = (float)(cpg * spatial);
    const float mean = sum / count;
    const float var = sum_sq / count - mean * mean;
    stats[2 * idx] = mean;
    stats[2 * idx + 1] = 1.0f / sqrtf(var + eps);
    float s1 = 0.0f, s2 = 0.0f;
    for (int64_t c = 0; c < cpg; ++c) {
      const int64_t ch = g * cpg + c;
      const int64_t base = n * channels * spatial + ch * spatial;
      for (int64_t s = 0; s < spatial; ++s) {
        const float dx_hat = grad_out[base + s] * gamma[ch];
        const float x_hat = (input[base + s] - stats[2 * idx]) * stats[2 * idx + 1];
        s1 += dx_hat;
        s2 += dx_hat * x_hat;
      }
    }
    sums[2 * idx] = s1;
    sums[2 * idx + 1] = s2;
  }
  const int64_t total = batch * channels * spatial;
  for (int64_t idx = 0; idx < total; ++idx) {
    const int64_t ch = (idx / spatial) % channels, n = idx / (spatial * channels);
    const int64_t si = n * groups + ch / cpg;
    const float mean = stats[2 * si], inv_std = stats[2 * si + 1];
    const float x_hat = (input[idx] - mean) * inv_std;
    const float dx_hat = grad_out[idx] * gamma[ch];
    const float count = (float)(cpg * spatial);
    d_input[idx] = inv_std * (dx_hat - (sums[2 * si] + x_hat * sums[2 * si + 1]) / count);
  }
  for (int64_t ch = 0; ch < channels; ++ch) {
    const int64_t g = ch / cpg;
    float dg = 0.0f, db = 0.0f;
    for (int64_t n = 0; n < batch; ++n) {
      const int64_t si = n * groups + g;
      const int64_t base = n * channels * spatial + ch * spatial;
      for (int64_t s = 0; s < spatial; ++s) {
        const float x_hat = (input[base + s] - stats[2 * si]) * stats[2 * si + 1];
        dg += grad_out[base + s] * x_hat;
        db += grad_out[base + s];
      }
    }
    d_gamma[ch] = dg;
    d_beta[ch] = db;
  }
  free(stats);
  free(sums);
}

/* cpu_sigmoid / cpu_swish: src/ops/elementwise.rs:260-261. */
float oracle_sigmoid1(float x) { return 1.0f / (1.0f + expf(-x)); }
float oracle_swish1(float x) { return x * oracle_sigmoid1(x); }

/* Elementwise family, the WGSL shader formulas: src/ops/elementwise.rs:9-187.
 * op: 0 add 1 sub 2 mul 3 relu 4 sigmoid 5 swish 6 tanh 7 scale
 *     8 relu_bwd 9 sigmoid_bwd 10 swish_bwd 11 tanh_bwd (a = grad_out, b = saved). */
void oracle_elementwise(int op, const float* a, const float* b, float s, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const float x = a[i];
    float y = 0.0f;
    switch (op) {
      case 0: y = x + b[i]; break;
      case 1: y = x - b[i]; break;
      case 2: y = x * b[i]; break;
      case 3: y = fmaxf(x, 0.0f); break;
      case 4: y = 1.0f / (1.0f + expf(-x)); break;
      case 5: y = x / (1.0f + expf(-x)); break;
      case 6: y = tanhf(x); break;
      case 7: y = x * s; break;
      case 8: y = b[i] > 0.0f ? x : 0.0f; break;
      case 9: y = x * b[i] * (1.0f - b[i]); break;
      case 10: {
        const float t = 1.0f / (1.0f + expf(-b[i]));
        y = x * (t + b[i] * t * (1.0f - t));
        break;
      }
      case 11: y = x * (1.0f - b[i] * b[i]); break;
      default: y = NAN;
    }
    out[i] = y;
  }
}

/* SHADER_TRANSPOSE index map: src/ops/tensor_ops.rs:205-221. */
void oracle_transpose(const float* a, float* out, int64_t outer, int64_t d0, int64_t d1,
                      int64_t inner) {
  const int64_t block = d0 * d1 * inner;
  const int64_t total = outer * block;
  for (int64_t idx = 0; idx < total; ++idx) {
    const int64_t o = idx / block, rem = idx % block;
    const int64_t i1 = rem / (d0 * inner), rem2 = rem % (d0 * inner);
    const int64_t i0 = rem2 / inner, ii = rem2 % inner;
    out[idx] = a[o * block + i0 * (d1 * inner) + i1 * inner + ii];
  }
}

/* SHADER_ADD_PER_COL: src/ops/tensor_ops.rs:143-167. */
void oracle_add_per_col(const float* a, const float* b, float* out, int64_t rows, int64_t cols) {
  for (int64_t i = 0; i < rows * cols; ++i) out[i] = a[i] + b[i % cols];
}

/* SHADER_BROADCAST_ADD: src/ops/tensor_ops.rs:87-100. */
void oracle_add_broadcast(const float* a, const float* b, float* out, int64_t outer,
                          int64_t inner) {
  for (int64_t i = 0; i < outer * inner; ++i) out[i] = a[i] + b[i / inner];
}

/* SHADER_SUM_INNER: src/ops/tensor_ops.rs:113-129 (serial fp32 sum per row). */
void oracle_sum_inner(const float* src, float* out, int64_t outer, int64_t inner) {
  for (int64_t o = 0; o < outer; ++o) {
    float s = 0.0f;
    for (int64_t i = 0; i < inner; ++i) s += src[o * inner + i];
    out[o] = s;
  }
}

/* SHADER_SUM_ROWS: src/ops/tensor_ops.rs:160-176 (serial fp32 sum per column). */
void oracle_sum_rows(const float* src, float* out, int64_t rows, int64_t cols) {
  for (int64_t c = 0; c < cols; ++c) {
    float s = 0.0f;
    for (int64_t r = 0; r < rows; ++r) s += src[r * cols + c];
    out[c] = s;
  }
}

/* SHADER_CONCAT: src/ops/tensor_ops.rs:20-41. */
void oracle_concat(const float* a, const float* b, float* out, int64_t outer, int64_t a_inner,
                   int64_t b_inner) {
  const int64_t w = a_inner + b_inner;
  for (int64_t i = 0; i < outer * w; ++i) {
    const int64_t o = i / w, j = i % w;
    out[i] = j < a_inner ? a[o * a_inner + j] : b[o * b_inner + (j - a_inner)];
  }
}

/* SHADER_SLICE: src/ops/tensor_ops.rs:59-72. */
void oracle_slice_per_block(const float* src, float* dst, int64_t outer, int64_t size,
                            int64_t offset, int64_t combined) {
  for (int64_t i = 0; i < outer * size; ++i)
    dst[i] = src[(i / size) * combined + offset + i % size];
}

/* SHADER_UPSAMPLE_NEAREST: src/ops/upsample.rs:21-45 (ih = oh * in_h / out_h). */
void oracle_upsample_nearest2d(const float* in, float* out, int64_t batch, int64_t channels,
                               int64_t in_h, int64_t in_w, int64_t sh, int64_t sw) {
  const int64_t out_h = in_h * sh, out_w = in_w * sw;
  const int64_t total = batch * channels * out_h * out_w;
  for (int64_t i = 0; i < total; ++i) {
    const int64_t ow = i % out_w, oh = (i / out_w) % out_h, pl = i / (out_w * out_h);
    out[i] = in[(pl * in_h + oh * in_h / out_h) * in_w + ow * in_w / out_w];
  }
}

/* SHADER_UPSAMPLE_NEAREST_BACKWARD: src/ops/upsample.rs:49-78 (dy outer, dx inner). */
void oracle_upsample_nearest2d_backward(const float* go, float* gi, int64_t batch,
                                        int64_t channels, int64_t in_h, int64_t in_w, int64_t sh,
                                        int64_t sw) {
  const int64_t out_h = in_h * sh, out_w = in_w * sw;
  const int64_t total = batch * channels * in_h * in_w;
  for (int64_t i = 0; i < total; ++i) {
    const int64_t iw = i % in_w, ih = (i / in_w) % in_h, pl = i / (in_w * in_h);
    float s = 0.0f;
    for (int64_t dy = 0; dy < sh; ++dy)
      for (int64_t dx = 0; dx < sw; ++dx)
        s += go[pl * out_h * out_w + (ih * sh + dy) * out_w + iw * sw + dx];
    gi[i] = s;
  }
}

/* SHADER_MSE_SUM: src/ops/attention.rs:72-87 (serial fp32 sum, then / f32(n)). */
float oracle_mse_loss(const float* pred, const float* target, int64_t n) {
  float s = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    const float d = pred[i] - target[i];
    s += d * d;
  }
  return s / (float)n;
}

/* RMSNorm (not in the reference; standard formula, parity unpinned):
 * y = x / sqrt(mean(x^2) + eps) * w, per row of `cols`. */
void oracle_rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t cols,
                    float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    float ss = 0.0f;
    for (int64_t c = 0; c < cols; ++c) ss += x[r * cols + c] * x[r * cols + c];
    const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
    for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = x[r * cols + c] * inv * w[c];
  }
}

/* RoPE (not in the reference; standard rotate-half form, parity unpinned).
 * x: [batch, seq, heads, dim]; pair (i, i + dim/2) rotated by angle
 * pos * base^(-2i/dim). */
void oracle_rope(const float* x, float* out, int64_t batch, int64_t seq, int64_t heads,
                 int64_t dim, float base) {
  const int64_t half = dim / 2;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t s = 0; s < seq; ++s)
      for (int64_t h = 0; h < heads; ++h) {
        const float* xi = x + ((b * seq + s) * heads + h) * dim;
        float* o = out + ((b * seq + s) * heads + h) * dim;
        for (int64_t i = 0; i < half; ++i) {
          const double inv_freq = pow((double)base, -2.0 * (double)i / (double)dim);
          const double ang = (double)s * inv_freq;
          const float c = (float)cos(ang), sn = (float)sin(ang);
          const float x0 = xi[i], x1 = xi[i + half];
          o[i] = x0 * c - x1 * sn;
          o[i + half] = x1 * c + x0 * sn;
        }
      }
}

/* f32 powi as Rust lowers it (square-and-multiply in f32). */
static float powi_f32(float a, int64_t b) {
  float r = 1.0f;
  for (;;) {
    if (b & 1) r *= a;
    b >>= 1;
    if (b == 0) break;
    a *= a;
  }
  return r;
}

/* oracle_adamw: one AdamW step on one tensor, SHADER_ADAMW
 * (src/optim.rs:22-51) element by element, with beta^t as AdamW::step
 * computes it (src/optim.rs:84-86: f32 powi). */
void oracle_adamw(float* param, const float* grad, float* m, float* v, int64_t n, float lr,
                  float beta1, float beta2, float eps, float weight_decay, int64_t step) {
  const float b1t = powi_f32(beta1, step), b2t = powi_f32(beta2, step);
  for (int64_t i = 0; i < n; ++i) {
    const float g = grad[i];
    m[i] = beta1 * m[i] + (1.0f - beta1) * g;
    v[i] = beta2 * v[i] + (1.0f - beta2) * g * g;
    const float m_hat = m[i] / (1.0f - b1t);
    const float v_hat = v[i] / (1.0f - b2t);
    param[i] = param[i] * (1.0f - lr * weight_decay) - lr * m_hat / (sqrtf(v_hat) + eps);
  }
}
