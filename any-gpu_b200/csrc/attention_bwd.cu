// Backward of scaled_dot_product_attention: dQ, dK, dV from dO.
//
// The reference has no attention node on its tape; differentiating its SDPA
// composition (src/ops/attention.rs:149-169: transpose(K) -> batch_matmul ->
// scale -> softmax -> batch_matmul) with its own rules -- the matmul rule of
// src/autograd.rs:357-366 (dA = dC B^T, dB = A^T dC) for both products, the
// scale rule, and the softmax Jacobian-vector product -- gives, per head,
//
//   S  = Q K^T,  P = softmax(scale * S)          (recomputed, causal mask 0)
//   dV = P^T dO                                  (matmul rule, second product)
//   dP = dO V^T
//   dS = scale * P o (dP - rowsum(P o dP))       (softmax rule, then scale)
//   dQ = dS K,   dK = dS^T Q                     (matmul rule, first product)
//
// The five products run on the tensor-core GEMMs (launch_gemm: tcgen05 in
// TF32, 3xTF32 or exact FFMA per the precision mode), with the transposes
// folded into operand majors -- kind::tf32 reads either major -- so no
// transpose pass.  Heads are processed in chunks of at most 2^30 score
// elements.  Two ways, the same math:
//
//  * TF32 where the CTA-pair kernels run both the forward and the S-sized
//    products (S >= 256, d 64 or 128): the forward is rerun to give each
//    row's log-sum-exp L and O; D = rowsum(dO o O) (= rowsum(P o dP), since
//    O = P V); then P = 2^(S * scale * log2 e - L) is formed in the S
//    product's epilogue and dS = P o (dP - D) * scale in the dP product's
//    epilogue, in place over P -- no row pass over the [heads, S, S]
//    matrices and one such buffer instead of two;
//  * otherwise P and dP/dS in two [heads, S, S] pool buffers and the two row
//    kernels below (probabilities, softmax backward), HBM-bound: one block
//    per row (grid-stride), each row read once from HBM and again from cache.
//    AGPU_SDPA_BWD_FUSED=0 in the environment keeps this way for every shape.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "agpu_internal.cuh"

namespace agpu {

namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < kRowThreads / 32 ? red[lane] : -INFINITY;
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < kRowThreads / 32 ? red[lane] : 0.f;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// In place over rows of `cols` scores: P = exp(scale*x - max) / sum over the
// row's unmasked columns (causal: column j of query row i = row % seq is
// masked when j > i), masked entries 0.  Grid-stride over rows.
__global__ void __launch_bounds__(kRowThreads) attn_probs_kernel(float* __restrict__ p,
                                                                 long long rows, int cols,
                                                                 int seq, float scale,
                                                                 int causal) {
  __shared__ float red[kRowThreads / 32];
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    float* x = p + r * (long long)cols;
    const int lim = causal ? (int)(r % seq) + 1 : cols;  // columns [0, lim) are live
    float m = -INFINITY;
    for (int j = threadIdx.x; j < lim; j += kRowThreads) m = fmaxf(m, scale * x[j]);
    m = block_reduce_max(m, red);
    float s = 0.f;
    for (int j = threadIdx.x; j < lim; j += kRowThreads) s += expf(scale * x[j] - m);
    s = block_reduce_sum(s, red);
    const float inv = 1.0f / s;
    for (int j = threadIdx.x; j < cols; j += kRowThreads)
      x[j] = j < lim ? expf(scale * x[j] - m) * inv : 0.f;
  }
}

// In place over rows: dp <- scale * p * (dp - sum_j p*dp)  (the softmax
// Jacobian-vector product, then the scale rule).  Grid-stride over rows.
__global__ void __launch_bounds__(kRowThreads) attn_softmax_bwd_kernel(
    const float* __restrict__ p, float* __restrict__ dp, long long rows, int cols, float scale) {
  __shared__ float red[kRowThreads / 32];
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* pr = p + r * (long long)cols;
    float* g = dp + r * (long long)cols;
    float dot = 0.f;
    for (int j = threadIdx.x; j < cols; j += kRowThreads) dot += pr[j] * g[j];
    dot = block_reduce_sum(dot, red);
    for (int j = threadIdx.x; j < cols; j += kRowThreads) g[j] = scale * pr[j] * (g[j] - dot);
  }
}

// D[r] = sum_c dO[r, c] * O[r, c]: one warp per row of d (64 or 128) floats.
__global__ void __launch_bounds__(256) attn_rowdot_kernel(const float* __restrict__ a,
                                                          const float* __restrict__ b,
                                                          float* __restrict__ out, long long rows,
                                                          int d) {
  const long long r = (long long)blockIdx.x * 8 + threadIdx.x / 32;
  if (r >= rows) return;
  const int lane = threadIdx.x % 32;
  const float* x = a + r * d;
  const float* y = b + r * d;
  float acc = 0.f;
  for (int c = lane * 2; c < d; c += 64) {
    const float2 u = *reinterpret_cast<const float2*>(x + c);
    const float2 w = *reinterpret_cast<const float2*>(y + c);
    acc += u.x * w.x + u.y * w.y;
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[r] = acc;
}

bool bwd_fused_enabled() {
  static const bool on = [] {
    const char* e = getenv("AGPU_SDPA_BWD_FUSED");
    return !(e && e[0] == '0');
  }();
  return on;
}

}  // namespace

agpu_status launch_attention_backward(agpu_device* dev, const float* q, const float* k,
                                      const float* v, const float* dout, float* dq, float* dk,
                                      float* dv, uint32_t bh, uint32_t s, uint32_t d,
                                      bool causal, cudaStream_t st) {
  if ((uint64_t)bh * s * d == 0) return AGPU_OK;
  const float scale = 1.0f / std::sqrt((float)d);
  const uint64_t ss = (uint64_t)s * s;
  const uint64_t chunk = std::max<uint64_t>(1, std::min<uint64_t>(bh, (1ull << 30) / ss));
  // the epilogue way: every chunk's S-sized products on the pair kernel (the
  // last, smaller chunk included) and the forward on CTA pairs
  const uint32_t last = (uint32_t)(bh - (bh - 1) / chunk * chunk);
  // decided before anything launches: every operand 16-byte aligned (each
  // head's [s, d] block then is too), so no product of a later chunk refuses
  const bool aligned = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(dout)) &
                        15u) == 0;
  const bool fused = bwd_fused_enabled() && effective_precision(dev) == AGPU_PREC_TF32 &&
                     aligned && (d == 64 || d == 128) && s >= 256 && s % 4 == 0 &&
                     gemm_rowvec_mode_ok(dev, q, k, q, (uint32_t)std::min<uint64_t>(chunk, bh),
                                         s, s, d) &&
                     gemm_rowvec_mode_ok(dev, q, k, q, last, s, s, d);
  if (fused) {
    const uint64_t od = chunk * s * d, rows_max = chunk * s;
    void *pbuf = nullptr, *obuf = nullptr;
    AGPU_TRY(pool_alloc(dev, chunk * ss * sizeof(float), &pbuf, st));
    agpu_status rc = pool_alloc(dev, (od + 2 * rows_max) * sizeof(float), &obuf, st);
    if (rc != AGPU_OK) {
      pool_free(dev, pbuf, st);
      return rc;
    }
    float* P = static_cast<float*>(pbuf);
    float* O = static_cast<float*>(obuf);
    float* L = O + od;           // od % 4 == 0: 16-byte aligned
    float* Dv = L + rows_max;    // rows_max % 4 == 0 (s % 4 == 0)
    for (uint64_t h0 = 0; h0 < bh && rc == AGPU_OK; h0 += chunk) {
      const uint32_t n = (uint32_t)std::min<uint64_t>(chunk, bh - h0);
      const uint64_t off = h0 * s * d;
      const long long rows = (long long)n * s;
      // forward rerun: O and each row's log-sum-exp
      rc = launch_attention_lse(dev, q + off, k + off, v + off, O, L, n, s, d, causal, st);
      if (rc != AGPU_OK) break;
      attn_rowdot_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, st>>>(dout + off, O, Dv, rows,
                                                                      (int)d);
      rc = after_launch(dev, "attn_rowdot_kernel");
      // P = 2^(Q K^T * scale * log2 e - L), masked above the diagonal if causal
      GemmEpilogue e1;
      e1.mode = 1;
      e1.rowvec = L;
      e1.scale = scale * 1.4426950408889634f;
      e1.causal = causal;
      if (rc == AGPU_OK) rc = launch_gemm_ex(dev, q + off, k + off, P, n, s, s, d, false, true, e1, st);
      // dV = P^T dO
      if (rc == AGPU_OK) rc = launch_gemm(dev, P, dout + off, dv + off, n, s, d, s, true, false, st);
      // dS = P o (dO V^T - D) * scale, in place over P
      GemmEpilogue e2;
      e2.mode = 2;
      e2.rowvec = Dv;
      e2.scale = scale;
      if (rc == AGPU_OK) rc = launch_gemm_ex(dev, dout + off, v + off, P, n, s, s, d, false, true, e2, st);
      // dQ = dS K;  dK = dS^T Q
      if (rc == AGPU_OK) rc = launch_gemm(dev, P, k + off, dq + off, n, s, d, s, false, false, st);
      if (rc == AGPU_OK) rc = launch_gemm(dev, P, q + off, dk + off, n, s, d, s, true, false, st);
    }
    pool_free(dev, obuf, st);
    pool_free(dev, pbuf, st);
    return rc;
  }
  void *pbuf = nullptr, *gbuf = nullptr;
  AGPU_TRY(pool_alloc(dev, chunk * ss * sizeof(float), &pbuf, st));
  agpu_status rc = pool_alloc(dev, chunk * ss * sizeof(float), &gbuf, st);
  if (rc != AGPU_OK) {
    pool_free(dev, pbuf, st);
    return rc;
  }
  float* P = static_cast<float*>(pbuf);
  float* G = static_cast<float*>(gbuf);
  const long long row_grid_cap = 32LL * dev->sm_count;
  for (uint64_t h0 = 0; h0 < bh && rc == AGPU_OK; h0 += chunk) {
    const uint32_t n = (uint32_t)std::min<uint64_t>(chunk, bh - h0);
    const uint64_t off = h0 * s * d;
    const long long rows = (long long)n * s;
    const unsigned grid = (unsigned)std::min<long long>(rows, row_grid_cap);
    // S = Q K^T, then P in place
    rc = launch_gemm(dev, q + off, k + off, P, n, s, s, d, false, true, st);
    if (rc != AGPU_OK) break;
    attn_probs_kernel<<<grid, kRowThreads, 0, st>>>(P, rows, (int)s, (int)s, scale,
                                                    causal ? 1 : 0);
    rc = after_launch(dev, "attn_probs_kernel");
    // dV = P^T dO (P stored [queries, keys] = A^T)
    if (rc == AGPU_OK) rc = launch_gemm(dev, P, dout + off, dv + off, n, s, d, s, true, false, st);
    // dP = dO V^T, then dS in place
    if (rc == AGPU_OK) rc = launch_gemm(dev, dout + off, v + off, G, n, s, s, d, false, true, st);
    if (rc != AGPU_OK) break;
    attn_softmax_bwd_kernel<<<grid, kRowThreads, 0, st>>>(P, G, rows, (int)s, scale);
    rc = after_launch(dev, "attn_softmax_bwd_kernel");
    // dQ = dS K;  dK = dS^T Q
    if (rc == AGPU_OK) rc = launch_gemm(dev, G, k + off, dq + off, n, s, d, s, false, false, st);
    if (rc == AGPU_OK) rc = launch_gemm(dev, G, q + off, dk + off, n, s, d, s, true, false, st);
  }
  pool_free(dev, gbuf, st);
  pool_free(dev, pbuf, st);
  return rc;
}

}  // namespace agpu
