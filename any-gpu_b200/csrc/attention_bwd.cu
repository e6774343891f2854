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
// transpose pass.  P and dP/dS live in two [heads, S, S] scratch buffers from
// the device pool, processed in head chunks of at most 2^30 elements each; the
// two row kernels below (probabilities, softmax backward) are HBM-bound: one
// block per row (grid-stride), each row read once from HBM and again from
// cache.
#include <algorithm>
#include <cmath>

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

}  // namespace

agpu_status launch_attention_backward(agpu_device* dev, const float* q, const float* k,
                                      const float* v, const float* dout, float* dq, float* dk,
                                      float* dv, uint32_t bh, uint32_t s, uint32_t d,
                                      bool causal, cudaStream_t st) {
  if ((uint64_t)bh * s * d == 0) return AGPU_OK;
  const float scale = 1.0f / std::sqrt((float)d);
  const uint64_t ss = (uint64_t)s * s;
  const uint64_t chunk = std::max<uint64_t>(1, std::min<uint64_t>(bh, (1ull << 30) / ss));
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
