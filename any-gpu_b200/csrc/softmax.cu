// Row softmax on sm_100a.
//
// Replaces the reference's two-pass softmax (src/ops/attention.rs:9-61,
// 91-145): pass 1 is one thread per row computing max and sum(exp(x - max))
// serially, pass 2 one thread per element computing exp(x - max) / sum.
// Same math, B200 layout:
//   * rows of up to 2048 floats: one warp per row, the row is held in
//     registers (float4 loads, NV vectors per lane), max and sum are warp
//     shuffle reductions -> exactly one HBM read and one write per element;
//   * longer or unaligned rows: one 256-thread CTA per row, online
//     (max, sum) merge in one pass, normalise in a second (L2-resident) pass.
// exp(x - max) is evaluated as 2^((x - max) * log2 e) on the hardware ex2 unit.
#include <algorithm>

#include "agpu_internal.cuh"

namespace agpu {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row; each lane owns NV float4 vectors: v = lane + 32*j.
template <int NV>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const float* __restrict__ x,
                                                           float* __restrict__ y, uint64_t rows,
                                                           uint32_t cols) {
  const uint64_t row = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x % 32;
  const uint32_t nvec = cols / 4;
  const float4* src = reinterpret_cast<const float4*>(x + row * cols);
  float4 v[NV];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t idx = lane + 32 * j;
    if (idx < nvec) {
      v[j] = __ldcs(src + idx);  // streamed once: do not keep in L1
      m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
    } else {
      v[j] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    v[j].x = ex2((v[j].x - m) * kLog2e);
    v[j].y = ex2((v[j].y - m) * kLog2e);
    v[j].z = ex2((v[j].z - m) * kLog2e);
    v[j].w = ex2((v[j].w - m) * kLog2e);
    s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  }
  s = warp_sum(s);
  const float inv = 1.0f / s;
  float4* dst = reinterpret_cast<float4*>(y + row * cols);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t idx = lane + 32 * j;
    if (idx < nvec)
      __stcs(dst + idx, make_float4(v[j].x * inv, v[j].y * inv, v[j].z * inv, v[j].w * inv));
  }
}

// (max, sum) pair merge for the online softmax.
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * ex2((m - mn) * kLog2e) + s2 * ex2((m2 - mn) * kLog2e);
  m = mn;
}

// One CTA per row, any length / alignment.
__global__ void __launch_bounds__(256) softmax_block_kernel(const float* __restrict__ x,
                                                            float* __restrict__ y, uint32_t cols) {
  const uint64_t row = blockIdx.x;
  const float* src = x + row * cols;
  float* dst = y + row * cols;
  float m = -INFINITY, s = 0.f;
  for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float v = src[i];
    if (v > m) {
      s = s * ex2((m - v) * kLog2e) + 1.0f;
      m = v;
    } else {
      s += ex2((v - m) * kLog2e);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, m2, s2);
  }
  __shared__ float sm[8], ss[8];
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) { sm[w] = m; ss[w] = s; }
  __syncthreads();
  if (w == 0) {
    m = lane < 8 ? sm[lane] : -INFINITY;
    s = lane < 8 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge(m, s, m2, s2);
    }
    if (lane == 0) { sm[0] = m; ss[0] = s; }
  }
  __syncthreads();
  m = sm[0];
  const float inv = 1.0f / ss[0];
  for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x)
    dst[i] = ex2((src[i] - m) * kLog2e) * inv;
}

template <int NV>
agpu_status run_warp(agpu_device* dev, const float* x, float* y, uint64_t rows, uint32_t cols,
                     cudaStream_t s) {
  const uint64_t blocks = ceil_div(rows, 8);
  softmax_warp_kernel<NV><<<(unsigned)blocks, 256, 0, s>>>(x, y, rows, cols);
  return after_launch(dev, "softmax_warp_kernel");
}

}  // namespace

agpu_status launch_softmax(agpu_device* dev, const float* x, float* y, uint64_t rows,
                           uint32_t cols, cudaStream_t s) {
  if (rows == 0 || cols == 0) return AGPU_OK;
  const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) |
                                        reinterpret_cast<uintptr_t>(y)) & 15u) == 0;
  if (vec && ceil_div(rows, 8) <= 0x7fffffffull) {
    const uint32_t nvec = cols / 4;
    if (nvec <= 32) return run_warp<1>(dev, x, y, rows, cols, s);
    if (nvec <= 64) return run_warp<2>(dev, x, y, rows, cols, s);
    if (nvec <= 128) return run_warp<4>(dev, x, y, rows, cols, s);
    if (nvec <= 256) return run_warp<8>(dev, x, y, rows, cols, s);
    if (nvec <= 512) return run_warp<16>(dev, x, y, rows, cols, s);
  }
  if (rows > 0x7fffffffull) return fail(AGPU_ERR_UNSUPPORTED, "softmax: too many rows");
  softmax_block_kernel<<<(unsigned)rows, 256, 0, s>>>(x, y, cols);
  return after_launch(dev, "softmax_block_kernel");
}

}  // namespace agpu
