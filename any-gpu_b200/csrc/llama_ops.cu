// Ops of the LLaMA-style decoder layer that the reference crate does not
// have: RMSNorm, rotary position embedding (RoPE), and the fused SwiGLU
// product swish(gate) * up.  The reference composes the last one from its own
// ops (`swish` src/ops/elementwise.rs:211 then `mul` :198); the other two have
// no counterpart, so their definition is the standard formula:
//   RMSNorm  y = x / sqrt(mean(x^2) + eps) * w                    (per row)
//   RoPE     rotate-half: for i < d/2, angle = pos * base^(-2i/d),
//            y_i = x_i cos - x_{i+d/2} sin,  y_{i+d/2} = x_{i+d/2} cos + x_i sin
// All three are HBM-bound: one read and one write per element.
#include <algorithm>

#include "agpu_internal.cuh"

namespace agpu {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxVec = 8;  // float4 per thread held in registers (rows <= 8192)

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) s += red[i];
  return s;
}

// One CTA per row, the row held in registers (cols % 4 == 0, cols <= 8192).
__global__ void __launch_bounds__(kThreads) rmsnorm_vec_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               float* __restrict__ y, int cols,
                                                               float eps) {
  __shared__ float red[kThreads / 32];
  const long long row = blockIdx.x;
  const float4* src = reinterpret_cast<const float4*>(x + row * cols);
  const float4* wv = reinterpret_cast<const float4*>(w);
  float4* dst = reinterpret_cast<float4*>(y + row * cols);
  const int nvec = cols / 4;
  float4 v[kMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      v[j] = __ldcs(src + i);
      ss += (v[j].x * v[j].x + v[j].y * v[j].y) + (v[j].z * v[j].z + v[j].w * v[j].w);
    }
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      const float4 g = __ldg(wv + i);
      __stcs(dst + i, make_float4(v[j].x * inv * g.x, v[j].y * inv * g.y, v[j].z * inv * g.z,
                                  v[j].w * inv * g.w));
    }
  }
}

// Any row length / alignment: two passes over the (L1/L2-resident) row.
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const float* __restrict__ x,
                                                           const float* __restrict__ w,
                                                           float* __restrict__ y, int cols,
                                                           float eps) {
  __shared__ float red[kThreads / 32];
  const long long row = blockIdx.x;
  const float* xr = x + row * cols;
  float ss = 0.f;
  for (int i = threadIdx.x; i < cols; i += kThreads) ss += xr[i] * xr[i];
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
  for (int i = threadIdx.x; i < cols; i += kThreads) y[row * cols + i] = xr[i] * inv * w[i];
}

// One CTA per (batch, position): the first dim/2 threads compute that
// position's cos / sin in double precision (the angle reaches pos radians, so
// an fp32 angle would lose ~1e-4), then all threads rotate every head.
// x and y rows are `row_stride` elements apart, heads `dim` apart inside a row
// (so the Q or K part of a packed QKV projection can be rotated in place).
__global__ void __launch_bounds__(kThreads) rope_kernel(const float* __restrict__ x,
                                                        float* __restrict__ y, int seq, int heads,
                                                        int dim, long long row_stride,
                                                        double log2_base) {
  extern __shared__ float cs[];  // [dim/2] cos, then [dim/2] sin
  const long long rowi = blockIdx.x;  // b * seq + s
  const int pos = (int)(rowi % seq);
  const int half = dim / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const double inv_freq = exp2(-2.0 * (double)i / (double)dim * log2_base);
    double sn, c;
    sincos((double)pos * inv_freq, &sn, &c);
    cs[i] = (float)c;
    cs[half + i] = (float)sn;
  }
  __syncthreads();
  const float* xr = x + rowi * row_stride;
  float* yr = y + rowi * row_stride;
  const int pairs = heads * half;
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const int h = p / half, i = p % half;
    const float x0 = xr[h * dim + i], x1 = xr[h * dim + i + half];
    const float c = cs[i], sn = cs[half + i];
    yr[h * dim + i] = x0 * c - x1 * sn;
    yr[h * dim + i + half] = x1 * c + x0 * sn;
  }
}

// out[r, c] = swish(gate[r, c]) * up[r, c], each with its own row stride.
__global__ void swish_mul_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                 float* __restrict__ out, long long rows, int cols, long long gs,
                                 long long us, long long os) {
  const long long n = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols;
    const int c = (int)(i % cols);
    const float g = gate[r * gs + c];
    out[r * os + c] = g / (1.0f + expf(-g)) * up[r * us + c];
  }
}

__global__ void swish_mul_vec_kernel(const float4* __restrict__ gate, const float4* __restrict__ up,
                                     float4* __restrict__ out, long long rows, int cols4,
                                     long long gs4, long long us4, long long os4) {
  const long long n = rows * cols4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols4;
    const int c = (int)(i % cols4);
    const float4 g = __ldcs(gate + r * gs4 + c), u = __ldcs(up + r * us4 + c);
    __stcs(out + r * os4 + c,
           make_float4(g.x / (1.0f + expf(-g.x)) * u.x, g.y / (1.0f + expf(-g.y)) * u.y,
                       g.z / (1.0f + expf(-g.z)) * u.z, g.w / (1.0f + expf(-g.w)) * u.w));
  }
}

unsigned grid_for(const agpu_device* dev, long long work) {
  const long long want = (work + kThreads - 1) / kThreads;
  return (unsigned)std::max<long long>(1, std::min<long long>(want, (long long)dev->sm_count * 8));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

agpu_status launch_rmsnorm(agpu_device* dev, const float* x, const float* w, float* y,
                           uint64_t rows, uint32_t cols, float eps, cudaStream_t s) {
  if (rows == 0 || cols == 0) return AGPU_OK;
  if (rows > 0x7fffffffull) return fail(AGPU_ERR_UNSUPPORTED, "rmsnorm: too many rows");
  if (cols % 4 == 0 && cols <= kThreads * kMaxVec * 4 && aligned16(x) && aligned16(w) &&
      aligned16(y))
    rmsnorm_vec_kernel<<<(unsigned)rows, kThreads, 0, s>>>(x, w, y, cols, eps);
  else
    rmsnorm_kernel<<<(unsigned)rows, kThreads, 0, s>>>(x, w, y, cols, eps);
  return after_launch(dev, "rmsnorm_kernel");
}

agpu_status launch_rope(agpu_device* dev, const float* x, float* y, uint32_t batch, uint32_t seq,
                        uint32_t heads, uint32_t dim, uint64_t row_stride, float base,
                        cudaStream_t s) {
  const uint64_t rows = (uint64_t)batch * seq;
  if (rows == 0 || heads == 0 || dim == 0) return AGPU_OK;
  if (dim % 2) return fail(AGPU_ERR_SHAPE, "rope: head dim %u is odd", dim);
  if (rows > 0x7fffffffull) return fail(AGPU_ERR_UNSUPPORTED, "rope: too many rows");
  if (!(base > 0.f)) return fail(AGPU_ERR_INVALID, "rope: base must be positive");
  rope_kernel<<<(unsigned)rows, kThreads, dim * sizeof(float), s>>>(
      x, y, (int)seq, (int)heads, (int)dim, (long long)row_stride, log2((double)base));
  return after_launch(dev, "rope_kernel");
}

agpu_status launch_swish_mul(agpu_device* dev, const float* gate, const float* up, float* out,
                             uint64_t rows, uint32_t cols, uint64_t gs, uint64_t us, uint64_t os,
                             cudaStream_t s) {
  const long long n = (long long)rows * cols;
  if (n == 0) return AGPU_OK;
  if (cols % 4 == 0 && gs % 4 == 0 && us % 4 == 0 && os % 4 == 0 && aligned16(gate) &&
      aligned16(up) && aligned16(out))
    swish_mul_vec_kernel<<<grid_for(dev, n / 4), kThreads, 0, s>>>(
        reinterpret_cast<const float4*>(gate), reinterpret_cast<const float4*>(up),
        reinterpret_cast<float4*>(out), (long long)rows, (int)(cols / 4), (long long)gs / 4,
        (long long)us / 4, (long long)os / 4);
  else
    swish_mul_kernel<<<grid_for(dev, n), kThreads, 0, s>>>(gate, up, out, (long long)rows,
                                                           (int)cols, (long long)gs,
                                                           (long long)us, (long long)os);
  return after_launch(dev, "swish_mul_kernel");
}

}  // namespace agpu
