// The remaining ops of the reference's autograd tape on sm_100a: the loss, the
// bias reductions of the broadcast adds, concat / slice (UNet skip
// connections) and nearest-neighbour upsampling with its backward.
//
// Replaces these WGSL shaders of the reference:
//   SHADER_MSE_SUM             src/ops/attention.rs:72-87   (one invocation, serial sum)
//   SHADER_BROADCAST_ADD       src/ops/tensor_ops.rs:87-100
//   SHADER_SUM_INNER           src/ops/tensor_ops.rs:113-129 (one thread per row)
//   SHADER_SUM_ROWS            src/ops/tensor_ops.rs:160-176 (one thread per column)
//   SHADER_CONCAT              src/ops/tensor_ops.rs:20-41
//   SHADER_SLICE               src/ops/tensor_ops.rs:59-72
//   SHADER_UPSAMPLE_NEAREST    src/ops/upsample.rs:21-45
//   SHADER_UPSAMPLE_NEAREST_BACKWARD src/ops/upsample.rs:49-78
//
// The copies are grid-stride loops over float4 when every offset allows it.
// The reductions are split over many CTAs in a fixed partition that depends
// only on the shape, and each partial list is summed in a fixed order, so
// every result is deterministic; they are tree sums, not the reference's
// serial fp32 loops (equal up to fp32 rounding).  The upsample backward sums
// its scale_h x scale_w window in the reference's order (dy, then dx), so it
// is bit-exact.
#include <algorithm>

#include "agpu_internal.cuh"

namespace agpu {

namespace {

constexpr int kThreads = 256;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline unsigned grid_for(const agpu_device* dev, uint64_t work) {
  const uint64_t want = ceil_div(work, (uint64_t)kThreads);
  const uint64_t cap = (uint64_t)dev->sm_count * 8;
  return (unsigned)std::max<uint64_t>(1, std::min(want, cap));
}

// Sum of v over the CTA, the same value in every thread (fixed order).
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

// ------------------------------------------------------------------ mse --
// Stage 1: CTA b sums (pred - target)^2 over its contiguous range.
__global__ void __launch_bounds__(kThreads) mse_partial_kernel(const float* __restrict__ p,
                                                               const float* __restrict__ t,
                                                               float* __restrict__ partial,
                                                               uint64_t n, uint64_t per) {
  __shared__ float red[kThreads / 32];
  const uint64_t b0 = blockIdx.x * per, b1 = std::min<uint64_t>(b0 + per, n);
  float s = 0.f;
  for (uint64_t i = b0 + threadIdx.x; i < b1; i += kThreads) {
    const float d = p[i] - t[i];
    s += d * d;
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

// Stage 2: one CTA sums the partials in order and divides by n
// (src/ops/attention.rs:85: sum / f32(n)).
__global__ void __launch_bounds__(kThreads) mse_final_kernel(const float* __restrict__ partial,
                                                             int parts, float* __restrict__ out,
                                                             uint64_t n) {
  __shared__ float red[kThreads / 32];
  float s = 0.f;
  for (int i = threadIdx.x; i < parts; i += kThreads) s += partial[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) out[0] = s / (float)n;
}

// ------------------------------------------------------------- sum_rows --
// out[c] = sum_r src[r, c].  Stage 1: CTA (x, y) sums columns [32x, 32x+32)
// over row chunk y (threads (32, 8): coalesced 128-byte row segments), the 8
// row-phases merged in order; stage 2 sums the chunks in order.
__global__ void sum_rows_partial_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                        uint64_t rows, uint64_t cols, uint64_t rows_per) {
  __shared__ float red[8][33];
  const uint64_t c = (uint64_t)blockIdx.x * 32 + threadIdx.x;
  const uint64_t r0 = blockIdx.y * rows_per, r1 = std::min<uint64_t>(r0 + rows_per, rows);
  float s = 0.f;
  if (c < cols)
    for (uint64_t r = r0 + threadIdx.y; r < r1; r += 8) s += src[r * cols + c];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i][threadIdx.x];
    dst[(uint64_t)blockIdx.y * cols + c] = t;
  }
}

__global__ void sum_chunks_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                  uint64_t cols, uint64_t chunks) {
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < cols;
       c += (uint64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (uint64_t k = 0; k < chunks; ++k) s += partial[k * cols + c];
    out[c] = s;
  }
}

// ------------------------------------------------------------ sum_inner --
// out[o] = sum_i src[o, i].  Short rows: one warp per row.  Long rows: CTA
// (o, s) sums chunk s of row o, then the chunks are summed in order.
__global__ void sum_inner_warp_kernel(const float* __restrict__ src, float* __restrict__ out,
                                      uint64_t outer, uint64_t inner) {
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32;
  const uint64_t nwarps = (uint64_t)gridDim.x * blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (uint64_t o = warp; o < outer; o += nwarps) {
    const float* row = src + o * inner;
    float s = 0.f;
    for (uint64_t i = lane; i < inner; i += 32) s += row[i];
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
    if (lane == 0) out[o] = s;
  }
}

constexpr uint64_t kInnerChunk = 8192;

__global__ void __launch_bounds__(kThreads) sum_inner_chunk_kernel(const float* __restrict__ src,
                                                                   float* __restrict__ partial,
                                                                   uint64_t inner,
                                                                   uint64_t chunks) {
  __shared__ float red[kThreads / 32];
  const uint64_t o = blockIdx.x, k = blockIdx.y;
  const uint64_t i0 = k * kInnerChunk, i1 = std::min<uint64_t>(i0 + kInnerChunk, inner);
  const float* row = src + o * inner;
  float s = 0.f;
  for (uint64_t i = i0 + threadIdx.x; i < i1; i += kThreads) s += row[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) partial[o * chunks + k] = s;
}

__global__ void sum_row_chunks_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                      uint64_t outer, uint64_t chunks) {
  for (uint64_t o = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; o < outer;
       o += (uint64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (uint64_t k = 0; k < chunks; ++k) s += partial[o * chunks + k];
    out[o] = s;
  }
}

// -------------------------------------------------------- add_broadcast --
// out[o, i] = a[o, i] + b[o]
__global__ void add_broadcast_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                     float* __restrict__ out, uint64_t n, uint64_t inner) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = a[i] + b[i / inner];
}

__global__ void add_broadcast_vec_kernel(const float4* __restrict__ a, const float* __restrict__ b,
                                         float4* __restrict__ out, uint64_t n4, uint64_t inner4) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float4 x = a[i];
    const float y = b[i / inner4];
    out[i] = make_float4(x.x + y, x.y + y, x.z + y, x.w + y);
  }
}

// ------------------------------------------------------ concat / slice --
// Both are row copies between [outer, w_src] and [outer, w_dst] with column
// offsets; T = float4 when every width and offset is a multiple of 4.
template <typename T>
__global__ void concat_kernel(const T* __restrict__ a, const T* __restrict__ b,
                              T* __restrict__ out, uint64_t outer, uint64_t ai, uint64_t bi) {
  const uint64_t w = ai + bi, n = outer * w;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t o = i / w, j = i % w;
    out[i] = j < ai ? a[o * ai + j] : b[o * bi + (j - ai)];
  }
}

template <typename T>
__global__ void slice_kernel(const T* __restrict__ src, T* __restrict__ dst, uint64_t outer,
                             uint64_t size, uint64_t offset, uint64_t combined) {
  const uint64_t n = outer * size;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    dst[i] = src[(i / size) * combined + offset + i % size];
}

// ------------------------------------------------------------- upsample --
// out[n, c, oh, ow] = in[n, c, oh * in_h / out_h, ow * in_w / out_w]
// (src/ops/upsample.rs:37-38), one thread per output element.
__global__ void upsample_nearest_kernel(const float* __restrict__ in, float* __restrict__ out,
                                        uint64_t planes, uint64_t in_h, uint64_t in_w,
                                        uint64_t out_h, uint64_t out_w) {
  const uint64_t n = planes * out_h * out_w;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t ow = i % out_w, oh = (i / out_w) % out_h, pl = i / (out_w * out_h);
    const uint64_t ih = oh * in_h / out_h, iw = ow * in_w / out_w;
    out[i] = in[(pl * in_h + ih) * in_w + iw];
  }
}

// grad_in[n, c, ih, iw] = sum over dy < sh, then dx < sw, of
// grad_out[n, c, ih*sh + dy, iw*sw + dx] (src/ops/upsample.rs:66-75).
__global__ void upsample_nearest_bwd_kernel(const float* __restrict__ go, float* __restrict__ gi,
                                            uint64_t planes, uint64_t in_h, uint64_t in_w,
                                            uint32_t sh, uint32_t sw) {
  const uint64_t n = planes * in_h * in_w;
  const uint64_t out_h = in_h * sh, out_w = in_w * sw;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t iw = i % in_w, ih = (i / in_w) % in_h, pl = i / (in_w * in_h);
    const float* base = go + pl * out_h * out_w;
    float s = 0.f;
    for (uint32_t dy = 0; dy < sh; ++dy)
      for (uint32_t dx = 0; dx < sw; ++dx) s += base[(ih * sh + dy) * out_w + iw * sw + dx];
    gi[i] = s;
  }
}

}  // namespace

agpu_status launch_mse_loss(agpu_device* dev, const float* pred, const float* target, float* out,
                            uint64_t n, cudaStream_t s) {
  if (n == 0) {  // 0 / 0 as in the reference's f32 division: NaN
    mse_final_kernel<<<1, kThreads, 0, s>>>(nullptr, 0, out, 0);
    return after_launch(dev, "mse_final_kernel");
  }
  // fixed partition: at most 1024 ranges of >= 4096 elements (shape-only)
  const uint64_t parts = std::min<uint64_t>(1024, ceil_div(n, 4096));
  const uint64_t per = ceil_div(n, parts);
  const uint64_t used = ceil_div(n, per);
  void* buf = nullptr;
  AGPU_TRY(pool_alloc(dev, used * sizeof(float), &buf, s));
  float* partial = static_cast<float*>(buf);
  mse_partial_kernel<<<(unsigned)used, kThreads, 0, s>>>(pred, target, partial, n, per);
  mse_final_kernel<<<1, kThreads, 0, s>>>(partial, (int)used, out, n);
  agpu_status st = after_launch(dev, "mse_loss kernels", 2);
  pool_free(dev, buf, s);
  return st;
}

agpu_status launch_sum_rows(agpu_device* dev, const float* src, float* out, uint64_t rows,
                            uint64_t cols, cudaStream_t s) {
  if (cols == 0) return AGPU_OK;
  if (rows == 0) {
    AGPU_CUDA(cudaMemsetAsync(out, 0, cols * sizeof(float), s));
    return AGPU_OK;
  }
  const uint64_t ctiles = ceil_div(cols, 32);
  if (ctiles > 0x7fffffffull) return fail(AGPU_ERR_UNSUPPORTED, "sum_rows: too many columns");
  // row chunks of >= 256 rows, at most 1024 of them (shape-only partition)
  const uint64_t chunks = std::min<uint64_t>(1024, ceil_div(rows, 256));
  const uint64_t rows_per = ceil_div(rows, chunks);
  const uint64_t used = ceil_div(rows, rows_per);
  if (used == 1) {
    sum_rows_partial_kernel<<<dim3((unsigned)ctiles, 1), dim3(32, 8), 0, s>>>(src, out, rows,
                                                                              cols, rows_per);
    return after_launch(dev, "sum_rows_partial_kernel");
  }
  void* buf = nullptr;
  AGPU_TRY(pool_alloc(dev, used * cols * sizeof(float), &buf, s));
  float* partial = static_cast<float*>(buf);
  sum_rows_partial_kernel<<<dim3((unsigned)ctiles, (unsigned)used), dim3(32, 8), 0, s>>>(
      src, partial, rows, cols, rows_per);
  sum_chunks_kernel<<<grid_for(dev, cols), kThreads, 0, s>>>(partial, out, cols, used);
  agpu_status st = after_launch(dev, "sum_rows kernels", 2);
  pool_free(dev, buf, s);
  return st;
}

agpu_status launch_sum_inner(agpu_device* dev, const float* src, float* out, uint64_t outer,
                             uint64_t inner, cudaStream_t s) {
  if (outer == 0) return AGPU_OK;
  if (inner == 0) {
    AGPU_CUDA(cudaMemsetAsync(out, 0, outer * sizeof(float), s));
    return AGPU_OK;
  }
  if (inner <= 2048) {
    sum_inner_warp_kernel<<<grid_for(dev, outer * 32), kThreads, 0, s>>>(src, out, outer, inner);
    return after_launch(dev, "sum_inner_warp_kernel");
  }
  const uint64_t chunks = ceil_div(inner, kInnerChunk);
  if (outer > 0x7fffffffull || chunks > 65535)
    return fail(AGPU_ERR_UNSUPPORTED, "sum_inner: %llu rows of %llu too large",
                (unsigned long long)outer, (unsigned long long)inner);
  void* buf = nullptr;
  AGPU_TRY(pool_alloc(dev, outer * chunks * sizeof(float), &buf, s));
  float* partial = static_cast<float*>(buf);
  sum_inner_chunk_kernel<<<dim3((unsigned)outer, (unsigned)chunks), kThreads, 0, s>>>(
      src, partial, inner, chunks);
  sum_row_chunks_kernel<<<grid_for(dev, outer), kThreads, 0, s>>>(partial, out, outer, chunks);
  agpu_status st = after_launch(dev, "sum_inner kernels", 2);
  pool_free(dev, buf, s);
  return st;
}

agpu_status launch_add_broadcast(agpu_device* dev, const float* a, const float* b, float* out,
                                 uint64_t outer, uint64_t inner, cudaStream_t s) {
  const uint64_t n = outer * inner;
  if (n == 0) return AGPU_OK;
  if (inner % 4 == 0 && aligned16(a) && aligned16(out))
    add_broadcast_vec_kernel<<<grid_for(dev, n / 4), kThreads, 0, s>>>(
        reinterpret_cast<const float4*>(a), b, reinterpret_cast<float4*>(out), n / 4, inner / 4);
  else
    add_broadcast_kernel<<<grid_for(dev, n), kThreads, 0, s>>>(a, b, out, n, inner);
  return after_launch(dev, "add_broadcast_kernel");
}

agpu_status launch_concat(agpu_device* dev, const float* a, const float* b, float* out,
                          uint64_t outer, uint64_t ai, uint64_t bi, cudaStream_t s) {
  const uint64_t n = outer * (ai + bi);
  if (n == 0) return AGPU_OK;
  if (ai % 4 == 0 && bi % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out))
    concat_kernel<float4><<<grid_for(dev, n / 4), kThreads, 0, s>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
        reinterpret_cast<float4*>(out), outer, ai / 4, bi / 4);
  else
    concat_kernel<float><<<grid_for(dev, n), kThreads, 0, s>>>(a, b, out, outer, ai, bi);
  return after_launch(dev, "concat_kernel");
}

agpu_status launch_slice_per_block(agpu_device* dev, const float* src, float* dst, uint64_t outer,
                                   uint64_t size, uint64_t offset, uint64_t combined,
                                   cudaStream_t s) {
  const uint64_t n = outer * size;
  if (n == 0) return AGPU_OK;
  if (size % 4 == 0 && offset % 4 == 0 && combined % 4 == 0 && aligned16(src) && aligned16(dst))
    slice_kernel<float4><<<grid_for(dev, n / 4), kThreads, 0, s>>>(
        reinterpret_cast<const float4*>(src), reinterpret_cast<float4*>(dst), outer, size / 4,
        offset / 4, combined / 4);
  else
    slice_kernel<float><<<grid_for(dev, n), kThreads, 0, s>>>(src, dst, outer, size, offset,
                                                              combined);
  return after_launch(dev, "slice_kernel");
}

agpu_status launch_upsample_nearest2d(agpu_device* dev, const float* in, float* out,
                                      uint64_t planes, uint32_t in_h, uint32_t in_w, uint32_t sh,
                                      uint32_t sw, cudaStream_t s) {
  const uint64_t out_h = (uint64_t)in_h * sh, out_w = (uint64_t)in_w * sw;
  const uint64_t n = planes * out_h * out_w;
  if (n == 0) return AGPU_OK;
  upsample_nearest_kernel<<<grid_for(dev, n), kThreads, 0, s>>>(in, out, planes, in_h, in_w,
                                                                out_h, out_w);
  return after_launch(dev, "upsample_nearest_kernel");
}

agpu_status launch_upsample_nearest2d_backward(agpu_device* dev, const float* go, float* gi,
                                               uint64_t planes, uint32_t in_h, uint32_t in_w,
                                               uint32_t sh, uint32_t sw, cudaStream_t s) {
  const uint64_t n = planes * in_h * in_w;
  if (n == 0) return AGPU_OK;
  upsample_nearest_bwd_kernel<<<grid_for(dev, n), kThreads, 0, s>>>(go, gi, planes, in_h, in_w,
                                                                    sh, sw);
  return after_launch(dev, "upsample_nearest_bwd_kernel");
}

}  // namespace agpu
