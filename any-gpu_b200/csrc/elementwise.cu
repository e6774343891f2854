// Elementwise family, transpose and per-column bias on sm_100a.
//
// Replaces the one-thread-per-element WGSL shaders of the reference:
//   SHADER_ADD/SUB/MUL, RELU/SIGMOID/SWISH/TANH, SCALE and the four
//   activation-backward shaders (src/ops/elementwise.rs:9-187),
//   SHADER_TRANSPOSE (src/ops/tensor_ops.rs:199-222) and
//   SHADER_ADD_PER_COL (src/ops/tensor_ops.rs:143-167).
// The formulas are the reference's (e.g. swish = x / (1 + exp(-x)),
// src/ops/elementwise.rs:87; swish' = s + x s (1 - s), :167-169).
//
// Kernels are grid-stride loops over 16-byte vectors (one float4 per thread
// per iteration, grid = a multiple of the SM count), with a scalar path for
// unaligned pointers and the ragged tail.  All index math is 64-bit.
#include <algorithm>

#include "agpu_internal.cuh"

namespace agpu {

namespace {

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

template <Unary OP>
__device__ __forceinline__ float unary_f(float x, float s) {
  if constexpr (OP == Unary::Relu) return fmaxf(x, 0.0f);
  if constexpr (OP == Unary::Sigmoid) return sigmoid_f(x);
  if constexpr (OP == Unary::Swish) return x / (1.0f + expf(-x));
  if constexpr (OP == Unary::Tanh) return tanhf(x);
  if constexpr (OP == Unary::Scale) return x * s;
  return x;
}

template <Binary OP>
__device__ __forceinline__ float binary_f(float a, float b) {
  if constexpr (OP == Binary::Add) return a + b;
  if constexpr (OP == Binary::Sub) return a - b;
  if constexpr (OP == Binary::Mul) return a * b;
  // a = grad_out, b = saved tensor
  if constexpr (OP == Binary::ReluBwd) return b > 0.0f ? a : 0.0f;
  if constexpr (OP == Binary::SigmoidBwd) return a * b * (1.0f - b);
  if constexpr (OP == Binary::SwishBwd) {
    const float s = sigmoid_f(b);
    return a * (s + b * s * (1.0f - s));
  }
  if constexpr (OP == Binary::TanhBwd) return a * (1.0f - b * b);
  return a;
}

template <Unary OP>
__global__ void unary_vec_kernel(const float4* __restrict__ a, float4* __restrict__ out,
                                 uint64_t n4, float s) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float4 v = a[i];
    v.x = unary_f<OP>(v.x, s); v.y = unary_f<OP>(v.y, s);
    v.z = unary_f<OP>(v.z, s); v.w = unary_f<OP>(v.w, s);
    out[i] = v;
  }
}

template <Unary OP>
__global__ void unary_scalar_kernel(const float* __restrict__ a, float* __restrict__ out,
                                    uint64_t begin, uint64_t n, float s) {
  for (uint64_t i = begin + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = unary_f<OP>(a[i], s);
}

template <Binary OP>
__global__ void binary_vec_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                  float4* __restrict__ out, uint64_t n4) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float4 x = a[i], y = b[i];
    out[i] = make_float4(binary_f<OP>(x.x, y.x), binary_f<OP>(x.y, y.y), binary_f<OP>(x.z, y.z),
                         binary_f<OP>(x.w, y.w));
  }
}

template <Binary OP>
__global__ void binary_scalar_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                     float* __restrict__ out, uint64_t begin, uint64_t n) {
  for (uint64_t i = begin + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = binary_f<OP>(a[i], b[i]);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline unsigned grid_for(const agpu_device* dev, uint64_t work, int threads) {
  // Enough CTAs to fill every SM several times, never more than the work.
  const uint64_t want = ceil_div(work, (uint64_t)threads);
  const uint64_t cap = (uint64_t)dev->sm_count * 8;
  return (unsigned)std::max<uint64_t>(1, std::min(want, cap));
}

template <Unary OP>
agpu_status run_unary(agpu_device* dev, const float* a, float* out, uint64_t n, float s,
                      cudaStream_t st) {
  int launches = 0;
  uint64_t done = 0;
  if (aligned16(a) && aligned16(out) && n >= 4) {
    const uint64_t n4 = n / 4;
    unary_vec_kernel<OP><<<grid_for(dev, n4, 256), 256, 0, st>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<float4*>(out), n4, s);
    ++launches;
    done = n4 * 4;
  }
  if (done < n) {
    unary_scalar_kernel<OP><<<grid_for(dev, n - done, 256), 256, 0, st>>>(a, out, done, n, s);
    ++launches;
  }
  return after_launch(dev, "unary_kernel", launches);
}

template <Binary OP>
agpu_status run_binary(agpu_device* dev, const float* a, const float* b, float* out, uint64_t n,
                       cudaStream_t st) {
  int launches = 0;
  uint64_t done = 0;
  if (aligned16(a) && aligned16(b) && aligned16(out) && n >= 4) {
    const uint64_t n4 = n / 4;
    binary_vec_kernel<OP><<<grid_for(dev, n4, 256), 256, 0, st>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
        reinterpret_cast<float4*>(out), n4);
    ++launches;
    done = n4 * 4;
  }
  if (done < n) {
    binary_scalar_kernel<OP><<<grid_for(dev, n - done, 256), 256, 0, st>>>(a, b, out, done, n);
    ++launches;
  }
  return after_launch(dev, "binary_kernel", launches);
}

// [outer, d0, d1] -> [outer, d1, d0] through a padded 32x32 shared tile.
__global__ void transpose_tile_kernel(const float* __restrict__ a, float* __restrict__ out,
                                      uint64_t d0, uint64_t d1) {
  __shared__ float tile[32][33];
  const uint64_t o = blockIdx.z;
  const uint64_t base = o * d0 * d1;
  const uint64_t c0 = (uint64_t)blockIdx.x * 32;  // along d1
  const uint64_t r0 = (uint64_t)blockIdx.y * 32;  // along d0
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const uint64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < d0 && c < d1) tile[i][threadIdx.x] = a[base + r * d1 + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const uint64_t r = c0 + i, c = r0 + threadIdx.x;  // out row along d1, col along d0
    if (r < d1 && c < d0) out[base + r * d0 + c] = tile[threadIdx.x][i];
  }
}

// General case inner > 1: each warp moves one contiguous inner run.
__global__ void transpose_rows_kernel(const float* __restrict__ a, float* __restrict__ out,
                                      uint64_t outer, uint64_t d0, uint64_t d1, uint64_t inner) {
  const uint64_t runs = outer * d0 * d1;
  const uint64_t warp_id = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32;
  const uint64_t nwarps = (uint64_t)gridDim.x * blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (uint64_t r = warp_id; r < runs; r += nwarps) {
    // output run index r = (o, i1, i0) -> source run (o, i0, i1)
    const uint64_t o = r / (d0 * d1);
    const uint64_t rem = r % (d0 * d1);
    const uint64_t i1 = rem / d0, i0 = rem % d0;
    const float* src = a + ((o * d0 + i0) * d1 + i1) * inner;
    float* dst = out + r * inner;
    for (uint64_t j = lane; j < inner; j += 32) dst[j] = src[j];
  }
}

__global__ void add_per_col_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                   float* __restrict__ out, uint64_t rows, uint64_t cols) {
  const uint64_t n = rows * cols;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = a[i] + b[i % cols];
}

__global__ void add_per_col_vec_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                       float4* __restrict__ out, uint64_t rows, uint64_t cols4) {
  const uint64_t n = rows * cols4;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float4 x = a[i], y = b[i % cols4];
    out[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
  }
}

}  // namespace

agpu_status launch_unary(agpu_device* dev, Unary op, const float* a, float* out, uint64_t n,
                         float s, cudaStream_t st) {
  if (n == 0) return AGPU_OK;
  switch (op) {
    case Unary::Relu: return run_unary<Unary::Relu>(dev, a, out, n, s, st);
    case Unary::Sigmoid: return run_unary<Unary::Sigmoid>(dev, a, out, n, s, st);
    case Unary::Swish: return run_unary<Unary::Swish>(dev, a, out, n, s, st);
    case Unary::Tanh: return run_unary<Unary::Tanh>(dev, a, out, n, s, st);
    case Unary::Scale: return run_unary<Unary::Scale>(dev, a, out, n, s, st);
  }
  return fail(AGPU_ERR_INVALID, "unknown unary op");
}

agpu_status launch_binary(agpu_device* dev, Binary op, const float* a, const float* b, float* out,
                          uint64_t n, cudaStream_t st) {
  if (n == 0) return AGPU_OK;
  switch (op) {
    case Binary::Add: return run_binary<Binary::Add>(dev, a, b, out, n, st);
    case Binary::Sub: return run_binary<Binary::Sub>(dev, a, b, out, n, st);
    case Binary::Mul: return run_binary<Binary::Mul>(dev, a, b, out, n, st);
    case Binary::ReluBwd: return run_binary<Binary::ReluBwd>(dev, a, b, out, n, st);
    case Binary::SigmoidBwd: return run_binary<Binary::SigmoidBwd>(dev, a, b, out, n, st);
    case Binary::SwishBwd: return run_binary<Binary::SwishBwd>(dev, a, b, out, n, st);
    case Binary::TanhBwd: return run_binary<Binary::TanhBwd>(dev, a, b, out, n, st);
  }
  return fail(AGPU_ERR_INVALID, "unknown binary op");
}

agpu_status launch_transpose(agpu_device* dev, const float* a, float* out, uint64_t outer,
                             uint64_t d0, uint64_t d1, uint64_t inner, cudaStream_t st) {
  const uint64_t n = outer * d0 * d1 * inner;
  if (n == 0) return AGPU_OK;
  if (inner == 1 && outer <= 65535) {
    dim3 grid((unsigned)ceil_div(d1, 32), (unsigned)ceil_div(d0, 32), (unsigned)outer);
    if (grid.y > 65535) return fail(AGPU_ERR_UNSUPPORTED, "transpose: d0 too large");
    transpose_tile_kernel<<<grid, dim3(32, 8), 0, st>>>(a, out, d0, d1);
  } else {
    const uint64_t runs = outer * d0 * d1;
    transpose_rows_kernel<<<grid_for(dev, runs * 32, 256), 256, 0, st>>>(a, out, outer, d0, d1,
                                                                         inner);
  }
  return after_launch(dev, "transpose_kernel");
}

agpu_status launch_add_per_col(agpu_device* dev, const float* a, const float* b, float* out,
                               uint64_t rows, uint64_t cols, cudaStream_t st) {
  const uint64_t n = rows * cols;
  if (n == 0) return AGPU_OK;
  if (cols % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out)) {
    add_per_col_vec_kernel<<<grid_for(dev, n / 4, 256), 256, 0, st>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
        reinterpret_cast<float4*>(out), rows, cols / 4);
  } else {
    add_per_col_kernel<<<grid_for(dev, n, 256), 256, 0, st>>>(a, b, out, rows, cols);
  }
  return after_launch(dev, "add_per_col_kernel");
}

}  // namespace agpu
