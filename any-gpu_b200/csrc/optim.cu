// AdamW step for many parameter tensors in one launch.
//
// Replaces the reference's SHADER_ADAMW (src/optim.rs:22-51), dispatched once
// per parameter tensor by AdamW::step (src/optim.rs:82-138).  Same update,
// element by element:
//   m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2
//   p = p (1 - lr wd) - lr (m / (1 - b1^t)) / (sqrt(v / (1 - b2^t)) + eps)
// Here a device table of (param, grad, m, v, n) entries is walked by one grid
// (blockIdx.y = tensor): the update is HBM-bound (28 bytes per element), and
// one launch replaces one per tensor.
#include <algorithm>
#include <cmath>

#include "agpu_internal.cuh"

namespace agpu {

namespace {

__global__ void __launch_bounds__(256) adamw_kernel(const agpu_adamw_tensor* __restrict__ table,
                                                    float lr, float b1, float b2, float eps,
                                                    float wd, float bc1, float bc2) {
  const agpu_adamw_tensor t = table[blockIdx.y];
  const float decay = 1.0f - lr * wd;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < t.n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float g = t.grad[i];
    const float m = b1 * t.m[i] + (1.0f - b1) * g;
    const float v = b2 * t.v[i] + (1.0f - b2) * g * g;
    t.m[i] = m;
    t.v[i] = v;
    const float m_hat = m / bc1;
    const float v_hat = v / bc2;
    t.param[i] = t.param[i] * decay - lr * m_hat / (sqrtf(v_hat) + eps);
  }
}

// beta^t as the reference computes it: f32::powi (src/optim.rs:85-86), i.e.
// binary exponentiation in f32 (square-and-multiply).  1 - beta^t amplifies
// its rounding several hundred times at beta = 0.999, so the same algorithm
// is used here rather than a more exact power.
float powi_f32(float a, uint32_t b) {
  float r = 1.0f;
  for (;;) {
    if (b & 1u) r *= a;
    b >>= 1;
    if (b == 0) break;
    a *= a;
  }
  return r;
}

}  // namespace

agpu_status launch_adamw(agpu_device* dev, const agpu_adamw_tensor* tensors, uint32_t count,
                         float lr, float beta1, float beta2, float eps, float weight_decay,
                         uint32_t step, cudaStream_t s) {
  if (count == 0) return AGPU_OK;
  if (count > 65535) return fail(AGPU_ERR_UNSUPPORTED, "adamw: more than 65535 tensors");
  if (step == 0) return fail(AGPU_ERR_INVALID, "adamw: step counts from 1");
  uint64_t max_n = 0;
  for (uint32_t i = 0; i < count; ++i) {
    const agpu_adamw_tensor& t = tensors[i];
    if (t.n && (!t.param || !t.grad || !t.m || !t.v))
      return fail(AGPU_ERR_INVALID, "adamw: tensor %u has a NULL pointer", i);
    max_n = std::max(max_n, t.n);
  }
  if (max_n == 0) return AGPU_OK;
  // bias corrections 1 - beta^t (src/optim.rs:85-86), computed once per step
  const float bc1 = 1.0f - powi_f32(beta1, step);
  const float bc2 = 1.0f - powi_f32(beta2, step);
  void* buf = nullptr;
  AGPU_TRY(pool_alloc(dev, count * sizeof(agpu_adamw_tensor), &buf, s));
  cudaError_t e = cudaMemcpyAsync(buf, tensors, count * sizeof(agpu_adamw_tensor),
                                  cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) {
    pool_free(dev, buf, s);
    return cuda_status(e, "adamw: table upload");
  }
  const uint64_t want = (max_n + 255) / 256;
  const unsigned gx = (unsigned)std::max<uint64_t>(
      1, std::min<uint64_t>(want, (uint64_t)dev->sm_count * 8 / std::max<uint32_t>(1, count) + 1));
  adamw_kernel<<<dim3(gx, count), 256, 0, s>>>(static_cast<const agpu_adamw_tensor*>(buf), lr,
                                                beta1, beta2, eps, weight_decay, bc1, bc2);
  agpu_status st = after_launch(dev, "adamw_kernel");
  pool_free(dev, buf, s);
  return st;
}

}  // namespace agpu
