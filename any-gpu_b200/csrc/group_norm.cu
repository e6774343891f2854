// GroupNorm (optionally fused with swish) on sm_100a.
//
// Replaces the reference's two-pass group norm (src/ops/norm.rs:22-87,
// 210-278): SHADER_GN_STATS computes mean and 1/sqrt(E[x^2]-mean^2+eps) with
// one thread per (n, g) group, SHADER_GN_NORM applies (x-mean)*rstd*gamma+beta
// per element.  Same definition here, B200 layout:
//
//  * Chunked, two kernels: kernel 1 reduces each 8192-element chunk of a
//    group to (mean, M2) -- the exact chunk mean, then the centered sum of
//    squares, two plain block sums (no E[x^2]-mean^2 cancellation); kernel 2
//    loads its chunk, merges the group's chunk summaries with Chan's formula
//    in a fixed order in every thread (while its loads are in flight), and
//    normalises.  x is read twice; a tensor up to the 126 MB L2 is mostly
//    served from L2 the second time.  Measured against a single-pass kernel
//    holding each group in registers (one 1024-thread CTA per group) and a
//    persistent cluster kernel streaming slices through shared memory, both
//    latency-bound, this is the fastest (UNet block: 49.8 vs 58.7 vs 91 us).
//    Also measured and dropped: one cooperative launch rolling the chunk
//    list through the resident CTAs (stats of round r, normalise round r-1,
//    so x crosses HBM once: 59.7 us, the CTAs move in lockstep and HBM
//    idles during their reductions), and splitting the groups into 24-40 MB
//    slabs run back to back so the re-read hits L2 (61-85 us); and one pass
//    on a cluster of 4 CTAs per group holding the group in registers, the
//    exact mean and M2 exchanged through distributed shared memory (49.5 us:
//    x crosses HBM once, but the CTAs wait on each other with the data held,
//    so it is latency-bound at the same time).  Kernel 1 loads with an L2
//    evict-last policy, which keeps more of x in L2 for kernel 2 (52 -> 50
//    us).  Float4 loads when x, y are 16-byte aligned and spatial % 4 == 0,
//    a scalar pair of kernels otherwise.
//  * `swish` fuses the UNet block's activation, y = z / (1 + exp(-z))
//    (src/ops/elementwise.rs:77-89), into the store.
#include <algorithm>

#include "agpu_internal.cuh"

namespace agpu {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) s += red[i];  // same order in every thread
  return s;
}

__device__ __forceinline__ float act(float z, bool swish) {
  return swish ? z / (1.0f + expf(-z)) : z;
}

__device__ __forceinline__ float act_fast(float z, bool swish) {
  // swish with the fast exponential and divide: |error| ~ 1e-6 relative, far
  // below the op's 1e-5 tolerance; 1 + e^-z = inf gives the limit 0.
  return swish ? __fdividef(z, 1.0f + __expf(-z)) : z;
}

// Chan et al. merge of two (count, mean, M2) summaries.
__device__ __forceinline__ void chan_merge(float& n, float& mean, float& m2, float nb, float mb,
                                           float m2b) {
  const float nt = n + nb;
  if (nt == 0.f) return;
  const float d = mb - mean;
  const float f = nb / nt;
  mean += d * f;
  m2 += m2b + d * d * n * f;
  n = nt;
}

// ------------------------------------------------------- chunked fallback --
// Kernel 1: (mean, M2) of chunk blockIdx.x of group blockIdx.y -> scratch.
__global__ void __launch_bounds__(kThreads) gn_partial_kernel(const float* __restrict__ x,
                                                              float2* __restrict__ partials,
                                                              long long gsize, int chunk) {
  __shared__ float red[kThreads / 32];
  const long long grp = blockIdx.y;
  const long long c0 = (long long)blockIdx.x * chunk;
  const long long c1 = std::min<long long>(c0 + chunk, gsize);
  const float* xg = x + grp * gsize;
  float s = 0.f;
  for (long long i = c0 + threadIdx.x; i < c1; i += kThreads) s += xg[i];
  s = block_sum(s, red);
  const float cnt = (float)(c1 - c0);
  const float mean = s / cnt;
  float q = 0.f;
  for (long long i = c0 + threadIdx.x; i < c1; i += kThreads) {
    const float d = xg[i] - mean;
    q += d * d;
  }
  q = block_sum(q, red);
  if (threadIdx.x == 0) partials[grp * gridDim.x + blockIdx.x] = make_float2(mean, q);
}

// Kernel 2: merge the group's chunk partials (Chan et al. parallel variance,
// fixed order) and normalise chunk blockIdx.x.
template <bool SWISH>
__global__ void __launch_bounds__(kThreads) gn_apply_kernel(
    const float* __restrict__ x, const float2* __restrict__ partials,
    const float* __restrict__ gamma, const float* __restrict__ beta, float* __restrict__ y,
    long long gsize, int chunk, int nchunks, int spatial, int cpg, int groups, float eps) {
  __shared__ float stat[2];
  const long long grp = blockIdx.y;
  const int g = (int)(grp % groups);
  if (threadIdx.x == 0) {
    double n = 0.0, mean = 0.0, m2 = 0.0;
    for (int c = 0; c < nchunks; ++c) {
      const float2 p = partials[grp * nchunks + c];
      const double nb = (double)(std::min<long long>((long long)(c + 1) * chunk, gsize) -
                                 (long long)c * chunk);
      const double delta = (double)p.x - mean;
      const double nt = n + nb;
      mean += delta * nb / nt;
      m2 += (double)p.y + delta * delta * n * nb / nt;
      n = nt;
    }
    stat[0] = (float)mean;
    stat[1] = (float)(1.0 / sqrt(m2 / n + (double)eps));
  }
  __syncthreads();
  const float mean = stat[0], rstd = stat[1];
  const long long c0 = (long long)blockIdx.x * chunk;
  const long long c1 = std::min<long long>(c0 + chunk, gsize);
  const float* xg = x + grp * gsize;
  float* yg = y + grp * gsize;
  for (long long i = c0 + threadIdx.x; i < c1; i += kThreads) {
    const int ch = g * cpg + (int)(i / spatial);
    yg[i] = act((xg[i] - mean) * rstd * gamma[ch] + beta[ch], SWISH);
  }
}

// Vectorised chunked path (x, y 16-byte aligned, spatial % 4 == 0): kernel
// 1 reduces each 8192-element chunk from registers to (mean, M2); kernel 2
// loads its chunk first, merges the group's partials while the loads are in
// flight, then normalises.  x is read twice, but a tensor that fits in L2
// (126 MB) is mostly served from there the second time.
constexpr int kChunkVec = 8;  // float4 per thread: 8192-element chunks
constexpr int kMergeBatch = 8;  // chunk summaries fetched together by the apply kernel

// Load with an L2 evict-last policy: the chunk stays in L2 for the apply
// kernel's second read (measured: UNet block group norm 52 -> 50 us).
__device__ __forceinline__ float4 ld_keep(const float4* p, uint64_t pol) {
  float4 v;
  asm("ld.global.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

__global__ void __launch_bounds__(kThreads) gn_partial_vec_kernel(const float* __restrict__ x,
                                                                  float2* __restrict__ partials,
                                                                  long long gsize, int chunk) {
  __shared__ float red[kThreads / 32];
  const long long grp = blockIdx.y;
  const long long c0 = (long long)blockIdx.x * chunk;
  const int n = (int)(std::min<long long>(c0 + chunk, gsize) - c0);
  const int nvec = n / 4;
  const float4* src = reinterpret_cast<const float4*>(x + grp * gsize + c0);
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  float4 v[kChunkVec];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kChunkVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      v[j] = ld_keep(src + i, pol);  // the apply kernel re-reads this chunk
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
  }
  // exact chunk mean, then the centered M2: two plain block sums
  const float mean = block_sum(s, red) / (float)n;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < kChunkVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  q = block_sum(q, red);
  if (threadIdx.x == 0) partials[grp * gridDim.x + blockIdx.x] = make_float2(mean, q);
}

template <bool SWISH>
__global__ void __launch_bounds__(kThreads) gn_apply_vec_kernel(
    const float* __restrict__ x, const float2* __restrict__ partials,
    const float* __restrict__ gamma, const float* __restrict__ beta, float* __restrict__ y,
    long long gsize, int chunk, int nchunks, int spatial, int cpg, int groups, float eps) {
  const long long grp = blockIdx.y;
  const int g = (int)(grp % groups);
  const long long c0 = (long long)blockIdx.x * chunk;
  const int nvec = (int)(std::min<long long>(c0 + chunk, gsize) - c0) / 4;
  const float4* src = reinterpret_cast<const float4*>(x + grp * gsize + c0);
  float4 v[kChunkVec];
#pragma unroll
  for (int j = 0; j < kChunkVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) v[j] = __ldcs(src + i);  // last use of x
  }
  // every thread merges the group's chunk summaries (Chan et al., fixed
  // order), while its loads are in flight; the first kMergeBatch summaries
  // are fetched together (one L2 round trip, not one per merge step)
  auto chunk_n = [&](int c) {
    return (float)(std::min<long long>((long long)(c + 1) * chunk, gsize) - (long long)c * chunk);
  };
  const float2* gp = partials + grp * nchunks;
  float2 pp[kMergeBatch];
#pragma unroll
  for (int c = 0; c < kMergeBatch; ++c)
    if (c < nchunks) pp[c] = __ldg(gp + c);
  float n = 0.f, mean = 0.f, m2 = 0.f;
#pragma unroll
  for (int c = 0; c < kMergeBatch; ++c)
    if (c < nchunks) chan_merge(n, mean, m2, chunk_n(c), pp[c].x, pp[c].y);
  for (int c = kMergeBatch; c < nchunks; ++c) {
    const float2 q = __ldg(gp + c);
    chan_merge(n, mean, m2, chunk_n(c), q.x, q.y);
  }
  const float rstd = 1.0f / sqrtf(m2 / n + eps);
  float4* dst = reinterpret_cast<float4*>(y + grp * gsize + c0);
  const float inv_sp = 1.0f / (float)spatial;
#pragma unroll
  for (int j = 0; j < kChunkVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      // channel of element c0 + 4i inside the group (spatial % 4 == 0): a
      // reciprocal estimate, then exact by one correction step either way
      // (the quotient is below cpg, so the estimate is off by at most one)
      const long long e = c0 + 4LL * i;
      int cq = (int)((float)e * inv_sp);
      if ((long long)cq * spatial > e) --cq;
      else if ((long long)(cq + 1) * spatial <= e) ++cq;
      const int ch = g * cpg + cq;
      const float ga = __ldg(gamma + ch) * rstd, be = __ldg(beta + ch);
      float4 o;
      o.x = act_fast((v[j].x - mean) * ga + be, SWISH);
      o.y = act_fast((v[j].y - mean) * ga + be, SWISH);
      o.z = act_fast((v[j].z - mean) * ga + be, SWISH);
      o.w = act_fast((v[j].w - mean) * ga + be, SWISH);
      __stcs(dst + i, o);
    }
  }
}

// The two chunked kernels (vectorised when `vec`), partials in `partials`.
void launch_chunked(const float* x, float2* partials, const float* gamma, const float* beta,
                    float* y, long long gsize, int chunk, int nchunks, int spatial, int cpg,
                    int groups, float eps, bool swish, bool vec, dim3 grid, cudaStream_t s) {
  if (vec) {
    gn_partial_vec_kernel<<<grid, kThreads, 0, s>>>(x, partials, gsize, chunk);
    if (swish)
      gn_apply_vec_kernel<true><<<grid, kThreads, 0, s>>>(x, partials, gamma, beta, y, gsize,
                                                          chunk, nchunks, spatial, cpg, groups,
                                                          eps);
    else
      gn_apply_vec_kernel<false><<<grid, kThreads, 0, s>>>(x, partials, gamma, beta, y, gsize,
                                                           chunk, nchunks, spatial, cpg, groups,
                                                           eps);
    return;
  }
  gn_partial_kernel<<<grid, kThreads, 0, s>>>(x, partials, gsize, chunk);
  if (swish)
    gn_apply_kernel<true><<<grid, kThreads, 0, s>>>(x, partials, gamma, beta, y, gsize, chunk,
                                                    nchunks, spatial, cpg, groups, eps);
  else
    gn_apply_kernel<false><<<grid, kThreads, 0, s>>>(x, partials, gamma, beta, y, gsize, chunk,
                                                     nchunks, spatial, cpg, groups, eps);
}

// --------------------------------------------------------------- backward --
// GpuDevice::group_norm_backward (src/ops/norm.rs:282-438, shaders :88-205):
// with x_hat = (x - mean) * rstd per (n, g) and count = cpg * spatial,
//   s1 = sum_group(dy * gamma),  s2 = sum_group(dy * gamma * x_hat)
//   dx = rstd * (dy * gamma - (s1 + x_hat * s2) / count)
//   dgamma[c] = sum_{n,s}(dy * x_hat),  dbeta[c] = sum_{n,s}(dy)
// in four launches; 1 and 3 run one CTA per chunk (<= 4096 elements) of one
// (n, channel) row:
//   1. per chunk: (mean, M2) of x, E = sum dy, A = sum dy * (x - chunk mean),
//      merged up the CTA with Chan's rules (A moves with the mean:
//      A' = A1 + A2 + (m1 - m) E1 + (m2 - m) E2), so x and dy are read once;
//   2. per group (n, g): merge its chunks in a fixed order into mean, rstd,
//      s1 = sum gamma_c E, s2 = rstd sum gamma_c (A + (m_chunk - mean) E);
//   3. per chunk: dx (x and dy read again);
//   4. per channel: dbeta = sum E, dgamma = sum rstd (A + (m_chunk - mean) E)
//      over (n, chunk) in a fixed order.
// Every sum is in a fixed order, so the result is deterministic.
constexpr int kBwdChunk = 4096;
constexpr int kBwdPer = kBwdChunk / kThreads;  // elements per thread

struct BwdSum {
  float n, mean, m2, e, a;
};

__device__ __forceinline__ void bwd_merge(BwdSum& s, const BwdSum& b) {
  const float nt = s.n + b.n;
  if (nt == 0.f) return;
  const float d = b.mean - s.mean;
  const float f = b.n / nt;
  const float mean = s.mean + d * f;
  s.m2 += b.m2 + d * d * s.n * f;
  s.a += b.a + (s.mean - mean) * s.e + (b.mean - mean) * b.e;
  s.e += b.e;
  s.mean = mean;
  s.n = nt;
}

__device__ __forceinline__ BwdSum bwd_shfl(const BwdSum& s, int o) {
  BwdSum r;
  r.n = __shfl_xor_sync(0xffffffffu, s.n, o);
  r.mean = __shfl_xor_sync(0xffffffffu, s.mean, o);
  r.m2 = __shfl_xor_sync(0xffffffffu, s.m2, o);
  r.e = __shfl_xor_sync(0xffffffffu, s.e, o);
  r.a = __shfl_xor_sync(0xffffffffu, s.a, o);
  return r;
}

// grid (chunks per row, channels, batch)
__global__ void __launch_bounds__(kThreads) gn_bwd_partial_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, float4* __restrict__ partials,
    int channels, long long spatial) {
  __shared__ BwdSum wsum[kThreads / 32];
  const int sc = blockIdx.x, ch = blockIdx.y, n = blockIdx.z;
  const long long row = ((long long)n * channels + ch) * spatial;
  const long long s0 = (long long)sc * kBwdChunk;
  const int len = (int)std::min<long long>(kBwdChunk, spatial - s0);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float xv[kBwdPer], gv[kBwdPer];
  BwdSum t{0.f, 0.f, 0.f, 0.f, 0.f};
  float sx = 0.f;
#pragma unroll
  for (int k = 0; k < kBwdPer; ++k) {
    const int i = threadIdx.x + k * kThreads;
    xv[k] = 0.f;
    gv[k] = 0.f;
    if (i < len) {
      xv[k] = x[row + s0 + i];
      gv[k] = dy[row + s0 + i];
      sx += xv[k];
      t.e += gv[k];
      t.n += 1.f;
    }
  }
  t.mean = t.n > 0.f ? sx / t.n : 0.f;
#pragma unroll
  for (int k = 0; k < kBwdPer; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < len) {
      const float d = xv[k] - t.mean;
      t.m2 += d * d;
      t.a += gv[k] * d;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const BwdSum b = bwd_shfl(t, o);
    if (lane & o) {  // lower lane's summary first: both partners get the same bits
      BwdSum lo = b;
      bwd_merge(lo, t);
      t = lo;
    } else {
      bwd_merge(t, b);
    }
  }
  if (lane == 0) wsum[warp] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    BwdSum r = wsum[0];
    for (int w = 1; w < kThreads / 32; ++w) bwd_merge(r, wsum[w]);
    partials[((long long)n * channels + ch) * gridDim.x + sc] = make_float4(r.mean, r.m2, r.e, r.a);
  }
}

// Merge the chunk partials of group (n, g) in a fixed order (double precision).
__device__ void bwd_group_stats(const float4* __restrict__ partials, const float* __restrict__ gamma,
                                int n, int g, int cpg, int channels, int nsch, long long spatial,
                                float eps, float* mean_out, float* rstd_out, float* s1_out,
                                float* s2_out) {
  double cnt = 0.0, mean = 0.0, m2 = 0.0;
  for (int c = 0; c < cpg; ++c) {
    const int ch = g * cpg + c;
    for (int sc = 0; sc < nsch; ++sc) {
      const float4 p = partials[((long long)n * channels + ch) * nsch + sc];
      const double nb = (double)std::min<long long>(kBwdChunk, spatial - (long long)sc * kBwdChunk);
      const double d = (double)p.x - mean, nt = cnt + nb;
      mean += d * nb / nt;
      m2 += (double)p.y + d * d * cnt * nb / nt;
      cnt = nt;
    }
  }
  const double rstd = 1.0 / sqrt(m2 / cnt + (double)eps);
  double s1 = 0.0, t = 0.0;
  for (int c = 0; c < cpg; ++c) {
    const int ch = g * cpg + c;
    const double ga = (double)gamma[ch];
    for (int sc = 0; sc < nsch; ++sc) {
      const float4 p = partials[((long long)n * channels + ch) * nsch + sc];
      s1 += ga * (double)p.z;
      t += ga * ((double)p.w + ((double)p.x - mean) * (double)p.z);
    }
  }
  *mean_out = (float)mean;
  *rstd_out = (float)rstd;
  *s1_out = (float)s1;
  *s2_out = (float)(rstd * t);
}

// One thread per group (n, g): (mean, rstd, s1, s2).
__global__ void gn_bwd_stats_kernel(const float4* __restrict__ partials,
                                    const float* __restrict__ gamma, float4* __restrict__ gstat,
                                    long long groups_total, int groups, int cpg, int channels,
                                    int nsch, long long spatial, float eps) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= groups_total) return;
  float4 r;
  bwd_group_stats(partials, gamma, (int)(i / groups), (int)(i % groups), cpg, channels, nsch,
                  spatial, eps, &r.x, &r.y, &r.z, &r.w);
  gstat[i] = r;
}

__global__ void __launch_bounds__(kThreads) gn_bwd_dx_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ gamma,
    const float4* __restrict__ gstat, float* __restrict__ dx, int channels, long long spatial,
    int cpg, int groups) {
  const int sc = blockIdx.x, ch = blockIdx.y, n = blockIdx.z;
  const long long row = ((long long)n * channels + ch) * spatial;
  const long long s0 = (long long)sc * kBwdChunk;
  const int len = (int)std::min<long long>(kBwdChunk, spatial - s0);
  const float4 st = gstat[(long long)n * groups + ch / cpg];  // mean, rstd, s1, s2
  const float inv_count = 1.0f / ((float)cpg * (float)spatial);
  const float ga = gamma[ch];
#pragma unroll
  for (int k = 0; k < kBwdPer; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < len) {
      const float xh = (__ldcs(x + row + s0 + i) - st.x) * st.y;
      __stcs(dx + row + s0 + i,
             st.y * (__ldcs(dy + row + s0 + i) * ga - (st.z + xh * st.w) * inv_count));
    }
  }
}

// One thread per channel.
__global__ void __launch_bounds__(kThreads) gn_bwd_affine_kernel(
    const float4* __restrict__ partials, const float4* __restrict__ gstat,
    float* __restrict__ dgamma, float* __restrict__ dbeta, int batch, int channels, int nsch,
    int cpg, int groups) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= channels) return;
  const int g = ch / cpg;
  float dg = 0.f, db = 0.f;
  for (int n = 0; n < batch; ++n) {
    const float4 gs = gstat[(long long)n * groups + g];  // mean, rstd, s1, s2
    for (int sc = 0; sc < nsch; ++sc) {
      const float4 p = partials[((long long)n * channels + ch) * nsch + sc];
      db += p.z;
      dg += gs.y * (p.w + (p.x - gs.x) * p.z);
    }
  }
  dgamma[ch] = dg;
  dbeta[ch] = db;
}

}  // namespace

// Number of 8192-element chunks per group on the chunked path.
uint64_t group_norm_chunk_count(uint64_t gsize) { return ceil_div(gsize, 8192); }

agpu_status launch_group_norm(agpu_device* dev, const float* x, const float* gamma,
                              const float* beta, float* y, uint32_t batch, uint32_t channels,
                              uint32_t spatial, uint32_t groups, float eps, bool swish,
                              cudaStream_t s) {
  if (batch == 0 || channels == 0 || spatial == 0) return AGPU_OK;
  const uint32_t cpg = channels / groups;
  const long long gsize = (long long)cpg * spatial;
  const long long groups_total = (long long)batch * groups;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) &
                        15u) == 0;
  // Chunked path with a scratch array of per-chunk partials.
  const int chunk = 8192;
  const long long nchunks = (long long)group_norm_chunk_count((uint64_t)gsize);
  const uint64_t need = (uint64_t)groups_total * nchunks * sizeof(float2);
  if (groups_total > 65535 || nchunks > 0x7fffffff)
    return fail(AGPU_ERR_UNSUPPORTED, "group_norm: %lld groups x %lld chunks too large",
                groups_total, nchunks);
  const bool vec = aligned && spatial % 4 == 0;
  void* buf = nullptr;
  AGPU_TRY(pool_alloc(dev, need, &buf, s));  // stream-ordered, freed after kernel 2
  dim3 grid((unsigned)nchunks, (unsigned)groups_total);
  launch_chunked(x, static_cast<float2*>(buf), gamma, beta, y, gsize, chunk, (int)nchunks,
                 (int)spatial, (int)cpg, (int)groups, eps, swish, vec,
                 grid, s);
  agpu_status st = after_launch(dev, "gn_partial/apply_kernel", 2);
  pool_free(dev, buf, s);
  return st;
}

agpu_status launch_group_norm_backward(agpu_device* dev, const float* dy, const float* x,
                                       const float* gamma, float* dx, float* dgamma,
                                       float* dbeta, uint32_t batch, uint32_t channels,
                                       uint32_t spatial, uint32_t groups, float eps,
                                       cudaStream_t s) {
  if (channels == 0) return AGPU_OK;
  if (batch == 0 || spatial == 0) {  // empty sums: zero gradients for gamma and beta
    AGPU_CUDA(cudaMemsetAsync(dgamma, 0, channels * sizeof(float), s));
    AGPU_CUDA(cudaMemsetAsync(dbeta, 0, channels * sizeof(float), s));
    return AGPU_OK;
  }
  if (channels > 65535 || batch > 65535)
    return fail(AGPU_ERR_UNSUPPORTED, "group_norm_backward: channels and batch must be <= 65535");
  const uint32_t cpg = channels / groups;
  const long long nsch = (long long)ceil_div(spatial, kBwdChunk);
  const uint64_t np = (uint64_t)batch * channels * nsch;
  const uint64_t ng = (uint64_t)batch * groups;
  const uint64_t bytes = (np + ng) * sizeof(float4);
  void* buf = nullptr;
  AGPU_TRY(pool_alloc(dev, bytes, &buf, s));
  float4* partials = static_cast<float4*>(buf);
  float4* gstat = partials + np;
  const dim3 grid((unsigned)nsch, channels, batch);
  gn_bwd_partial_kernel<<<grid, kThreads, 0, s>>>(dy, x, partials, (int)channels,
                                                  (long long)spatial);
  gn_bwd_stats_kernel<<<(unsigned)ceil_div(ng, 128), 128, 0, s>>>(
      partials, gamma, gstat, (long long)ng, (int)groups, (int)cpg, (int)channels, (int)nsch,
      (long long)spatial, eps);
  gn_bwd_dx_kernel<<<grid, kThreads, 0, s>>>(dy, x, gamma, gstat, dx, (int)channels,
                                             (long long)spatial, (int)cpg, (int)groups);
  gn_bwd_affine_kernel<<<(unsigned)ceil_div(channels, kThreads), kThreads, 0, s>>>(
      partials, gstat, dgamma, dbeta, (int)batch, (int)channels, (int)nsch, (int)cpg,
      (int)groups);
  agpu_status st = after_launch(dev, "group_norm backward kernels", 4);
  pool_free(dev, buf, s);
  return st;
}

// ---------------------------------------------------------------------------
// agpu_group_norm_noalloc: group norm that never allocates device memory.
//
// Some callers may not allocate device memory themselves: a serving process
// that owns every byte of device memory through its own arena and a hard cap,
// a foreign host (Rust, Go, JNI) that hands over only device pointers and a
// stream, or a latency-critical loop that cannot pay for an allocation's
// implicit synchronisation.  For them this entry point runs the chunked
// two-kernel group norm with its per-chunk (mean, M2) partials in the
// fixed-size array below instead of the device pool.
//
// * The array is part of this library's device image: every GPU that loads
//   the library holds its 512 KiB until the process exits.
// * Limit: batch * groups * ceil(channels/groups * spatial / 8192) partials
//   <= kNoAllocPartials (65536), and batch * groups <= 65535; larger shapes
//   return AGPU_ERR_UNSUPPORTED without launching anything.
// * All calls share the array and it keeps the last call's contents.  Nothing
//   in it has to start at zero: the first kernel writes every slot the second
//   one reads.  Calls that overlap on the GPU (other streams, other host
//   threads) race on it; order them on one stream or with events.
// * The first call on a device does the set-up for that device (looks up the
//   array's device address with cudaGetSymbolAddress, which also makes the
//   CUDA runtime load this library's module there).  Make that first call
//   before any stream capture.
namespace {

constexpr uint64_t kNoAllocPartials = 65536;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float2 g_gn_noalloc_partials[kNoAllocPartials];

std::mutex g_noalloc_mu;
float2* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the partials array on the current device (set up once).
agpu_status noalloc_partials(float2** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "group_norm_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(AGPU_ERR_UNSUPPORTED, "group_norm_noalloc: device ordinal %d >= %d", dev,
                kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gn_noalloc_partials);
    if (e != cudaSuccess)
      return cuda_status(e, "group_norm_noalloc: cudaGetSymbolAddress(partials)");
    g_noalloc_ptr[dev] = static_cast<float2*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return AGPU_OK;
}

}  // namespace

}  // namespace agpu

extern "C" agpu_status agpu_group_norm_noalloc(const float* x, const float* gamma,
                                               const float* beta, float* y, uint32_t batch,
                                               uint32_t channels, uint32_t spatial,
                                               uint32_t groups, float eps, int apply_swish,
                                               void* stream) {
  using namespace agpu;
  if (groups == 0 || channels % groups != 0)
    return fail(AGPU_ERR_SHAPE, "group_norm_noalloc: channels (%u) not divisible by groups (%u)",
                channels, groups);
  const uint64_t total = (uint64_t)batch * channels * spatial;
  if (total == 0) return AGPU_OK;
  if (!x || !gamma || !beta || !y)
    return fail(AGPU_ERR_INVALID, "group_norm_noalloc: NULL pointer");
  const uint64_t gsize = (uint64_t)(channels / groups) * spatial;
  const uint64_t groups_total = (uint64_t)batch * groups;
  const uint64_t nchunks = group_norm_chunk_count(gsize);
  if (groups_total > 65535 || groups_total * nchunks > kNoAllocPartials)
    return fail(AGPU_ERR_UNSUPPORTED,
                "group_norm_noalloc: %llu groups x %llu chunks of 8192 elements need %llu "
                "partials; the fixed scratch holds %llu (and at most 65535 groups)",
                (unsigned long long)groups_total, (unsigned long long)nchunks,
                (unsigned long long)(groups_total * nchunks),
                (unsigned long long)kNoAllocPartials);
  float2* partials = nullptr;
  AGPU_TRY(noalloc_partials(&partials));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int chunk = 8192;
  dim3 grid((unsigned)nchunks, (unsigned)groups_total);
  const uint32_t cpg = channels / groups;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u) == 0 &&
                   spatial % 4 == 0;
  launch_chunked(x, partials, gamma, beta, y, (long long)gsize, chunk, (int)nchunks,
                 (int)spatial, (int)cpg, (int)groups, eps, apply_swish != 0, vec, grid, s);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "group_norm_noalloc: launch");
  return AGPU_OK;
}
