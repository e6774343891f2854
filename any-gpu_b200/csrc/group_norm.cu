// GroupNorm (optionally fused with swish) on sm_100a.
//
// Replaces the reference's two-pass group norm (src/ops/norm.rs:22-87,
// 210-278): SHADER_GN_STATS computes mean and 1/sqrt(E[x^2]-mean^2+eps) with
// one thread per (n, g) group, SHADER_GN_NORM applies (x-mean)*rstd*gamma+beta
// per element.  Same definition here, B200 layout:
//
//  * Cluster path (group fits on-chip): a thread-block cluster of CL CTAs per
//    (n, g) group; every thread keeps its float4 slice of the group in
//    registers, the CTAs exchange partial sums through distributed shared
//    memory, so x is read from HBM once and y written once.  The variance is
//    computed from centered values (sum((x-mean)^2)/count), which is the
//    reference's quantity without the E[x^2]-mean^2 cancellation.
//  * Chunked path (any size): kernel 1 writes per-chunk (mean, M2) partials
//    into scratch, kernel 2 merges a group's partials with Chan's formula in
//    a fixed order and normalises its chunk.
//  * `swish` fuses the UNet block's activation, y = z / (1 + exp(-z))
//    (src/ops/elementwise.rs:77-89), into the store.
#include <cooperative_groups.h>

#include <algorithm>

#include "agpu_internal.cuh"

namespace cg = cooperative_groups;

namespace agpu {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxVec = 16;  // float4 per thread held in registers

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

// grid.x = CL * groups, cluster (CL,1,1); slice = elements per CTA (multiple of 4).
template <bool SWISH>
__global__ void __launch_bounds__(kThreads) gn_cluster_kernel(
    const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ y, int channels, int spatial, int cpg, int groups, float eps,
    int slice) {
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float red[kThreads / 32];
  __shared__ float part[2];
  const int CL = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const long long grp = blockIdx.x / CL;  // n * groups + g
  const int g = (int)(grp % groups);
  const long long gsize = (long long)cpg * spatial;
  const long long off = grp * gsize + (long long)rank * slice;
  const float4* src = reinterpret_cast<const float4*>(x + off);
  const int nvec = slice / 4;

  float4 v[kMaxVec];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      v[j] = __ldcs(src + i);
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) part[0] = s;
  cluster.sync();
  float total = 0.f;
  for (int r = 0; r < CL; ++r) total += *cluster.map_shared_rank(&part[0], r);
  const float mean = total / (float)gsize;

  float q = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  q = block_sum(q, red);
  if (threadIdx.x == 0) part[1] = q;
  cluster.sync();
  float m2 = 0.f;
  for (int r = 0; r < CL; ++r) m2 += *cluster.map_shared_rank(&part[1], r);
  cluster.sync();  // no CTA leaves while a peer still reads its partials
  const float rstd = 1.0f / sqrtf(m2 / (float)gsize + eps);

  float4* dst = reinterpret_cast<float4*>(y + off);
  const long long e0 = (long long)rank * slice;  // element offset inside the group
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      const int ch = g * cpg + (int)((e0 + 4LL * i) / spatial);  // spatial % 4 == 0
      const float ga = gamma[ch] * rstd, be = beta[ch];
      float4 o;
      o.x = act((v[j].x - mean) * ga + be, SWISH);
      o.y = act((v[j].y - mean) * ga + be, SWISH);
      o.z = act((v[j].z - mean) * ga + be, SWISH);
      o.w = act((v[j].w - mean) * ga + be, SWISH);
      __stcs(dst + i, o);
    }
  }
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

template <bool SWISH>
agpu_status launch_cluster(agpu_device* dev, const float* x, const float* gamma,
                           const float* beta, float* y, long long groups_total, int channels,
                           int spatial, int cpg, int groups, float eps, int cl, int slice,
                           cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(groups_total * cl), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AGPU_CUDA(cudaLaunchKernelEx(&cfg, gn_cluster_kernel<SWISH>, x, gamma, beta, y, channels,
                               spatial, cpg, groups, eps, slice));
  return after_launch(dev, "gn_cluster_kernel");
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
  // Cluster path: slice per CTA must be a multiple of 4 and fit in registers.
  if (aligned && spatial % 4 == 0 && gsize <= (long long)8 * kThreads * kMaxVec * 4 &&
      groups_total * 8 < (1LL << 31)) {
    for (int cl = 1; cl <= 8; cl *= 2) {
      if (gsize % (4LL * cl) != 0) continue;
      const long long slice = gsize / cl;
      if (slice > (long long)kThreads * kMaxVec * 4) continue;
      // prefer >= 4 float4 per thread before splitting further
      return swish ? launch_cluster<true>(dev, x, gamma, beta, y, groups_total, channels,
                                          spatial, cpg, groups, eps, cl, (int)slice, s)
                   : launch_cluster<false>(dev, x, gamma, beta, y, groups_total, channels,
                                           spatial, cpg, groups, eps, cl, (int)slice, s);
    }
  }
  // Chunked path with a scratch array of per-chunk partials.
  const int chunk = 8192;
  const long long nchunks = (long long)group_norm_chunk_count((uint64_t)gsize);
  const uint64_t need = (uint64_t)groups_total * nchunks * sizeof(float2);
  if (groups_total > 65535 || nchunks > 0x7fffffff)
    return fail(AGPU_ERR_UNSUPPORTED, "group_norm: %lld groups x %lld chunks too large",
                groups_total, nchunks);
  void* buf = nullptr;
  AGPU_TRY(pool_alloc(dev, need, &buf, s));  // stream-ordered, freed after kernel 2
  dim3 grid((unsigned)nchunks, (unsigned)groups_total);
  gn_partial_kernel<<<grid, kThreads, 0, s>>>(x, static_cast<float2*>(buf), gsize, chunk);
  if (swish)
    gn_apply_kernel<true><<<grid, kThreads, 0, s>>>(x, static_cast<const float2*>(buf), gamma,
                                                    beta, y, gsize, chunk, (int)nchunks,
                                                    spatial, cpg, groups, eps);
  else
    gn_apply_kernel<false><<<grid, kThreads, 0, s>>>(x, static_cast<const float2*>(buf), gamma,
                                                     beta, y, gsize, chunk, (int)nchunks,
                                                     spatial, cpg, groups, eps);
  agpu_status st = after_launch(dev, "gn_partial/apply_kernel", 2);
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
  gn_partial_kernel<<<grid, kThreads, 0, s>>>(x, partials, (long long)gsize, chunk);
  if (apply_swish)
    gn_apply_kernel<true><<<grid, kThreads, 0, s>>>(x, partials, gamma, beta, y,
                                                    (long long)gsize, chunk, (int)nchunks,
                                                    (int)spatial, (int)cpg, (int)groups, eps);
  else
    gn_apply_kernel<false><<<grid, kThreads, 0, s>>>(x, partials, gamma, beta, y,
                                                     (long long)gsize, chunk, (int)nchunks,
                                                     (int)spatial, (int)cpg, (int)groups, eps);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "group_norm_noalloc: launch");
  return AGPU_OK;
}
