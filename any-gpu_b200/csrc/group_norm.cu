// GroupNorm (optionally fused with swish) on sm_100a.
//
// Replaces the reference's two-pass group norm (src/ops/norm.rs:22-87,
// 210-278): SHADER_GN_STATS computes mean and 1/sqrt(E[x^2]-mean^2+eps) with
// one thread per (n, g) group, SHADER_GN_NORM applies (x-mean)*rstd*gamma+beta
// per element.  Same definition here, B200 layout:
//
//  * Streaming cluster path (group fits on-chip): a persistent grid of
//    thread-block clusters, CL CTAs per cluster, walks the (n, g) groups; each
//    CTA owns one 1/CL slice of every group.  Slices are brought in by bulk
//    copies (cp.async.bulk) into a 2-4 deep shared-memory ring, so the reads
//    of the next groups are in flight while the current one is reduced and
//    written: x is read from HBM once, y written once.  Each CTA reduces its
//    slice to (mean, M2) (Chan merges up the warps), pushes the pair into
//    every peer's shared memory with st.async, which completes on the peer's
//    mbarrier -- no cluster barrier, so no fence waits on the previous
//    group's stores -- and all CTAs merge the CL pairs in the same order.  The variance is computed from centered
//    values, which is the reference's quantity without the E[x^2]-mean^2
//    cancellation.
//  * Chunked path (any size): kernel 1 writes per-chunk (mean, M2) partials
//    into scratch, kernel 2 merges a group's partials with Chan's formula in
//    a fixed order and normalises its chunk.
//  * `swish` fuses the UNet block's activation, y = z / (1 + exp(-z))
//    (src/ops/elementwise.rs:77-89), into the store.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "agpu_internal.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

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

// One CTA of T threads per (n, g) group, the whole group in registers (VEC
// float4 per thread): every SM issues one burst of loads for its group, two
// block reductions give the exact mean and the centered M2, then the group is
// normalised and stored.  No cluster, no exchange: CTAs of different groups
// overlap each other's phases.
template <int T>
__device__ __forceinline__ float group_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();  // red is free (previous reduction fully read)
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = lane < T / 32 ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;  // same value in every thread (same butterfly order)
}

template <bool SWISH, int T, int VEC>
__global__ void __launch_bounds__(T, 1) gn_group_kernel(
    const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ y, int spatial, int cpg, int groups, float eps) {
  __shared__ float red[32];
  const long long grp = blockIdx.x;
  const int g = (int)(grp % groups);
  const int gsize = cpg * spatial;
  const int nvec = gsize / 4;
  const float4* src = reinterpret_cast<const float4*>(x + grp * gsize);
  float4 v[VEC];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const int i = threadIdx.x + j * T;
    if (i < nvec) {
      v[j] = __ldcs(src + i);
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
  }
  const float mean = group_sum<T>(s, red) / (float)gsize;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const int i = threadIdx.x + j * T;
    if (i < nvec) {
      const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float rstd = 1.0f / sqrtf(group_sum<T>(q, red) / (float)gsize + eps);
  float4* dst = reinterpret_cast<float4*>(y + grp * gsize);
  const unsigned sp = (unsigned)spatial;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const int i = threadIdx.x + j * T;
    if (i < nvec) {
      const int ch = g * cpg + (int)((4u * (unsigned)i) / sp);  // spatial % 4 == 0
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

// Persistent: grid.x = CL * clusters, cluster (CL,1,1).  slice = elements per
// CTA (multiple of 4); stages = ring depth (>= 3).
//
// Iteration li normalises group li and, before that, reduces group li+1 and
// sends its summary, so the exchange of group li's summaries has a whole
// iteration to land: no CTA waits on a slower peer in steady state.  A CTA's
// summary of group k goes to slot k % 4 of every peer (st.async, completing
// on the peer's xbar[k % 4]); four slots are enough because a CTA sends
// summary k+1 only after it received everyone's summary k-1, which each peer
// sent after finishing iteration k-3, i.e. after it last read slot (k+1) % 4.
template <bool SWISH>
__global__ void __launch_bounds__(kThreads) gn_stream_kernel(
    const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ y, long long groups_total, int spatial, int cpg, int groups, float eps,
    int slice, int stages, unsigned int* status) {
  constexpr int NS = 4;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(128) uint8_t gn_smem[];
  __shared__ float3 wpart[kThreads / 32];       // per-warp (count, mean, M2)
  __shared__ __align__(8) float2 part[NS][8];   // [slot][rank]: (mean, M2)
  __shared__ __align__(8) uint64_t xbar[NS];    // completes when all CL pairs landed
  float* ring = reinterpret_cast<float*>(gn_smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(gn_smem + (size_t)stages * slice * 4);
  const int CL = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const long long cid = blockIdx.x / CL, ncl = gridDim.x / CL;
  const long long n_local = cid < groups_total ? (groups_total - cid + ncl - 1) / ncl : 0;
  const int gsize = cpg * spatial;  // < 2^31: bounded by the launcher
  const uint32_t bytes = (uint32_t)slice * 4u;
  const int nvec = slice / 4;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) ptx::mbar_init(&full[i], 1);
    for (int i = 0; i < NS; ++i) ptx::mbar_init(&xbar[i], 1);
    ptx::fence_mbar_init();
  }
  cluster.sync();  // every CTA's barriers exist before any peer signals them
  auto issue = [&](long long li) {
    if (li >= n_local) return;
    const long long grp = cid + li * ncl;
    const int st = (int)(li % stages);
    ptx::mbar_arrive_expect_tx(&full[st], bytes);
    ptx::bulk_load(ring + (size_t)st * slice, x + grp * gsize + (long long)rank * slice, bytes,
                   &full[st]);
  };
  // Reduce the slice of local group li (already in its stage) and send the
  // (mean, M2) summary to every CTA of the cluster.  A timed-out wait is
  // recorded and the summary is sent anyway, so no peer waits for one that
  // never comes.
  auto reduce_send = [&](long long li) {
    const int st = (int)(li % stages);
    if (threadIdx.x == 0) ptx::mbar_arrive_expect_tx(&xbar[li % NS], (uint32_t)(8 * CL));
    ptx::mbar_wait(&full[st], (uint32_t)((li / stages) & 1), status, 0x401, nullptr);
    const float4* src = reinterpret_cast<const float4*>(ring + (size_t)st * slice);
    float s = 0.f, cnt = 0.f;
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      const float4 v = src[i];
      s += (v.x + v.y) + (v.z + v.w);
      cnt += 4.f;
    }
    float mean = cnt > 0.f ? s / cnt : 0.f, m2 = 0.f;
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      const float4 v = src[i];
      const float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
      m2 += (a * a + b * b) + (c * c + d * d);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float nb = __shfl_xor_sync(0xffffffffu, cnt, o);
      const float mb = __shfl_xor_sync(0xffffffffu, mean, o);
      const float qb = __shfl_xor_sync(0xffffffffu, m2, o);
      if (lane & o) {  // lower lane's summary first: both partners get the same bits
        float n2 = nb, mean2 = mb, m22 = qb;
        chan_merge(n2, mean2, m22, cnt, mean, m2);
        cnt = n2; mean = mean2; m2 = m22;
      } else {
        chan_merge(cnt, mean, m2, nb, mb, qb);
      }
    }
    if (lane == 0) wpart[warp] = make_float3(cnt, mean, m2);
    __syncthreads();
    if (threadIdx.x < CL) {
      float n = 0.f, mn = 0.f, q = 0.f;
      for (int w = 0; w < kThreads / 32; ++w) chan_merge(n, mn, q, wpart[w].x, wpart[w].y, wpart[w].z);
      const uint32_t peer = threadIdx.x;
      ptx::st_async_v2(ptx::mapa(ptx::smem_u32(&part[li % NS][rank]), peer), mn, q,
                       ptx::mapa(ptx::smem_u32(&xbar[li % NS]), peer));
    }
    __syncthreads();  // wpart is reused by the next reduction
  };

  if (threadIdx.x == 0)
    for (int i = 0; i < stages - 1; ++i) issue(i);
  if (n_local > 0) reduce_send(0);
  for (long long li = 0; li < n_local; ++li) {
    // the stage of li + stages - 1 was freed at the end of iteration li - 1
    if (threadIdx.x == 0) issue(li + stages - 1);
    if (li + 1 < n_local) reduce_send(li + 1);
    const int slot = (int)(li % NS);
    ptx::mbar_wait(&xbar[slot], (uint32_t)((li / NS) & 1), status, 0x402, nullptr);
    // equal-count merge of the CL slices, same order in every CTA
    float gn = 0.f, gmean = 0.f, gm2 = 0.f;
    for (int r = 0; r < CL; ++r)
      chan_merge(gn, gmean, gm2, (float)slice, part[slot][r].x, part[slot][r].y);
    const float rstd = 1.0f / sqrtf(gm2 / (float)gsize + eps);

    const long long grp = cid + li * ncl;
    const int g = (int)(grp % groups);
    const float4* src = reinterpret_cast<const float4*>(ring + (size_t)(li % stages) * slice);
    float4* dst = reinterpret_cast<float4*>(y + grp * gsize + (long long)rank * slice);
    const unsigned e0 = (unsigned)(rank * slice);  // element offset inside the group
    const unsigned sp = (unsigned)spatial;
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      const float4 v = src[i];
      const int ch = g * cpg + (int)((e0 + 4u * (unsigned)i) / sp);  // spatial % 4 == 0
      const float ga = __ldg(gamma + ch) * rstd, be = __ldg(beta + ch);
      float4 o;
      o.x = act_fast((v.x - gmean) * ga + be, SWISH);
      o.y = act_fast((v.y - gmean) * ga + be, SWISH);
      o.z = act_fast((v.z - gmean) * ga + be, SWISH);
      o.w = act_fast((v.w - gmean) * ga + be, SWISH);
      __stcs(dst + i, o);
    }
    __syncthreads();  // stage li is free for the copy issued next iteration
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

// Vectorised chunked path (x, y 16-byte aligned, spatial % 4 == 0): kernel
// 1 reduces each 8192-element chunk from registers to (mean, M2); kernel 2
// loads its chunk first, merges the group's partials while the loads are in
// flight, then normalises.  x is read twice, but a tensor that fits in L2
// (126 MB) is mostly served from there the second time.
constexpr int kChunkVec = 8;  // float4 per thread: 8192-element chunks

__global__ void __launch_bounds__(kThreads) gn_partial_vec_kernel(const float* __restrict__ x,
                                                                  float2* __restrict__ partials,
                                                                  long long gsize, int chunk) {
  __shared__ float3 wpart[kThreads / 32];
  const long long grp = blockIdx.y;
  const long long c0 = (long long)blockIdx.x * chunk;
  const int nvec = (int)(std::min<long long>(c0 + chunk, gsize) - c0) / 4;
  const float4* src = reinterpret_cast<const float4*>(x + grp * gsize + c0);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float4 v[kChunkVec];
  float s = 0.f, cnt = 0.f;
#pragma unroll
  for (int j = 0; j < kChunkVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      v[j] = src[i];  // default caching: the apply kernel re-reads this chunk
      s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
      cnt += 4.f;
    }
  }
  float mean = cnt > 0.f ? s / cnt : 0.f, m2 = 0.f;
#pragma unroll
  for (int j = 0; j < kChunkVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
      m2 += (a * a + b * b) + (c * c + d * d);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float nb = __shfl_xor_sync(0xffffffffu, cnt, o);
    const float mb = __shfl_xor_sync(0xffffffffu, mean, o);
    const float qb = __shfl_xor_sync(0xffffffffu, m2, o);
    if (lane & o) {  // lower lane's summary first: both partners get the same bits
      float n2 = nb, mean2 = mb, m22 = qb;
      chan_merge(n2, mean2, m22, cnt, mean, m2);
      cnt = n2; mean = mean2; m2 = m22;
    } else {
      chan_merge(cnt, mean, m2, nb, mb, qb);
    }
  }
  if (lane == 0) wpart[warp] = make_float3(cnt, mean, m2);
  __syncthreads();
  if (threadIdx.x == 0) {
    float n = 0.f, mn = 0.f, q = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) chan_merge(n, mn, q, wpart[w].x, wpart[w].y, wpart[w].z);
    partials[grp * gridDim.x + blockIdx.x] = make_float2(mn, q);
  }
}

template <bool SWISH>
__global__ void __launch_bounds__(kThreads) gn_apply_vec_kernel(
    const float* __restrict__ x, const float2* __restrict__ partials,
    const float* __restrict__ gamma, const float* __restrict__ beta, float* __restrict__ y,
    long long gsize, int chunk, int nchunks, int spatial, int cpg, int groups, float eps) {
  __shared__ float stat[2];
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
  float4* dst = reinterpret_cast<float4*>(y + grp * gsize + c0);
#pragma unroll
  for (int j = 0; j < kChunkVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < nvec) {
      const int ch = g * cpg + (int)((c0 + 4LL * i) / spatial);  // spatial % 4 == 0
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

constexpr int kStreamSmem = 100 * 1024;  // ring budget: two CTAs per SM
constexpr int kSliceMax = 16 * 1024;      // floats per CTA slice (64 KiB)

template <bool SWISH>
agpu_status launch_stream(agpu_device* dev, const float* x, const float* gamma,
                          const float* beta, float* y, long long groups_total, int spatial,
                          int cpg, int groups, float eps, int cl, int slice, cudaStream_t s) {
  const int bytes = slice * 4;
  const int stages = std::max(3, std::min(6, kStreamSmem / bytes));
  const int smem = stages * bytes + stages * 8;
  auto kern = gn_stream_kernel<SWISH>;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)cl, 1, 1);
  // co-resident clusters for (device, CL, ring size), looked up once
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int> fits;
  int active = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev->ordinal, cl, smem);
    auto it = fits.find(key);
    if (it == fits.end()) {
      // one limit for every ring size (3 x 64 KiB slices is the largest)
      AGPU_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     3 * kSliceMax * 4 + 64));
      AGPU_CUDA(cudaOccupancyMaxActiveClusters(&active, kern, &cfg));
      it = fits.emplace(key, active).first;
    }
    active = it->second;
  }
  if (active < 1) return fail(AGPU_ERR_UNSUPPORTED, "group_norm: cluster of %d does not fit", cl);
  const long long clusters = std::min<long long>(groups_total, active);
  cfg.gridDim = dim3((unsigned)(clusters * cl), 1, 1);
  AGPU_CUDA(cudaLaunchKernelEx(&cfg, kern, x, gamma, beta, y, groups_total, spatial, cpg, groups,
                               eps, slice, stages, dev->d_status));
  return after_launch(dev, "gn_stream_kernel");
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
  // One CTA per group with the group in registers, up to 48K elements.
  if (aligned && spatial % 4 == 0 && gsize <= 1024LL * 12 * 4 &&
      groups_total < (1LL << 31)) {
    const unsigned grid = (unsigned)groups_total;
    const int sp = (int)spatial, cp = (int)cpg, gr = (int)groups;
#define AGPU_GN_GROUP(T, V)                                                                    \
    if (gsize <= (long long)(T) * (V) * 4) {                                                   \
      if (swish) gn_group_kernel<true, T, V><<<grid, T, 0, s>>>(x, gamma, beta, y, sp, cp, gr, eps); \
      else gn_group_kernel<false, T, V><<<grid, T, 0, s>>>(x, gamma, beta, y, sp, cp, gr, eps); \
      return after_launch(dev, "gn_group_kernel");                                            \
    }
    AGPU_GN_GROUP(256, 4)
    AGPU_GN_GROUP(256, 8)
    AGPU_GN_GROUP(512, 8)
    AGPU_GN_GROUP(1024, 8)
    AGPU_GN_GROUP(1024, 12)
#undef AGPU_GN_GROUP
  }
  // Streaming cluster path: a group split over CL <= 8 CTAs, each slice a
  // multiple of 4 elements.  Prefer the smallest CL whose slice is at most
  // 24 KiB (a ring of four or more slices per CTA, two CTAs per SM), else the
  // smallest CL whose slice fits 64 KiB.
  if (aligned && spatial % 4 == 0 && gsize <= 8LL * kSliceMax) {
    int pick = 0;
    for (int pass = 0; pass < 2 && !pick; ++pass) {
      const long long cap = pass == 0 ? 6 * 1024 : kSliceMax;
      for (int cl = 1; cl <= 8; ++cl) {
        if (gsize % (4LL * cl) == 0 && gsize / cl <= cap) { pick = cl; break; }
      }
    }
    if (pick) {
      const int sl = (int)(gsize / pick);
      return swish ? launch_stream<true>(dev, x, gamma, beta, y, groups_total, (int)spatial,
                                         (int)cpg, (int)groups, eps, pick, sl, s)
                   : launch_stream<false>(dev, x, gamma, beta, y, groups_total, (int)spatial,
                                          (int)cpg, (int)groups, eps, pick, sl, s);
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
  launch_chunked(x, static_cast<float2*>(buf), gamma, beta, y, gsize, chunk, (int)nchunks,
                 (int)spatial, (int)cpg, (int)groups, eps, swish, aligned && spatial % 4 == 0,
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
