// fp32-in / fp32-out GEMM for matmul and batch_matmul on sm_100a.
//
// Replaces the reference's 16x16 shared-memory FFMA shaders SHADER_MATMUL and
// SHADER_BATCH_MATMUL (src/ops/conv.rs:23-78, 91-148), which compute
// C[b] = A[b] * B[b] row-major with one output per thread.
//
// Tensor-core path (tcgen05, kind::tf32, fp32 accumulate in tensor memory):
//   * persistent CTAs (one per SM), tiles 128 x BN (BN = 256 or 128), BK = 32
//     (one 128-byte swizzle atom of fp32), tiles walk batch-major with a
//     16-row-block group swizzle for L2 reuse;
//   * warp 0 issues TMA loads into a STAGES-deep shared-memory ring,
//     warp 1 owns tensor memory and issues tcgen05.mma from one thread,
//     warps 2-5 drain the double-buffered TMEM accumulator (tcgen05.ld),
//     transpose 32x32 blocks through shared memory and write coalesced rows;
//   * A may be K-major (stored [M,K]) or MN-major (stored [K,M]), B may be
//     MN-major (stored [K,N], the reference layout) or K-major (stored [N,K]);
//     kind::tf32 accepts both majors, so no transpose pre-pass is needed for
//     any of C=A*B, C=A*B^T, C=A^T*B (the autograd backward GEMMs).
//   * 3xTF32 mode: two converter warps split every staged tile in place into
//     hi = tf32(x) and lo = x - hi (a second buffer), and the MMA warp issues
//     hi*hi + hi*lo + lo*hi into the same accumulator (error-corrected TF32,
//     Ootomo & Yokota 2022), giving fp32-level accuracy.
//
// SIMT path (exact fp32 FFMA): shapes whose row pitch is not a multiple of
// 16 bytes (TMA cannot address them), tiny problems, and AGPU_PREC_FFMA.
#include <cuda.h>

#include <algorithm>

#include "agpu_internal.cuh"
#include "ptx.cuh"

namespace agpu {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;              // fp32 elements per 128-byte swizzle row
constexpr int kEpiWarps = 4;
constexpr int kEpiStride = 36;      // floats per staging row (conflict-free float4)

template <int BN, bool X3>
struct GemmCfg {
  static constexpr int STAGES = X3 ? (BN == 256 ? 2 : 3) : (BN == 256 ? 4 : 6);
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // X3 keeps a second ("lo") copy of each stage.
  static constexpr int RING_BYTES = STAGE_BYTES * STAGES * (X3 ? 2 : 1);
  static constexpr int EPI_BYTES = kEpiWarps * 32 * kEpiStride * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
  static constexpr int THREADS = 192 + (X3 ? 64 : 0);
};

struct GemmShape {
  int M, N, K, batch;
  int tiles_m, tiles_n;
  long long num_tiles;
  long long ldc;        // = N
  long long c_batch;    // = M*N
};

__device__ __forceinline__ void tile_coords(const GemmShape& s, long long t, int BN_, int& b,
                                            int& m0, int& n0) {
  const long long per_batch = (long long)s.tiles_m * s.tiles_n;
  b = (int)(t / per_batch);
  int r = (int)(t % per_batch);
  constexpr int G = 16;
  const int group_span = G * s.tiles_n;
  const int gid = r / group_span;
  const int first_m = gid * G;
  const int gsize = min(s.tiles_m - first_m, G);
  const int in_group = r % group_span;
  const int mb = first_m + in_group % gsize;
  const int nb = in_group / gsize;
  m0 = mb * BM;
  n0 = nb * BN_;
}

// Shared-memory descriptor of one MMA's K-slice of an operand tile.
//  K-major  (rows of 32 fp32 = 128 B along K): 128-byte swizzle (layout 2),
//           8-row groups 1024 B apart; the K-slice advances 32 B in the row.
//  MN-major (32-element MN chunks of BK rows, 4 KB per chunk): 128-byte
//           swizzle with 32-byte atoms (layout 1, the only layout the tensor
//           core accepts for MN-major 32-bit operands); chunks 4 KB apart
//           (leading offset), 4-row K groups 512 B apart (stride offset); the
//           K-slice of 8 rows advances 1024 B.
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t saddr) {
  return MN ? ptx::make_sdesc(saddr, BK * 128, 512, 1) : ptx::make_sdesc(saddr, 16, 1024, 2);
}

// Split every fp32 word of a staged tile into hi (kept in place, exactly a
// tf32 value) and lo = x - hi (written to the twin buffer).  Works on the
// raw smem image, so it is independent of the swizzle.
__device__ __forceinline__ void split_tf32(uint32_t* hi, uint32_t* lo, int words, int tid,
                                           int nthreads) {
  for (int i = tid * 4; i < words; i += nthreads * 4) {
    uint4 v = *reinterpret_cast<uint4*>(hi + i);
    uint4 h, l;
    h.x = v.x & 0xFFFFE000u; h.y = v.y & 0xFFFFE000u;
    h.z = v.z & 0xFFFFE000u; h.w = v.w & 0xFFFFE000u;
    l.x = __float_as_uint(__uint_as_float(v.x) - __uint_as_float(h.x));
    l.y = __float_as_uint(__uint_as_float(v.y) - __uint_as_float(h.y));
    l.z = __float_as_uint(__uint_as_float(v.z) - __uint_as_float(h.z));
    l.w = __float_as_uint(__uint_as_float(v.w) - __uint_as_float(h.w));
    *reinterpret_cast<uint4*>(hi + i) = h;
    *reinterpret_cast<uint4*>(lo + i) = l;
  }
}

template <int BN, bool A_MN, bool B_MN, bool X3>
__global__ void __launch_bounds__(GemmCfg<BN, X3>::THREADS, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b, float* __restrict__ C,
                     GemmShape shape, unsigned int* status) {
  using Cfg = GemmCfg<BN, X3>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* epi = reinterpret_cast<float*>(smem + Cfg::RING_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::RING_BYTES + Cfg::EPI_BYTES);
  uint64_t* full = bars;                 // [STAGES] TMA landed
  uint64_t* empty = bars + STAGES;       // [STAGES] MMA done reading
  uint64_t* conv = bars + 2 * STAGES;    // [STAGES] (X3) split done
  uint64_t* tfull = bars + 3 * STAGES;   // [2] accumulator ready
  uint64_t* tempty = tfull + 2;          // [2] accumulator drained
  uint64_t* drain = tempty + 2;          // [1] all MMAs retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  auto stage_a = [&](int s) { return ring + s * Cfg::STAGE_BYTES; };
  auto stage_b = [&](int s) { return ring + s * Cfg::STAGE_BYTES + Cfg::A_BYTES; };
  auto lo_a = [&](int s) { return ring + (STAGES + s) * Cfg::STAGE_BYTES; };
  auto lo_b = [&](int s) { return ring + (STAGES + s) * Cfg::STAGE_BYTES + Cfg::A_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      ptx::mbar_init(&conv[s], 64);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&tfull[i], 1);
      ptx::mbar_init(&tempty[i], kEpiWarps * 32);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_k = (shape.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer --
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      long long issued = 0;
      for (long long t = blockIdx.x; t < shape.num_tiles && ok; t += gridDim.x) {
        int b, m0, n0;
        tile_coords(shape, t, BN, b, m0, n0);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, status, 0x101, abort_flag)) {
            ok = false;
            break;
          }
          const int k0 = kb * BK;
          ptx::mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          uint8_t* sa = stage_a(stage);
          uint8_t* sb = stage_b(stage);
          if (!A_MN) {
            ptx::tma_load_3d(sa, &tmap_a, &full[stage], k0, m0, b);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 32; ++j)
              ptx::tma_load_3d(sa + j * BK * 128, &tmap_a, &full[stage], m0 + 32 * j, k0, b);
          }
          if (!B_MN) {
            ptx::tma_load_3d(sb, &tmap_b, &full[stage], k0, n0, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j)
              ptx::tma_load_3d(sb + j * BK * 128, &tmap_b, &full[stage], n0 + 32 * j, k0, b);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Never leave while TMA writes into this CTA's shared memory are still
      // in flight: wait (bounded) for the last load issued into each stage.
      for (int s = 0; s < STAGES && s < issued; ++s) {
        const long long round = (issued - 1 - s) / STAGES;
        ptx::mbar_wait(&full[s], (uint32_t)(round & 1), status, 0x107, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer --
    constexpr uint32_t idesc = ptx::make_idesc_tf32(BM, BN, A_MN, B_MN);
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (long long t = blockIdx.x; t < shape.num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!ptx::mbar_wait(&tempty[acc], acc_phase ^ 1, status, 0x102, abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          uint64_t* ready = X3 ? &conv[stage] : &full[stage];
          if (!ptx::mbar_wait(ready, phase, status, 0x103, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(stage_a(stage));
          const uint32_t b_addr = ptx::smem_u32(stage_b(stage));
          const uint32_t la_addr = ptx::smem_u32(lo_a(stage));
          const uint32_t lb_addr = ptx::smem_u32(lo_b(stage));
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            // K-major: advance 8 fp32 = 32 B inside the swizzle row.
            // MN-major: advance 8 rows of 128 B.
            const uint32_t a_off = A_MN ? kk * 1024 : kk * 32;
            const uint32_t b_off = B_MN ? kk * 1024 : kk * 32;
            const uint64_t ad = operand_desc<A_MN>(a_addr + a_off);
            const uint64_t bd = operand_desc<B_MN>(b_addr + b_off);
            const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
            ptx::mma_tf32_ss(d_tmem, ad, bd, idesc, accum);
            if (X3) {
              const uint64_t bl = operand_desc<B_MN>(lb_addr + b_off);
              const uint64_t al = operand_desc<A_MN>(la_addr + a_off);
              ptx::mma_tf32_ss(d_tmem, ad, bl, idesc, 1u);
              ptx::mma_tf32_ss(d_tmem, al, bd, idesc, 1u);
            }
          }
          ptx::mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit(&tfull[acc]);
      }
      // Retire every MMA this thread issued before tensor memory is freed.
      ptx::mma_commit(drain);
      ptx::mbar_wait(drain, 0, status, 0x104, nullptr);
    }
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue --
    const int q = warp & 3;  // TMEM sub-partition this warp may access
    float* stg = epi + (warp - 2) * 32 * kEpiStride;
    int local = 0;
    for (long long t = blockIdx.x; t < shape.num_tiles; t += gridDim.x, ++local) {
      int b, m0, n0;
      tile_coords(shape, t, BN, b, m0, n0);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!ptx::mbar_wait(&tfull[acc], acc_phase, status, 0x105, abort_flag)) break;
      ptx::tc_fence_after();
      float* Cb = C + (long long)b * shape.c_batch;
      const int row_base = m0 + q * 32;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        if (n0 + c * 32 >= shape.N) break;  // warp-uniform
        uint32_t v[32];
        ptx::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + c * 32, v);
        ptx::tmem_wait_ld();
        // lane holds row (row_base+lane), columns n0+c*32 .. +31
        float4* srow = reinterpret_cast<float4*>(stg + lane * kEpiStride);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          srow[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
        __syncwarp();
        const int col = n0 + c * 32 + (lane & 7) * 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = i * 4 + (lane >> 3);
          const int row = row_base + r;
          float4 val = *reinterpret_cast<const float4*>(stg + r * kEpiStride + (lane & 7) * 4);
          if (row < shape.M && col < shape.N)
            *reinterpret_cast<float4*>(Cb + (long long)row * shape.ldc + col) = val;
        }
        __syncwarp();
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&tempty[acc]);
    }
  } else if (X3) {
    // ---------------------------------------------- 3xTF32 split (2 warps) --
    const int ctid = threadIdx.x - (2 + kEpiWarps) * 32;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < shape.num_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < num_k; ++kb) {
        if (!ptx::mbar_wait(&full[stage], phase, status, 0x106, abort_flag)) { ok = false; break; }
        split_tf32(reinterpret_cast<uint32_t*>(stage_a(stage)),
                   reinterpret_cast<uint32_t*>(lo_a(stage)), Cfg::STAGE_BYTES / 4, ctid, 64);
        ptx::fence_proxy_async_smem();  // generic writes -> visible to the MMA (async proxy)
        ptx::mbar_arrive(&conv[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------ SIMT FFMA --
// Exact fp32 GEMM, 64x64 tile per 256 threads, 4x4 outputs per thread,
// arbitrary strides/alignment.  a_trans: A stored [K,M]; b_trans: B stored [N,K].
template <bool AT, bool BT>
__global__ void __launch_bounds__(256) gemm_ffma_kernel(const float* __restrict__ A,
                                                        const float* __restrict__ B,
                                                        float* __restrict__ C, int M, int N,
                                                        int K) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int b = blockIdx.z;
  A += (long long)b * M * K;
  B += (long long)b * K * N;
  C += (long long)b * M * N;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i / 64, mm = i % 64;
      const int gm = m0 + mm, gk = k0 + kk;
      float av = 0.f;
      if (gm < M && gk < K) av = AT ? A[(long long)gk * M + gm] : A[(long long)gm * K + gk];
      As[kk][mm] = av;
      const int gn = n0 + mm;
      float bv = 0.f;
      if (gn < N && gk < K) bv = BT ? B[(long long)gn * K + gk] : B[(long long)gk * N + gn];
      Bs[kk][mm] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn < N) C[(long long)gm * N + gn] = acc[i][j];
    }
  }
}

// ------------------------------------------------------ tensor-map encode --
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

// 3-D fp32 tensor map {inner, outer, batch}.  `mn_major` selects the
// 128-byte swizzle with 32-byte atoms that MN-major tf32 operands need;
// otherwise the plain 128-byte swizzle.
agpu_status make_tmap_f32_3d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer,
                             uint64_t batch, uint64_t batch_stride_elems, uint32_t box_inner,
                             uint32_t box_outer, bool mn_major) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AGPU_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {inner * 4, batch_stride_elems * 4};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(AGPU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) inner=%llu outer=%llu", (int)r,
                (unsigned long long)inner, (unsigned long long)outer);
  return AGPU_OK;
}

template <int BN, bool A_MN, bool B_MN, bool X3>
static agpu_status run_tc(agpu_device* dev, const float* a, const float* b, float* c,
                          uint32_t batch, uint32_t m, uint32_t n, uint32_t k, cudaStream_t s) {
  using Cfg = GemmCfg<BN, X3>;
  CUtensorMap ta, tb;
  // A: K-major stored [M,K] -> dims {K, M}; MN-major stored [K,M] -> dims {M, K}.
  if (!A_MN)
    AGPU_TRY(make_tmap_f32_3d(&ta, a, k, m, batch, (uint64_t)m * k, BK, BM, false));
  else
    AGPU_TRY(make_tmap_f32_3d(&ta, a, m, k, batch, (uint64_t)m * k, 32, BK, true));
  // B: MN-major stored [K,N] -> dims {N, K}; K-major stored [N,K] -> dims {K, N}.
  if (B_MN)
    AGPU_TRY(make_tmap_f32_3d(&tb, b, n, k, batch, (uint64_t)k * n, 32, BK, true));
  else
    AGPU_TRY(make_tmap_f32_3d(&tb, b, k, n, batch, (uint64_t)k * n, BK, BN, false));
  GemmShape sh;
  sh.M = m; sh.N = n; sh.K = k; sh.batch = batch;
  sh.tiles_m = (int)ceil_div(m, BM);
  sh.tiles_n = (int)ceil_div(n, BN);
  sh.num_tiles = (long long)sh.tiles_m * sh.tiles_n * batch;
  sh.ldc = n;
  sh.c_batch = (long long)m * n;
  auto kern = gemm_tf32_kernel<BN, A_MN, B_MN, X3>;
  AGPU_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
  const long long grid = std::min<long long>(sh.num_tiles, dev->sm_count);
  kern<<<(unsigned)grid, Cfg::THREADS, Cfg::SMEM, s>>>(ta, tb, c, sh, dev->d_status);
  return after_launch(dev, "gemm_tf32_kernel");
}

template <bool X3>
static agpu_status dispatch_tc(agpu_device* dev, const float* a, const float* b, float* c,
                               uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool at,
                               bool bt, cudaStream_t s) {
  const bool wide = n > 128;
  // B is MN-major unless stored transposed ([N,K]).
  if (wide) {
    if (!at && !bt) return run_tc<256, false, true, X3>(dev, a, b, c, batch, m, n, k, s);
    if (!at && bt) return run_tc<256, false, false, X3>(dev, a, b, c, batch, m, n, k, s);
    if (at && !bt) return run_tc<256, true, true, X3>(dev, a, b, c, batch, m, n, k, s);
    return run_tc<256, true, false, X3>(dev, a, b, c, batch, m, n, k, s);
  }
  if (!at && !bt) return run_tc<128, false, true, X3>(dev, a, b, c, batch, m, n, k, s);
  if (!at && bt) return run_tc<128, false, false, X3>(dev, a, b, c, batch, m, n, k, s);
  if (at && !bt) return run_tc<128, true, true, X3>(dev, a, b, c, batch, m, n, k, s);
  return run_tc<128, true, false, X3>(dev, a, b, c, batch, m, n, k, s);
}

static agpu_status run_ffma(agpu_device* dev, const float* a, const float* b, float* c,
                            uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool at, bool bt,
                            cudaStream_t s) {
  dim3 grid((unsigned)ceil_div(n, 64), (unsigned)ceil_div(m, 64), batch);
  if (!at && !bt) gemm_ffma_kernel<false, false><<<grid, 256, 0, s>>>(a, b, c, m, n, k);
  else if (!at && bt) gemm_ffma_kernel<false, true><<<grid, 256, 0, s>>>(a, b, c, m, n, k);
  else if (at && !bt) gemm_ffma_kernel<true, false><<<grid, 256, 0, s>>>(a, b, c, m, n, k);
  else gemm_ffma_kernel<true, true><<<grid, 256, 0, s>>>(a, b, c, m, n, k);
  return after_launch(dev, "gemm_ffma_kernel");
}

// Whether the tensor-core path can address these operands with TMA: every
// row pitch and batch stride must be a multiple of 16 bytes.
bool gemm_tc_eligible(const float* a, const float* b, const float* c, uint32_t m, uint32_t n,
                      uint32_t k) {
  const uintptr_t mis = (reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(c)) & 15u;
  return mis == 0 && (k % 4 == 0) && (n % 4 == 0) && (m % 4 == 0) && k >= 8;
}

agpu_status launch_gemm(agpu_device* dev, const float* a, const float* b, float* c,
                        uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool a_trans,
                        bool b_trans, cudaStream_t s) {
  if (batch == 0 || m == 0 || n == 0) return AGPU_OK;
  if (k == 0) {
    AGPU_CUDA(cudaMemsetAsync(c, 0, (size_t)batch * m * n * sizeof(float), s));
    return AGPU_OK;
  }
  const agpu_precision p = dev->precision;
  const bool tiny = (uint64_t)m * n * k * batch < (1ull << 15);
  if (p == AGPU_PREC_FFMA || tiny || !gemm_tc_eligible(a, b, c, m, n, k))
    return run_ffma(dev, a, b, c, batch, m, n, k, a_trans, b_trans, s);
  if (p == AGPU_PREC_TF32X3)
    return dispatch_tc<true>(dev, a, b, c, batch, m, n, k, a_trans, b_trans, s);
  return dispatch_tc<false>(dev, a, b, c, batch, m, n, k, a_trans, b_trans, s);
}

}  // namespace agpu
