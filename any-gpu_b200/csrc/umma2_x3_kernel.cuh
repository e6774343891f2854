// 3xTF32 (error-corrected TF32, Ootomo & Yokota 2022) on CTA pairs: the
// fp32-accuracy GEMM mode on the same 256 x 256 cta_group::2 tiles as the
// TF32 pair kernel (umma2_kernel.cuh).
//
// Split.  Every operand x is x = hi + lo with hi = x with its low 13 mantissa
// bits cleared and lo = x - hi (exact in fp32).  The tensor core reads an
// fp32 operand as tf32 by ignoring those 13 bits, so it sees hi when given x
// itself: only lo is materialised, by one elementwise pass (tf32_lo_kernel)
// into scratch before the GEMM.  Per K-slice the MMA thread issues
//   D += lo(A) hi(B);  D += hi(A) lo(B);  D += hi(A) hi(B)
// (small terms first; lo(A) lo(B) is below fp32 resolution).  Each stage of
// the ring holds both parts of this CTA's halves: [A | B | lo(A) | lo(B)].
//
// K segments.  The tensor core's fp32 accumulation error grows with the
// number of MMAs summed into one accumulator, so a tile whose K loop is
// longer than `pol.seg` K-blocks is accumulated in segments: each segment
// into the accumulator (tensor-memory columns [0, BN)), and the epilogue
// warps add it in fp32 on the CUDA cores into a running sum kept in tensor
// memory (columns [BN, 2 BN)), storing to global memory only after the last
// segment.  Partial sums never leave the SM.  Tiles with one segment use
// both column ranges as a double-buffered accumulator instead.
//
// Roles, barriers and the bounded-wait / drain discipline are those of the
// TF32 pair kernel; see umma2_kernel.cuh.
#pragma once

#include <cuda.h>

#include "ptx.cuh"
#include "umma_kernel.cuh"
#include "umma2_kernel.cuh"

namespace agpu {
namespace umma {

template <int BN_>
struct PairX3Cfg {
  static constexpr int BN = BN_;
  static_assert(BN == 256, "3xTF32 pair tiles are 256 x 256");
  static constexpr int MMA_N = BN;
  static constexpr int A_BYTES = BM * BK * 4;          // 128 rows per CTA
  static constexpr int B_BYTES = (BN / 2) * BK * 4;    // BN/2 columns per CTA
  static constexpr int HI_BYTES = A_BYTES + B_BYTES;   // the operands as stored
  static constexpr int STAGE_BYTES = 2 * HI_BYTES;     // + their lo parts
  static constexpr int EPI_BYTES = kEpiWarps * kEpiWarpFloats * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int BUDGET = 227 * 1024 - 1024 - EPI_BYTES - BAR_BYTES;
  static constexpr int STAGES_RAW = BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static_assert(STAGES >= 2, "tile too large for the shared-memory ring");
  static constexpr int RING_BYTES = STAGE_BYTES * STAGES;
  static constexpr int SMEM = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // accumulator + running sum (or 2 accumulators)
  static constexpr int THREADS = 192;
};

// lo = x - hi(x), hi(x) = x with the low 13 mantissa bits cleared (what the
// tensor core reads from x in kind::tf32), for two operands in one launch:
// elements [0, n4a) of the float4 range are A's, the rest B's.  16-byte
// aligned, lengths in float4s.
__device__ __forceinline__ float tf32_lo(float v) {
  return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
}

__global__ void __launch_bounds__(256) tf32_lo_kernel(const float4* __restrict__ a,
                                                      float4* __restrict__ alo, long long n4a,
                                                      const float4* __restrict__ b,
                                                      float4* __restrict__ blo, long long n4b) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4a + n4b;
       i += stride) {
    const bool in_a = i < n4a;
    const long long j = in_a ? i : i - n4a;
    const float4 v = __ldg((in_a ? a : b) + j);
    (in_a ? alo : blo)[j] =
        make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
  }
}

// Policy requirements: those of umma_tf32_pair_kernel (tile, rank_tile, load,
// col_live, store, num_k, num_tiles, A_MN, B_MN, BN) plus `int seg`, the
// K-blocks per accumulator segment (<= 0: the whole K loop).  `load` is
// called twice per stage: with the operands' maps and with their lo maps.
template <class P>
__global__ void __launch_bounds__(PairX3Cfg<P::BN>::THREADS, 1)
    umma_x3_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_alo,
                        const __grid_constant__ CUtensorMap tmap_blo, const __grid_constant__ P pol,
                        unsigned int* status) {
  using C = PairX3Cfg<P::BN>;
  constexpr int BN = P::BN;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* epi = reinterpret_cast<float*>(smem + C::RING_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES + C::EPI_BYTES);
  uint64_t* full = bars;                // [STAGES] leader's is the one used
  uint64_t* empty = bars + STAGES;      // [STAGES] both CTAs
  uint64_t* tfull = bars + 2 * STAGES;  // [2] both CTAs
  uint64_t* tempty = tfull + 2;         // [2] leader's is the one used
  uint64_t* drain = tempty + 2;         // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int rank = (int)ptx::cluster_rank();
  const bool leader = rank == 0;
  auto stage_a = [&](int s) { return ring + s * C::STAGE_BYTES; };
  auto stage_b = [&](int s) { return ring + s * C::STAGE_BYTES + C::A_BYTES; };
  auto stage_alo = [&](int s) { return ring + s * C::STAGE_BYTES + C::HI_BYTES; };
  auto stage_blo = [&](int s) { return ring + s * C::STAGE_BYTES + C::HI_BYTES + C::A_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&tfull[i], 1);
      ptx::mbar_init(&tempty[i], 2 * kEpiWarps);  // one arrive per epilogue warp
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&tmap_alo);
    ptx::prefetch_tmap(&tmap_blo);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // peer barriers initialised, tensor memory allocated
  ptx::tc_fence_after();
  ptx::griddep_wait();  // the lo pass (the previous kernel) is visible from here on
  ptx::griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const int num_k = pol.num_k();
  const int seg = (pol.seg > 0 && pol.seg < num_k) ? pol.seg : (num_k > 0 ? num_k : 1);
  const int nseg = (num_k + seg - 1) / seg;
  // segmented tiles: one accumulator ([0, BN)) + the running sum ([BN, 2BN));
  // otherwise two accumulators, double-buffered across tiles
  const int nacc = nseg > 1 ? 1 : 2;
  const long long num_tiles = pol.num_tiles();
  const long long cluster_id = blockIdx.x / 2, n_clusters = gridDim.x / 2;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      long long issued = 0;
      for (long long t = cluster_id; t < num_tiles && ok; t += n_clusters) {
        const auto tile = pol.tile(t);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, status, 0x501, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) ptx::mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          const uint32_t lbar = ptx::mapa(ptx::smem_u32(&full[stage]), 0);
          pol.load(&tmap_a, &tmap_b, stage_a(stage), stage_b(stage), lbar, tile, kb, rank);
          pol.load(&tmap_alo, &tmap_blo, stage_alo(stage), stage_blo(stage), lbar, tile, kb,
                   rank);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (leader) {
        // the leader's full barriers count both CTAs' bytes: wait (bounded) for
        // the last round of each stage so no copy of the pair is in flight
        for (int s = 0; s < STAGES && s < issued; ++s) {
          const long long round = (issued - 1 - s) / STAGES;
          ptx::mbar_wait(&full[s], (uint32_t)(round & 1), status, 0x507, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = ptx::make_idesc_tf32(2 * BM, C::MMA_N, P::A_MN, P::B_MN);
      int stage = 0;
      uint32_t phase = 0;
      long long unit = 0;  // accumulator uses (segments) so far
      bool ok = true;
      for (long long t = cluster_id; t < num_tiles && ok; t += n_clusters) {
        for (int s = 0; s < nseg && ok; ++s, ++unit) {
          const int acc = (int)(unit % nacc);
          const uint32_t acc_phase = (uint32_t)((unit / nacc) & 1);
          // the peer's epilogue warps arrive with CTA-scope release
          if (!ptx::mbar_wait<true>(&tempty[acc], acc_phase ^ 1, status, 0x502, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          const int k0 = s * seg, k1 = min(num_k, k0 + seg);
          for (int kb = k0; kb < k1; ++kb) {
            if (!ptx::mbar_wait(&full[stage], phase, status, 0x503, abort_flag)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            const uint32_t a_addr = ptx::smem_u32(stage_a(stage));
            const uint32_t b_addr = ptx::smem_u32(stage_b(stage));
            const uint32_t alo_addr = ptx::smem_u32(stage_alo(stage));
            const uint32_t blo_addr = ptx::smem_u32(stage_blo(stage));
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk) {
              const uint32_t a_off = P::A_MN ? kk * 1024 : kk * 32;
              const uint32_t b_off = P::B_MN ? kk * 1024 : kk * 32;
              const uint64_t ah = operand_desc<P::A_MN>(a_addr + a_off);
              const uint64_t bh = operand_desc<P::B_MN>(b_addr + b_off);
              const uint64_t al = operand_desc<P::A_MN>(alo_addr + a_off);
              const uint64_t bl = operand_desc<P::B_MN>(blo_addr + b_off);
              ptx::mma_tf32_ss_pair(d_tmem, al, bh, idesc, (kb > k0 || kk > 0) ? 1u : 0u);
              ptx::mma_tf32_ss_pair(d_tmem, ah, bl, idesc, 1u);
              ptx::mma_tf32_ss_pair(d_tmem, ah, bh, idesc, 1u);
            }
            ptx::mma_commit_pair(&empty[stage], 0x3);
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          ptx::mma_commit_pair(&tfull[acc], 0x3);
        }
      }
      ptx::mma_commit_pair(drain, 0x3);
      ptx::mbar_wait(drain, 0, status, 0x504, nullptr);
    }
  } else {
    const int q = warp & 3;
    float* stg = epi + (warp - 2) * kEpiWarpFloats;
    long long unit = 0;
    bool ok = true;
    for (long long t = cluster_id; t < num_tiles && ok; t += n_clusters) {
      const auto tile = pol.rank_tile(pol.tile(t), rank);
      for (int s = 0; s < nseg; ++s, ++unit) {
        const int acc = (int)(unit % nacc);
        const uint32_t acc_phase = (uint32_t)((unit / nacc) & 1);
        // warp-uniform: every lane takes the same exit (the arrive below and
        // the policy's store use warp-wide syncs)
        if (!__all_sync(0xffffffffu, ptx::mbar_wait(&tfull[acc], acc_phase, status, 0x505,
                                                    abort_flag))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16);
        const bool last = s == nseg - 1;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          if (!pol.col_live(tile, c * 32)) break;  // warp-uniform, the same every segment
          uint32_t v[32];
          ptx::tmem_ld32(trow + acc * BN + c * 32, v);
          if (nseg > 1 && s > 0) {
            uint32_t r[32];
            ptx::tmem_ld32(trow + BN + c * 32, r);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              v[i] = __float_as_uint(__uint_as_float(v[i]) + __uint_as_float(r[i]));
          } else {
            ptx::tmem_wait_ld();
          }
          if (!last) {
            ptx::tmem_st32(trow + BN + c * 32, v);  // running sum
            continue;
          }
          pol.store(tile, q * 32 + lane, c * 32, v, stg, lane, false, true);
        }
        // the running-sum writes are complete before this thread reads them
        // back in the next segment
        if (!last) ptx::tmem_wait_st();
        // the accumulator (tensor memory) is free again; the handoff carries
        // no generic-memory data, so the peer's remote arrive is CTA-scope
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) ptx::mbar_arrive(&tempty[acc]);
          else ptx::mbar_arrive_remote(ptx::mapa(ptx::smem_u32(&tempty[acc]), 0));
        }
      }
    }
  }

  // the epilogue's bulk (TMA) stores of C are complete before the CTA exits
  if (warp >= 2 && lane == 0) ptx::bulk_wait0();
  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // the pair's MMAs are retired before either CTA frees TMEM
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace umma
}  // namespace agpu
