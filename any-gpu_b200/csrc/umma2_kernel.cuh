// CTA-pair (cta_group::2) version of the tcgen05 kind::tf32 mainloop: one
// 256 x BN tile per pair of CTAs (a cluster of 2 on neighbouring SMs).
//
// Each CTA stages only half of every K-block -- its 128 rows of A and BN/2
// columns of B -- and the pair's tensor cores read both halves of B, so each
// SM moves two thirds of the shared-memory bytes per FLOP of the single-CTA
// 128 x BN tile.  With fp32 operands the single-CTA tile needs more shared-
// memory bandwidth (TMA writes + MMA reads) than an SM has; the pair fits.
//
//   both CTAs  warp 0: TMA of the CTA's halves; completion is signalled on the
//              leader CTA's full barrier (cp.async.bulk.tensor .cta_group::2),
//              no multicast.  warps 2-5: drain this CTA's TMEM rows (128 of
//              the tile's 256) and arrive (one lane per warp) on the leader's
//              "accumulator empty" barrier.  warp 1 allocates tensor memory for the pair.
//   leader     warp 1 lane 0 issues tcgen05.mma.cta_group::2 (M 256) and
//              commits to the barriers of both CTAs (commit multicast mask).
//
// Every mbarrier wait is bounded; both CTAs always reach the closing cluster
// barrier, after which the pair frees its tensor memory.
#pragma once

#include <cuda.h>

#include "ptx.cuh"
#include "umma_kernel.cuh"

namespace agpu {
namespace umma {

// Tiles wider than one MMA (BN > 256) issue NMMA = 2 MMAs of N = BN/2 per K
// step into adjacent TMEM columns; B is then staged as NMMA sub-blocks of
// MMA_N/2 columns per CTA (sub-block s of CTA r = tile columns
// s*MMA_N + r*MMA_N/2 ..).  An accumulator of 2*BN > 512 columns cannot be
// double-buffered: the MMA then waits for the epilogue between tiles, which
// the wider tile amortises (and it halves the TMA bytes per FLOP of B).
// EXTRA_: further epilogue shared memory a policy asks for (P::EPI_EXTRA,
// split evenly over the epilogue warps, 1024-byte aligned per warp).
template <int BN_, int EXTRA_ = 0>
struct PairCfg {
  static constexpr int BN = BN_;             // tile columns (both CTAs)
  static constexpr int NMMA = BN > 256 ? 2 : 1;
  static constexpr int MMA_N = BN / NMMA;
  static constexpr int ACC = 2 * BN <= 512 ? 2 : 1;      // accumulator buffers
  static_assert(BN % NMMA == 0 && MMA_N % 16 == 0 && MMA_N <= 256, "pair tile width");
  static constexpr int A_BYTES = BM * BK * 4;            // 128 rows per CTA
  static constexpr int B_BYTES = (BN / 2) * BK * 4;      // BN/2 columns per CTA
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static_assert(EXTRA_ % (kEpiWarps * 1024) == 0, "per-warp extra epilogue memory alignment");
  static constexpr int EPI_BYTES = kEpiWarps * kEpiWarpFloats * 4 + EXTRA_;
  static constexpr int BAR_BYTES = 256;
  static constexpr int BUDGET = 227 * 1024 - 1024 - EPI_BYTES - BAR_BYTES;
  static constexpr int STAGES_RAW = BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static_assert(STAGES >= 2, "tile too large for the shared-memory ring");
  static constexpr int RING_BYTES = STAGE_BYTES * STAGES;
  static constexpr int SMEM = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr int TMEM_COLS = ACC * BN <= 256 ? 256 : 512;
  static constexpr int THREADS = 192;
};

// Policy requirements as for umma_tf32_kernel, plus
//   void load(ta, tb, sa, sb, uint32_t leader_bar, const Tile&, int kb, int rank) const;
//       issues this CTA's STAGE_BYTES with tma_load_*_pair(..., leader_bar, ...)
//   Tile rank_tile(const Tile&, int rank) const;   // the CTA's 128-row half
//   static constexpr bool TILE_EPILOGUE;  // true: where whole_tile(),
//       bool store_tile(tile, row, tmem_row_addr, staging, extra, lane,
//                       status, abort_flag) drains the tile (false: a wait expired)
//   static constexpr int EPI_EXTRA;   // bytes of extra epilogue memory (0, or
//       with void init_extra(float* slice) run once per warp slice at start)
// and, for BN > 256, the B sub-block layout described at PairCfg.
// whether a TILE_EPILOGUE policy drains this launch's tiles with store_tile
template <class P>
__device__ __forceinline__ bool tile_epi(const P& pol) {
  if constexpr (P::TILE_EPILOGUE) return pol.whole_tile();
  else return false;
}

template <class P>
__global__ void __launch_bounds__(PairCfg<P::BN>::THREADS, 1)
    umma_tf32_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                          const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ P pol,
                          unsigned int* status) {
  using C = PairCfg<P::BN, P::EPI_EXTRA>;
  constexpr int BN = P::BN;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* epi = reinterpret_cast<float*>(smem + C::RING_BYTES);
  // the policy's extra epilogue memory: one slice per epilogue warp
  [[maybe_unused]] float* xtra_base = epi + kEpiWarps * kEpiWarpFloats;
  constexpr int kXtraWarpFloats = P::EPI_EXTRA / 4 / kEpiWarps;
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
    if constexpr (P::EPI_EXTRA > 0) {
      for (int w = 0; w < kEpiWarps; ++w) pol.init_extra(xtra_base + w * kXtraWarpFloats);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // peer barriers initialised, tensor memory allocated
  ptx::tc_fence_after();
  ptx::griddep_wait();  // the previous kernel's outputs are visible from here on
  ptx::griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const int num_k = pol.num_k();
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
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, status, 0x301, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) ptx::mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          const uint32_t lbar = ptx::mapa(ptx::smem_u32(&full[stage]), 0);
          pol.load(&tmap_a, &tmap_b, stage_a(stage), stage_b(stage), lbar, tile, kb, rank);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (leader) {
        // the leader's full barriers count both CTAs' bytes: wait (bounded) for
        // the last round of each stage so no copy of the pair is in flight
        for (int s = 0; s < STAGES && s < issued; ++s) {
          const long long round = (issued - 1 - s) / STAGES;
          ptx::mbar_wait(&full[s], (uint32_t)(round & 1), status, 0x307, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = ptx::make_idesc_tf32(2 * BM, C::MMA_N, P::A_MN, P::B_MN);
      // byte offset of B sub-block s in a stage (MN-major: 32-column chunks)
      constexpr uint32_t b_sub = P::B_MN ? (C::MMA_N / 2 / 32) * BK * 128 : (C::MMA_N / 2) * 128;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (long long t = cluster_id; t < num_tiles && ok; t += n_clusters, ++local) {
        const int acc = local % C::ACC;
        const uint32_t acc_phase = (local / C::ACC) & 1;
        // the peer's epilogue warps arrive with cluster-scope release
        if (!ptx::mbar_wait<true>(&tempty[acc], acc_phase ^ 1, status, 0x302, abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, status, 0x303, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(stage_a(stage));
          const uint32_t b_addr = ptx::smem_u32(stage_b(stage));
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint32_t a_off = P::A_MN ? kk * 1024 : kk * 32;
            const uint32_t b_off = P::B_MN ? kk * 1024 : kk * 32;
#pragma unroll
            for (int sub = 0; sub < C::NMMA; ++sub)
              ptx::mma_tf32_ss_pair(d_tmem + sub * C::MMA_N,
                                    operand_desc<P::A_MN>(a_addr + a_off),
                                    operand_desc<P::B_MN>(b_addr + sub * b_sub + b_off), idesc,
                                    (kb > 0 || kk > 0) ? 1u : 0u);
          }
          ptx::mma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit_pair(&tfull[acc], 0x3);
      }
      ptx::mma_commit_pair(drain, 0x3);
      ptx::mbar_wait(drain, 0, status, 0x304, nullptr);
    }
  } else {
    const int q = warp & 3;
    float* stg = epi + (warp - 2) * kEpiWarpFloats;
    int local = 0;
    for (long long t = cluster_id; t < num_tiles; t += n_clusters, ++local) {
      const auto tile = pol.rank_tile(pol.tile(t), rank);
      const int acc = local % C::ACC;
      const uint32_t acc_phase = (local / C::ACC) & 1;
      // warp-uniform: every lane takes the same exit (the arrive below and
      // the policy's store use warp-wide syncs)
      if (!__all_sync(0xffffffffu, ptx::mbar_wait(&tfull[acc], acc_phase, status, 0x305,
                                                  abort_flag)))
        break;
      ptx::tc_fence_after();
      const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if (pol.paired()) {  // SwiGLU: gate and up blocks of 32 columns side by side
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {
          if (!pol.col_live(tile, c * 32)) break;  // warp-uniform
          uint32_t g[32], u[32];
          ptx::tmem_ld32(trow + c * 32, g);
          ptx::tmem_ld32(trow + (c + 1) * 32, u);
          ptx::tmem_wait_ld();
          pol.store_swiglu(tile, q * 32 + lane, c * 32, g, u, stg, lane);
        }
      } else if (tile_epi(pol)) {  // the policy walks the tile's chunks itself
        if constexpr (P::TILE_EPILOGUE) {
          if (!pol.store_tile(tile, q * 32 + lane, trow, stg,
                              xtra_base + (warp - 2) * kXtraWarpFloats, lane, status,
                              abort_flag))
            break;  // an expired wait (status recorded); its copies have landed
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          if (!pol.col_live(tile, c * 32)) break;  // warp-uniform
          uint32_t v[32];
          ptx::tmem_ld32(trow + c * 32, v);
          ptx::tmem_wait_ld();
          pol.store(tile, q * 32 + lane, c * 32, v, stg, lane, false, true);
        }
      }
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
