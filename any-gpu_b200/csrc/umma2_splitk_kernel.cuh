// Split-K over a cluster of CTA pairs, for GEMMs with too few output tiles
// to occupy the SMs (512^3: 4 tiles of 256 x 256 for 74 pairs).
//
// One cluster of 2*S CTAs per output tile: pair p (cluster ranks 2p, 2p+1)
// runs the CTA-pair tcgen05 mainloop of umma2_kernel.cuh over K-blocks
// [p*nk/S, (p+1)*nk/S) into its own tensor memory.  The partial tile is then
// reduced through distributed shared memory: every CTA copies its 128 x BN
// fp32 partial into its (drained) operand ring, the cluster synchronises,
// and CTA (p, h) sums rows [p*128/S, (p+1)*128/S) of its half h over the S
// pairs in pair order (ld.shared::cluster), applies the epilogue (bias,
// residual, activation) and writes them with coalesced float4 stores.  The
// K sum is therefore deterministic; the S-way split adds one fp32 rounding
// per slice.  Each SM streams 1/S of the tile's operand bytes, which is what
// bounds these small GEMMs (the per-SM TMA rate, not the tensor core).
//
// Roles as in the pair kernel (warp 0 TMA, warp 1 TMEM + leader MMA issue,
// warps 2-5 TMEM drain), with barrier and commit targets offset to the pair's
// leader (rank 2p) and multicast mask 0b11 << 2p.  Every mbarrier wait is
// bounded; on expiry a CTA records the status code and skips the rest of its
// mainloop, but every CTA still reaches all three cluster barriers.
#pragma once

#include <cuda.h>

#include "ptx.cuh"
#include "umma_kernel.cuh"
#include "umma2_kernel.cuh"

namespace agpu {
namespace umma {

// Plain load from distributed shared memory (ordered after the cluster
// barrier by that barrier's own memory clobber; no clobber here, so the
// compiler can keep several in flight).
__device__ __forceinline__ float4 ld_dsmem_v4(uint32_t cluster_addr) {
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "r"(cluster_addr));
  return v;
}

// Exit barrier: a relaxed arrive does not wait for this CTA's outstanding
// global stores (a release arrive would); it only has to keep every CTA's
// shared memory alive until the others' reads of it have returned.
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;"
               ::: "memory");
}

__device__ __forceinline__ float splitk_act(float x, int act) {
  if (act == 1) return x / (1.0f + expf(-x));  // swish
  if (act == 2) return fmaxf(x, 0.0f);         // relu
  return x;
}

// P: GemmPairPolicy<256, ...> (tile(), load(), and the fields M, N, C,
// c_batch, bias, resid, act).  S: K slices (pairs per cluster), 2 or 4.
template <class P, int S>
__global__ void __launch_bounds__(PairCfg<P::BN>::THREADS, 1)
    umma_tf32_pair_splitk_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                 const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ P pol,
                                 unsigned int* status) {
  using C = PairCfg<P::BN>;
  constexpr int BN = P::BN;
  constexpr int STAGES = C::STAGES;
  constexpr int PITCH = BN + 4;          // floats per partial row (conflict-free float4)
  constexpr int ROWS = BM / S;           // rows of its half each CTA reduces
  static_assert(C::NMMA == 1 && C::ACC == 2, "split-K serves 256-column pair tiles");
  static_assert(BM * PITCH * 4 <= C::RING_BYTES, "partial tile must fit in the ring");
  static_assert(S == 2 || S == 4, "2 or 4 K slices");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* part = reinterpret_cast<float*>(smem);  // [BM][PITCH], reuses the ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES + C::EPI_BYTES);
  uint64_t* full = bars;             // [STAGES] the leader's are used
  uint64_t* empty = bars + STAGES;   // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = ptx::cluster_rank();
  const int p = (int)(rank >> 1), h = (int)(rank & 1);
  const uint32_t leader = rank & ~1u;
  const uint16_t mask = (uint16_t)(0x3u << leader);
  auto stage_a = [&](int s) { return ring + s * C::STAGE_BYTES; };
  auto stage_b = [&](int s) { return ring + s * C::STAGE_BYTES + C::A_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(tfull, 1);
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, BN);
    ptx::tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // barriers initialised, tensor memory allocated, cluster-wide
  ptx::tc_fence_after();
  ptx::griddep_wait();  // the previous kernel's outputs are visible from here on
  ptx::griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const long long tile_id = blockIdx.x / (2 * S);
  const auto tile = pol.tile(tile_id);
  const int nk = pol.num_k();
  const int kb0 = (int)((long long)p * nk / S), kb1 = (int)((long long)(p + 1) * nk / S);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!ptx::mbar_wait(&empty[stage], phase ^ 1, status, 0x311, abort_flag)) break;
        if (h == 0) ptx::mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
        const uint32_t lbar = ptx::mapa(ptx::smem_u32(&full[stage]), leader);
        pol.load(&tmap_a, &tmap_b, stage_a(stage), stage_b(stage), lbar, tile, kb, h);
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (h == 0) {
        // the leader's full barriers count both CTAs' bytes: no copy of the
        // pair may still be in flight when the ring is reused below
        for (int s = 0; s < STAGES && s < issued; ++s) {
          const int round = (issued - 1 - s) / STAGES;
          ptx::mbar_wait(&full[s], (uint32_t)(round & 1), status, 0x317, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && h == 0) {
      constexpr uint32_t idesc = ptx::make_idesc_tf32(2 * BM, C::MMA_N, P::A_MN, P::B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!ptx::mbar_wait(&full[stage], phase, status, 0x313, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t a_addr = ptx::smem_u32(stage_a(stage));
        const uint32_t b_addr = ptx::smem_u32(stage_b(stage));
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint32_t a_off = P::A_MN ? kk * 1024 : kk * 32;
          const uint32_t b_off = P::B_MN ? kk * 1024 : kk * 32;
          ptx::mma_tf32_ss_pair(tmem_base, operand_desc<P::A_MN>(a_addr + a_off),
                                operand_desc<P::B_MN>(b_addr + b_off), idesc,
                                (kb > kb0 || kk > 0) ? 1u : 0u);
        }
        ptx::mma_commit_pair(&empty[stage], mask);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (ok) ptx::mma_commit_pair(tfull, mask);
      ptx::mma_commit_pair(drain, mask);
      ptx::mbar_wait(drain, 0, status, 0x314, nullptr);
    }
  } else {
    // drain this CTA's 128 accumulator rows into the partial tile
    const int q = warp & 3;
    const int row = q * 32 + lane;
    if (__all_sync(0xffffffffu, ptx::mbar_wait(tfull, 0, status, 0x315, abort_flag))) {
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        ptx::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + c * 32, v);
        ptx::tmem_wait_ld();
        float4* dst = reinterpret_cast<float4*>(part + row * PITCH + c * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                               __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
      }
    }
  }

  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // every partial is in shared memory

  // reduce rows [p*ROWS, (p+1)*ROWS) of half h over the S pairs, in pair order
  // (after an expired wait the sums are of stale data; the status word says so)
  {
    constexpr int V4 = BN / 4;
    const uint32_t base = ptx::smem_u32(part);
    float* Cb = pol.C + (long long)tile.b * pol.c_batch;
    uint32_t src[S];  // the S partials of half h: cluster ranks h, 2 + h, ...
#pragma unroll
    for (int pp = 0; pp < S; ++pp) src[pp] = ptx::mapa(base, (uint32_t)(2 * pp + h));
    // U rows-chunks per thread per batch, all S*U loads issued before any use
    constexpr int U = 4, TOTAL = ROWS * V4;
    for (int f0 = threadIdx.x; f0 < TOTAL; f0 += U * C::THREADS) {
      float4 t[U][S];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int f = f0 + u * C::THREADS;
        if (f < TOTAL) {
          const int r = p * ROWS + f / V4, c4 = f % V4;
          const uint32_t off = (uint32_t)(r * PITCH + c4 * 4) * 4u;
#pragma unroll
          for (int pp = 0; pp < S; ++pp) t[u][pp] = ld_dsmem_v4(src[pp] + off);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int f = f0 + u * C::THREADS;
        if (f >= TOTAL) break;
        const int r = p * ROWS + f / V4, c4 = f % V4;
        float4 acc = t[u][0];
#pragma unroll
        for (int pp = 1; pp < S; ++pp) {
          acc.x += t[u][pp].x; acc.y += t[u][pp].y; acc.z += t[u][pp].z; acc.w += t[u][pp].w;
        }
        const int grow = tile.m0 + h * BM + r, col = tile.n0 + c4 * 4;
        if (grow < pol.M && col < pol.N) {
          const long long o = (long long)grow * pol.N + col;
          if (pol.bias) {
            const float4 bb = __ldg(reinterpret_cast<const float4*>(pol.bias + col));
            acc.x += bb.x; acc.y += bb.y; acc.z += bb.z; acc.w += bb.w;
          }
          if (pol.resid) {
            const float4 rr = __ldg(reinterpret_cast<const float4*>(
                pol.resid + (long long)tile.b * pol.c_batch + o));
            acc.x += rr.x; acc.y += rr.y; acc.z += rr.z; acc.w += rr.w;
          }
          if (pol.act) {
            acc.x = splitk_act(acc.x, pol.act); acc.y = splitk_act(acc.y, pol.act);
            acc.z = splitk_act(acc.z, pol.act); acc.w = splitk_act(acc.w, pol.act);
          }
          *reinterpret_cast<float4*>(Cb + o) = acc;
        }
      }
    }
  }
  cluster_sync_relaxed();  // no CTA leaves while another reads its shared memory
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, BN);
  }
}

}  // namespace umma
}  // namespace agpu
