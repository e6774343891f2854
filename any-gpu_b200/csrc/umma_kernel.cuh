// K segments: in 3xTF32 mode a tile's K loop is split into segments of
// kSegX3 K-blocks, each accumulated in its own TMEM buffer and summed by the
// epilogue in fp32, which bounds the number of MMAs accumulated into one
// tensor-memory accumulator (its rounding error grows with that count).
// All segments of a tile run on the same CTA, in order, so the epilogue's
// read-modify-write of the output needs no synchronisation.
//
// Warp-specialised tcgen05 (kind::tf32) mainloop shared by the contraction
// kernels (GEMM, implicit-GEMM conv2d).  A Policy supplies what differs:
// the tile scheduler, the TMA loads of one K-block, and the epilogue store.
//
//   warp 0      : TMA producer (one lane) into a STAGES-deep smem ring
//   warp 1      : TMEM owner; one lane issues tcgen05.mma (BK/8 per K-block)
//                 into a double-buffered 128 x BN fp32 accumulator
//   warps 2..5  : epilogue; warp w drains TMEM lanes 32*(w%4)..+31
//                 (tcgen05.ld 32x32b.x32) and hands each thread its row's 32
//                 consecutive accumulator columns to Policy::store
//   warps 6..7  : (3xTF32 only) split each staged tile into hi / lo parts
//
// Operand tiles are 128 (M) x BK and BN (N) x BK fp32, K-major with the
// 128-byte swizzle (rows of 32 fp32) or MN-major with the 128-byte/32-byte-
// atom swizzle (32-element chunks of BK rows).  Every mbarrier wait is
// bounded (ptx::mbar_wait); on expiry the kernel records a status code,
// drains its in-flight copies and MMAs, frees tensor memory and exits.
#pragma once

#include <cuda.h>

#include "ptx.cuh"

namespace agpu {
namespace umma {

constexpr int BM = 128;
constexpr int BK = 32;          // fp32 elements per 128-byte swizzle row
constexpr int kEpiWarps = 4;
constexpr int kEpiStride = 36;  // floats per epilogue staging row (conflict-free float4)
// Epilogue staging per warp: two 32 x 32 fp32 buffers (4 KB each, 1024-byte
// aligned) for the TMA-store epilogue; the transposing store uses the first
// 32 x kEpiStride floats.
constexpr int kEpiWarpFloats = 2048;
constexpr int kSegX3 = 16;      // K-blocks per accumulator segment in 3xTF32 mode

template <int BN_, bool X3>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_BYTES = kEpiWarps * kEpiWarpFloats * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int BUDGET = 227 * 1024 - 1024 - EPI_BYTES - BAR_BYTES;
  static constexpr int STAGES_RAW = BUDGET / (STAGE_BYTES * (X3 ? 2 : 1));
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static_assert(STAGES >= 2, "tile too large for the shared-memory ring");
  static constexpr int RING_BYTES = STAGE_BYTES * STAGES * (X3 ? 2 : 1);
  static constexpr int SMEM = 1024 + RING_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                  : (2 * BN <= 256) ? 256 : 512;
  static constexpr int THREADS = 192 + (X3 ? 64 : 0);
};

// Descriptor of one MMA K-slice (8 fp32) of an operand tile; see the header.
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t saddr) {
  return MN ? ptx::make_sdesc(saddr, BK * 128, 512, 1) : ptx::make_sdesc(saddr, 16, 1024, 2);
}

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

// Policy requirements (all __device__ const members):
//   static constexpr int BN; static constexpr bool A_MN, B_MN;
//   long long num_tiles() const;   int num_k() const;
//   struct Tile;  Tile tile(long long t) const;
//   void load(const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* sa, uint8_t* sb,
//             uint64_t* bar, const Tile&, int kb) const;       // issues STAGE_BYTES of TMA
//   void store(const Tile&, int row, int col0, const uint32_t (&v)[32], float* stg,
//              int lane, bool accumulate, bool last) const;
//                                 // row = accumulator lane 0..127, cols col0..col0+31;
//                                 // called by all 32 lanes of a warp together;
//                                 // accumulate: add to the value stored for the
//                                 // previous K segment of this tile; last:
//                                 // this is the tile's final K segment
//   bool col_live(const Tile&, int col0) const;  // warp-uniform: chunk has any valid column
template <class P, bool X3>
__global__ void __launch_bounds__(Cfg<P::BN, X3>::THREADS, 1)
    umma_tf32_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ P pol,
                     unsigned int* status) {
  using C = Cfg<P::BN, X3>;
  constexpr int BN = P::BN;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* epi = reinterpret_cast<float*>(smem + C::RING_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES + C::EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* conv = bars + 2 * STAGES;
  uint64_t* tfull = bars + 3 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  auto stage_a = [&](int s) { return ring + s * C::STAGE_BYTES; };
  auto stage_b = [&](int s) { return ring + s * C::STAGE_BYTES + C::A_BYTES; };
  auto lo_a = [&](int s) { return ring + (STAGES + s) * C::STAGE_BYTES; };
  auto lo_b = [&](int s) { return ring + (STAGES + s) * C::STAGE_BYTES + C::A_BYTES; };

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
    ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  ptx::griddep_wait();  // the previous kernel's outputs are visible from here on
  ptx::griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const int num_k = pol.num_k();
  const long long num_tiles = pol.num_tiles();
  const int kseg = X3 ? kSegX3 : (num_k > 0 ? num_k : 1);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      long long issued = 0;
      for (long long t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const auto tile = pol.tile(t);
        for (int kb = 0; kb < num_k; ++kb) {  // segments are consecutive K ranges
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, status, 0x101, abort_flag)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          pol.load(&tmap_a, &tmap_b, stage_a(stage), stage_b(stage), &full[stage], tile, kb);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Never leave while TMA writes into this CTA's shared memory are in
      // flight: wait (bounded) for the last load issued into each stage.
      for (int s = 0; s < STAGES && s < issued; ++s) {
        const long long round = (issued - 1 - s) / STAGES;
        ptx::mbar_wait(&full[s], (uint32_t)(round & 1), status, 0x107, nullptr);
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = ptx::make_idesc_tf32(BM, BN, P::A_MN, P::B_MN);
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (long long t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        for (int k0 = 0; k0 < num_k && ok; k0 += kseg, ++local) {
          const int k1 = min(num_k, k0 + kseg);
          const int acc = local & 1;
          const uint32_t acc_phase = (local >> 1) & 1;
          if (!ptx::mbar_wait(&tempty[acc], acc_phase ^ 1, status, 0x102, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          for (int kb = k0; kb < k1; ++kb) {
            uint64_t* ready = X3 ? &conv[stage] : &full[stage];
            if (!ptx::mbar_wait(ready, phase, status, 0x103, abort_flag)) { ok = false; break; }
            ptx::tc_fence_after();
            const uint32_t a_addr = ptx::smem_u32(stage_a(stage));
            const uint32_t b_addr = ptx::smem_u32(stage_b(stage));
            const uint32_t la_addr = ptx::smem_u32(lo_a(stage));
            const uint32_t lb_addr = ptx::smem_u32(lo_b(stage));
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk) {
              const uint32_t a_off = P::A_MN ? kk * 1024 : kk * 32;
              const uint32_t b_off = P::B_MN ? kk * 1024 : kk * 32;
              const uint64_t ad = operand_desc<P::A_MN>(a_addr + a_off);
              const uint64_t bd = operand_desc<P::B_MN>(b_addr + b_off);
              ptx::mma_tf32_ss(d_tmem, ad, bd, idesc, (kb > k0 || kk > 0) ? 1u : 0u);
              if (X3) {
                ptx::mma_tf32_ss(d_tmem, ad, operand_desc<P::B_MN>(lb_addr + b_off), idesc, 1u);
                ptx::mma_tf32_ss(d_tmem, operand_desc<P::A_MN>(la_addr + a_off), bd, idesc, 1u);
              }
            }
            ptx::mma_commit(&empty[stage]);
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          ptx::mma_commit(&tfull[acc]);
        }
      }
      ptx::mma_commit(drain);
      ptx::mbar_wait(drain, 0, status, 0x104, nullptr);
    }
  } else if (warp < 2 + kEpiWarps) {
    const int q = warp & 3;  // TMEM sub-partition this warp may access
    float* stg = epi + (warp - 2) * kEpiWarpFloats;
    int local = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const auto tile = pol.tile(t);
      for (int k0 = 0; k0 < num_k; k0 += kseg, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        // warp-uniform exit: the policy's store uses warp-wide syncs
        if (!__all_sync(0xffffffffu,
                        ptx::mbar_wait(&tfull[acc], acc_phase, status, 0x105, abort_flag))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          if (!pol.col_live(tile, c * 32)) break;  // warp-uniform
          uint32_t v[32];
          ptx::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + c * 32, v);
          ptx::tmem_wait_ld();
          pol.store(tile, q * 32 + lane, c * 32, v, stg, lane, k0 > 0, k0 + kseg >= num_k);
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(&tempty[acc]);
      }
    }
  } else if (X3) {
    const int ctid = threadIdx.x - (2 + kEpiWarps) * 32;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < num_k; ++kb) {
        if (!ptx::mbar_wait(&full[stage], phase, status, 0x106, abort_flag)) { ok = false; break; }
        split_tf32(reinterpret_cast<uint32_t*>(stage_a(stage)),
                   reinterpret_cast<uint32_t*>(lo_a(stage)), C::STAGE_BYTES / 4, ctid, 64);
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&conv[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  }

  // the epilogue's bulk (TMA) stores of C are complete before the CTA exits
  if (warp >= 2 && lane == 0) ptx::bulk_wait0();
  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace umma
}  // namespace agpu
