// Fused scaled-dot-product attention on sm_100a (flash-style, fp32 I/O,
// tcgen05 kind::tf32 with fp32 accumulation).
//
// Replaces the reference's unfused composition (src/ops/attention.rs:149-169):
// transpose(K) -> batch_matmul(Q, K^T) -> scale(1/sqrt(d)) -> softmax ->
// batch_matmul(P, V), which writes and re-reads the [BH, S, S] scores three
// times.  Same result, no scores in HBM:
//
//   Persistent: one CTA per SM walks tiles t = (128-row query tile, head,
//   batch), query tile fastest; 448 threads in four roles.
//   warps 10-13  Q loaders (thread = query row): the tile's Q row times
//              scale*log2(e), rounded to tf32, into one of two Q buffers in
//              tensor memory, so S = Q K^T takes its A operand from TMEM and
//              shared memory only carries K and V -- with fp32 operands the
//              per-SM shared-memory bandwidth, not the tensor core, is the
//              scarce resource.  The next tile's Q loads during this one.
//   warp 0     TMA: K_j and V_j blocks of 64 keys of every tile, in order,
//              through one 3-4 deep ring (V with the 32-byte-atom swizzle: it
//              is the MN-major B operand of P V).
//   warp 1     one lane issues the MMAs over the CTA's whole block sequence:
//                S_j  = Q K_j^T   (M 128, N 64, K = d), A = Q from TMEM -> S[j%2]
//                O   += P_j V_j   (M 128, N = d, K 64), A = P_j from TMEM
//              S of the next block -- the next tile's first one included --
//              is issued before P V of the current block, so the tensor core
//              has work while the softmax runs and across tile boundaries.
//   warps 2-9  softmax, two warps per 32 query rows (each takes half of a
//              block's 64 columns and half of O's head dims): read scores
//              (already base 2) from TMEM, online softmax, write P_j back over
//              S_j; O is rescaled only when the row max grows by more than
//              2^8 since the last rescale (exp2 never exceeds 256, most blocks
//              skip it).  At the end of a tile O / l goes to HBM and the
//              accumulator is handed back to the MMA warp.
// Shapes outside the tensor-core path (head dim not 64/128, unaligned
// pitches) use a warp-per-query SIMT kernel with the same online softmax.
#include <algorithm>
#include <cstdlib>

#include "agpu_internal.cuh"
#include "ptx.cuh"
#include "umma_kernel.cuh"

namespace agpu {

namespace {

constexpr int QT = 128;     // query rows per CTA
constexpr int KT = 64;      // keys per block
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;
constexpr int kAttnThreads = 64 + 256 + 128;  // TMA, MMA, 8 softmax, 4 Q-loader warps

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Round a finite non-negative float to tf32, nearest with ties to even (the
// tensor core would otherwise truncate P).
__device__ __forceinline__ uint32_t round_tf32(float x) {
  uint32_t u = __float_as_uint(x);
  u += 0xFFFu + ((u >> 13) & 1u);
  return u & 0xFFFFE000u;
}

// Output strides (elements) and which input maps order heads before sequence.
struct AttnOut {
  long long s, h, b;
  int hs;  // bit 1: k, bit 2: v
};

// Q is read by the softmax threads themselves (one row each) and parked in
// tensor memory, so it is passed as a pointer with (seq, head, batch) strides.
struct AttnQ {
  const float* p;
  long long s, h, b;
};

template <int D>
struct AttnCfg {
  static constexpr int K_BYTES = KT * D * 4;
  static constexpr int V_BYTES = KT * D * 4;
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int STAGES_RAW = (220 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 4 ? 4 : STAGES_RAW;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES + 768 * 4;
  static constexpr int S_COL = 0;           // S/P buffers: columns [0, 2*KT)
  static constexpr int O_COL = 2 * KT;      // O: columns [2*KT, 2*KT + D)
  static constexpr int Q_COL = 2 * KT + D;  // Q[2] (pre-scaled, tf32): 2 x D columns
  static constexpr int TMEM_COLS = (2 * KT + 3 * D <= 256) ? 256 : 512;
  static_assert(2 * KT + 3 * D <= 512, "tensor memory budget");
};

// Work split of the persistent grid: tile t = (query tile, head, batch) with
// the query tile fastest, so the CTAs working at one time share K and V in L2.
// Causal tiles go longest first (their key-block counts differ).
struct AttnTiles {
  int nqt, H, rows;  // query tiles per head, heads, query rows per tile
  long long total;
  __device__ void get(long long t, bool causal, int& q0, int& head, int& bat) const {
    int qt = (int)(t % nqt);
    if (causal) qt = nqt - 1 - qt;
    const long long r = t / nqt;
    q0 = qt * rows;
    head = (int)(r % H);
    bat = (int)(r / H);
  }
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_tf32_kernel(const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, AttnQ qin,
                          float* __restrict__ out, int S, float scale_log2, AttnOut ol,
                          AttnTiles tiles, unsigned int* status) {
  using C = AttnCfg<D>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + STAGES * C::STAGE_BYTES);
  uint64_t* k_full = bars;                   // [STAGES]
  uint64_t* v_full = k_full + STAGES;        // [STAGES]
  uint64_t* kv_empty = v_full + STAGES;      // [STAGES]
  uint64_t* s_full = kv_empty + STAGES;      // [2]
  uint64_t* p_full = s_full + 2;             // [2]
  uint64_t* q_full = p_full + 2;             // [2] Q buffer loaded
  uint64_t* q_empty = q_full + 2;            // [2] every S MMA reading it done
  uint64_t* o_done = q_empty + 2;            // [1] one phase per P V
  uint64_t* o_full = o_done + 1;             // [1] one phase per tile: its last P V done
  uint64_t* o_free = o_full + 1;             // [1] one phase per drained tile
  uint64_t* drain = o_free + 1;              // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xmax = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES + C::BAR_BYTES);
  float* lsum = xmax + 512;  // xmax [2 parity][2 half][128 rows], lsum [2 half][128 rows]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // 4-D maps {d, s, h, b}, or {d, h, s, b} when the head stride is the smaller
  // one (e.g. [batch, seq, heads, d] activations); the box is rows x 32 dims.
  auto load = [&](void* dst, const CUtensorMap* m, uint64_t* bar, int d0, int s0, int head,
                  int bat, bool hs) {
    if (hs) ptx::tma_load_4d(dst, m, bar, d0, head, s0, bat);
    else ptx::tma_load_4d(dst, m, bar, d0, s0, head, bat);
  };
  const int nb_all = (S + KT - 1) / KT;
  auto blocks = [&](int q0) { return CAUSAL ? min(nb_all, (q0 + QT - 1) / KT + 1) : nb_all; };
  auto stage_k = [&](int s) { return ring + s * C::STAGE_BYTES; };
  auto stage_v = [&](int s) { return ring + s * C::STAGE_BYTES + C::K_BYTES; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      ptx::mbar_init(&k_full[i], 1);
      ptx::mbar_init(&v_full[i], 1);
      ptx::mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&s_full[i], 1);
      ptx::mbar_init(&p_full[i], 256);
      ptx::mbar_init(&q_full[i], 128);
      ptx::mbar_init(&q_empty[i], 1);
    }
    ptx::mbar_init(o_done, 1);
    ptx::mbar_init(o_full, 1);
    ptx::mbar_init(o_free, 256);
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA --
    // K_j, V_j of every tile of this CTA, in order, through one ring.
    if (lane == 0) {
      long long g = 0;
      bool ok = true;
      for (long long t = blockIdx.x; t < tiles.total && ok; t += gridDim.x) {
        int q0, head, bat;
        tiles.get(t, CAUSAL, q0, head, bat);
        const int nb = blocks(q0);
        for (int j = 0; j < nb; ++j, ++g) {
          const int st = (int)(g % STAGES);
          const uint32_t par = (uint32_t)(((g / STAGES) & 1) ^ 1);
          if (!ptx::mbar_wait(&kv_empty[st], par, status, 0x201, abort_flag)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(&k_full[st], C::K_BYTES);
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            load(stage_k(st) + c * KT * 128, &tm_k, &k_full[st], c * 32, j * KT, head, bat,
                 ol.hs & 2);
          ptx::mbar_arrive_expect_tx(&v_full[st], C::V_BYTES);
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            load(stage_v(st) + c * KT * 128, &tm_v, &v_full[st], c * 32, j * KT, head, bat,
                 ol.hs & 4);
        }
      }
      // never exit with loads in flight into this CTA's shared memory
      for (long long i = std::max<long long>(0, g - STAGES); i < g; ++i) {
        const uint32_t par = (uint32_t)((i / STAGES) & 1);
        ptx::mbar_wait(&k_full[i % STAGES], par, status, 0x207, nullptr);
        ptx::mbar_wait(&v_full[i % STAGES], par, status, 0x207, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA --
    // Blocks of consecutive tiles form one sequence: S of the next block
    // (possibly the next tile's first) is issued before P V of the current
    // one, so the tensor core has work across tile boundaries.
    if (lane == 0) {
      constexpr uint32_t idesc_s = ptx::make_idesc_tf32(QT, KT, false, false);
      constexpr uint32_t idesc_o = ptx::make_idesc_tf32(QT, D, false, true);
      bool ok = true;
      // S of global block g (tile-local block j of local tile i) with Q buffer qb
      auto issue_s = [&](long long g, int j, int i) -> bool {
        const int qb = i & 1;
        if (j == 0) {
          if (!ptx::mbar_wait(&q_full[qb], (i >> 1) & 1, status, 0x20b, abort_flag))
            return false;
        }
        const int st = (int)(g % STAGES);
        if (!ptx::mbar_wait(&k_full[st], (uint32_t)((g / STAGES) & 1), status, 0x203,
                            abort_flag))
          return false;
        ptx::tc_fence_after();
        const uint32_t k_addr = ptx::smem_u32(stage_k(st));
        const uint32_t d_tmem = tmem + C::S_COL + (uint32_t)(g & 1) * KT;
        const uint32_t q_tmem = tmem + C::Q_COL + qb * D;
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
          const uint32_t off = (kk % 4) * 32;  // 8 fp32 inside the 128-byte row
          const uint64_t bd = umma::operand_desc<false>(k_addr + (kk / 4) * KT * 128 + off);
          ptx::mma_tf32_ts(d_tmem, q_tmem + kk * 8, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&s_full[g & 1]);
        return true;
      };
      // the block sequence: (tile t, local tile i, block j) with global index g
      long long t = blockIdx.x, g = 0;
      int i = 0;
      if (t < tiles.total) {
        int q0, head, bat;
        tiles.get(t, CAUSAL, q0, head, bat);
        int nb = blocks(q0);
        ok = issue_s(0, 0, 0);
        int j = 0;
        while (ok) {
          // the block after (t, j)
          long long tn = t;
          int jn = j + 1, in = i, nbn = nb;
          if (jn == nb) {
            tn = t + gridDim.x;
            jn = 0;
            in = i + 1;
            if (tn < tiles.total) {
              int q0n, hn, bn;
              tiles.get(tn, CAUSAL, q0n, hn, bn);
              nbn = blocks(q0n);
            }
            ptx::mma_commit(&q_empty[i & 1]);  // this tile's S MMAs are all issued
          }
          if (tn < tiles.total && !issue_s(g + 1, jn, in)) { ok = false; break; }
          const int st = (int)(g % STAGES);
          if (!ptx::mbar_wait(&p_full[g & 1], (uint32_t)((g >> 1) & 1), status, 0x204,
                              abort_flag)) { ok = false; break; }
          if (!ptx::mbar_wait(&v_full[st], (uint32_t)((g / STAGES) & 1), status, 0x205,
                              abort_flag)) { ok = false; break; }
          if (j == 0 && i > 0 &&
              !ptx::mbar_wait(o_free, (uint32_t)((i - 1) & 1), status, 0x20c, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t v_addr = ptx::smem_u32(stage_v(st));
          const uint32_t p_tmem = tmem + C::S_COL + (uint32_t)(g & 1) * KT;
#pragma unroll
          for (int kk = 0; kk < KT / 8; ++kk) {
            // V chunk c (32 head dims x 64 keys, 8 KB) at c * KT * 128; 8 keys = 1024 B
            const uint64_t bd = ptx::make_sdesc(v_addr + kk * 1024, KT * 128, 512, 1);
            ptx::mma_tf32_ts(tmem + C::O_COL, p_tmem + kk * 8, bd, idesc_o,
                             (j > 0 || kk > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&kv_empty[st]);
          ptx::mma_commit(o_done);
          if (jn == 0) ptx::mma_commit(o_full);  // the tile's last P V
          ++g;
          if (tn >= tiles.total) break;
          t = tn; j = jn; i = in; nb = nbn;
        }
      }
      ptx::mma_commit(drain);
      ptx::mbar_wait(drain, 0, status, 0x206, nullptr);
    }
  } else if (warp >= 10) {
    // -------------------------------------------------------- Q loaders --
    // Thread = query row: the row of Q times scale * log2(e) (scores come out
    // in base 2), rounded to tf32 (nearest, ties to even), into tensor memory
    // buffer i & 1 -- the A operand of every S = Q K^T of local tile i.
    const int qd = warp & 3;
    const int row = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    int i = 0;
    for (long long t = blockIdx.x; t < tiles.total; t += gridDim.x, ++i) {
      int q0, head, bat;
      tiles.get(t, CAUSAL, q0, head, bat);
      const int qb = i & 1;
      if (!__all_sync(0xffffffffu, ptx::mbar_wait(&q_empty[qb], (uint32_t)(((i >> 1) & 1) ^ 1),
                                                  status, 0x20d, abort_flag)))
        break;
      const int qrow = q0 + row;
      const float* qr = qin.p + (long long)bat * qin.b + (long long)head * qin.h +
                        (long long)qrow * qin.s;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
          if (qrow < S) f = __ldg(reinterpret_cast<const float4*>(qr + c * 32) + k);
          r[4 * k] = round_tf32(f.x * scale_log2);
          r[4 * k + 1] = round_tf32(f.y * scale_log2);
          r[4 * k + 2] = round_tf32(f.z * scale_log2);
          r[4 * k + 3] = round_tf32(f.w * scale_log2);
        }
        ptx::tmem_st32(tmem + lane_off + C::Q_COL + qb * D + c * 32, r);
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&q_full[qb]);
    }
  } else {
    // ------------------------------------------------------ softmax rows --
    // Warps w and w+4 share the 32 query rows of TMEM lane group w & 3 and
    // split every block's 64 columns (and O's head dims) in halves; they
    // exchange their half-row maxima through shared memory behind a
    // 64-thread named barrier, and keep separate row sums until the tile ends.
    // Every block runs that barrier, even after a failed wait (then with the
    // work skipped), so the two warps never fall out of step; `ok` is kept
    // warp-uniform for the .sync.aligned tensor-memory accesses.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;             // column half
    const int row = q * 32 + lane;            // accumulator lane = query row in tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    constexpr int HK = KT / 2, HD = D / 2;
    bool ok = true;
    long long g = 0;
    int tile_i = 0;
    for (long long t = blockIdx.x; t < tiles.total; t += gridDim.x, ++tile_i) {
      int q0, head, bat;
      tiles.get(t, CAUSAL, q0, head, bat);
      const int nb = blocks(q0);
      const int qrow = q0 + row;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nb; ++j, ++g) {
        const int sb = (int)(g & 1);
        if (ok) ok = __all_sync(0xffffffffu, ptx::mbar_wait(&s_full[sb], (uint32_t)((g >> 1) & 1),
                                                            status, 0x208, abort_flag));
        uint32_t sv[32];
        float tv[32];
        const uint32_t sbase = tmem + lane_off + C::S_COL + sb * KT + h * HK;
        float m = -INFINITY;
        if (ok) {
          ptx::tc_fence_after();
          ptx::tmem_ld32(sbase, sv);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) tv[k] = __uint_as_float(sv[k]);
          const int kv0 = j * KT + h * HK;
          if (kv0 + HK > S || (CAUSAL && kv0 + HK - 1 > q0)) {
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const int kv = kv0 + k;
              if (kv >= S || (CAUSAL && kv > qrow)) tv[k] = -INFINITY;
            }
          }
          float mx[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mx[k] = fmaxf(fmaxf(tv[k], tv[k + 8]), fmaxf(tv[k + 16], tv[k + 24]));
#pragma unroll
          for (int k = 0; k < 4; ++k) mx[k] = fmaxf(mx[k], mx[k + 4]);
          m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        }
        float* xm = xmax + sb * 256;
        xm[h * 128 + row] = m;
        ptx::named_bar_sync(1 + q, 64);
        m = fmaxf(m, xm[(h ^ 1) * 128 + row]);
        // a failed wait in either warp of the pair raised the flag before the
        // barrier: both warps see it here
        if (*abort_flag) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          const bool need = m > m_used + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            const float m_new = need ? m : m_used;
            const float alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
            if (j > 0) {
              // O holds this tile's P V so far; wait for the last one, then
              // rescale this warp's half of the head dims in place.  The
              // parity wait is exact: S_g completing (waited above) implies
              // every P V before P V_{g-1} completed (the MMA warp issued S_g
              // after them), and P V_g cannot run before P_g exists.
              ok = __all_sync(0xffffffffu, ptx::mbar_wait(o_done, (uint32_t)((g - 1) & 1),
                                                          status, 0x209, abort_flag));
              if (ok) {
                ptx::tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                  uint32_t o[32];
                  const uint32_t oaddr = tmem + lane_off + C::O_COL + h * HD + c * 32;
                  ptx::tmem_ld32(oaddr, o);
                  ptx::tmem_wait_ld();
#pragma unroll
                  for (int k = 0; k < 32; ++k)
                    o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                  ptx::tmem_st32(oaddr, o);
                }
                ptx::tmem_wait_st();
              }
            }
            l *= alpha;
            m_used = m_new;
          }
        }
        if (ok) {
          // P is handed to the tensor core already truncated to tf32 and the
          // row sum l accumulates exactly those values, so the weights P / l
          // that multiply V sum to one: truncation leaves no bias in O.
          float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            sv[k] = __float_as_uint(ex2(tv[k] - m_used)) & 0xFFFFE000u;
            ls[k & 3] += __uint_as_float(sv[k]);
          }
          l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
          ptx::tmem_st32(sbase, sv);
          ptx::tmem_wait_st();
          ptx::tc_fence_before();
          ptx::mbar_arrive(&p_full[sb]);
        }
      }
      // combine the two halves' row sums, then drain this tile's O and hand
      // the accumulator back to the MMA warp
      lsum[h * 128 + row] = l;
      ptx::named_bar_sync(1 + q, 64);
      l += lsum[(h ^ 1) * 128 + row];
      // One o_full phase per tile, awaited once each, in order (the o_done
      // parity of the last P V could be passed while the one before it is
      // still running).
      if (ok) ok = __all_sync(0xffffffffu, ptx::mbar_wait(o_full, (uint32_t)(tile_i & 1),
                                                          status, 0x20a, abort_flag));
      if (ok) {
        ptx::tc_fence_after();
        const float inv = 1.0f / l;
        float* orow = out + (long long)bat * ol.b + (long long)head * ol.h +
                      (long long)qrow * ol.s + h * HD;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          ptx::tmem_ld32(tmem + lane_off + C::O_COL + h * HD + c * 32, o);
          ptx::tmem_wait_ld();
          if (qrow < S) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
              __stcs(reinterpret_cast<float4*>(orow + c * 32) + k,
                     make_float4(__uint_as_float(o[4 * k]) * inv,
                                 __uint_as_float(o[4 * k + 1]) * inv,
                                 __uint_as_float(o[4 * k + 2]) * inv,
                                 __uint_as_float(o[4 * k + 3]) * inv));
          }
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(o_free);
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------ CTA pair --
// Same algorithm on a pair of CTAs (a cluster of 2 on neighbouring SMs):
// tiles of 256 query rows (CTA r owns rows q0 + 128 r ..), blocks of KB = 128
// keys, every MMA issued by the leader as tcgen05.mma.cta_group::2 (M 256):
//   S  = Q K^T  N = 128 keys: CTA r stages keys 64 r .. +63 of the block;
//   O += P V    N = d:        CTA r stages head dims d/2 r .. of all 128 keys.
// So each CTA moves half of every K and V block (TMA bytes per FLOP halved)
// and S runs at N = 128, the tensor core's full-rate width (at N = 64 it
// reaches about two thirds).  Q and P stay in each CTA's tensor memory.
// Barriers counted by both CTAs live in the leader (loads signal its k_full/
// v_full; one lane per softmax warp arrives on its q_full, p_full, o_free,
// through a cluster address from the peer); the leader's commits multicast
// to both CTAs' kv_empty, s_full, q_empty, o_done and o_full.  320 threads:
// TMA warp, MMA warp, 8 softmax warps, which also write the next tile's Q
// into tensor memory as soon as the current tile's last S is consumed.
constexpr int KB = 128;  // keys per block (pair)
constexpr int kPairAttnThreads = 64 + 256;  // TMA, MMA, 8 softmax warps
constexpr int KH = 64;   // keys per CTA in S

template <int D>
struct PairAttnCfg {
  static constexpr int K_BYTES = KH * D * 4;        // this CTA's keys of K
  static constexpr int V_BYTES = KB * (D / 2) * 4;  // this CTA's head dims of V
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int STAGES_RAW = (200 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 4 ? 4 : STAGES_RAW;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES + 768 * 4;
  static constexpr int S_COL = 0;            // S/P buffers: [0, 2*KB)
  static constexpr int O_COL = 2 * KB;       // O: [2*KB, 2*KB + D)
  static constexpr int Q_COL = 2 * KB + D;   // Q: [2*KB + D, 2*KB + 2*D)
  static constexpr int TMEM_COLS = 512;
  static_assert(2 * KB + 2 * D <= 512, "tensor memory budget");
};

template <int D, bool CAUSAL, bool LSE>
__global__ void __launch_bounds__(kPairAttnThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, AttnQ qin,
                          float* __restrict__ out, int S, float scale_log2, AttnOut ol,
                          AttnTiles tiles, unsigned int* status, float* __restrict__ lse) {
  using C = PairAttnCfg<D>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + STAGES * C::STAGE_BYTES);
  uint64_t* k_full = bars;                   // [STAGES] leader: both CTAs' bytes
  uint64_t* v_full = k_full + STAGES;        // [STAGES] leader
  uint64_t* kv_empty = v_full + STAGES;      // [STAGES] both
  uint64_t* s_full = kv_empty + STAGES;      // [2] both
  uint64_t* p_full = s_full + 2;             // [2] leader: one arrive per softmax warp
  uint64_t* q_full = p_full + 2;             // [1] leader: one arrive per softmax warp
  uint64_t* q_empty = q_full + 1;            // [1] both
  uint64_t* o_done = q_empty + 1;            // [1] both: one phase per P V
  uint64_t* o_full = o_done + 1;             // [1] both: one phase per tile
  uint64_t* o_free = o_full + 1;             // [1] leader: one arrive per softmax warp
  uint64_t* drain = o_free + 1;              // [1] leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xmax = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES + C::BAR_BYTES);
  float* lsum = xmax + 512;  // xmax [2 parity][2 half][128 rows], lsum [2 half][128 rows]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int rank = (int)ptx::cluster_rank();
  const bool leader = rank == 0;
  const long long cluster_id = blockIdx.x / 2, n_clusters = gridDim.x / 2;
  auto lead = [&](uint64_t* bar) { return ptx::mapa(ptx::smem_u32(bar), 0); };
  // One arrive per warp on a leader barrier, after every lane's prior work.
  // Everything these barriers hand over (Q, P, the drained O) is tensor
  // memory, ordered by tcgen05.wait + the tcgen05 fence pair, so the peer's
  // remote arrive keeps the default CTA-scope release (a cluster-scope
  // release cost ~1.4k cycles per warp and key block).
  auto warp_arrive = [&](uint64_t* bar) {
    __syncwarp();
    if (lane == 0) {
      if (leader) ptx::mbar_arrive(bar);
      else ptx::mbar_arrive_remote(lead(bar));
    }
  };
  auto load = [&](void* dst, const CUtensorMap* m, uint32_t bar, int d0, int s0, int head,
                  int bat, bool hs) {
    if (hs) ptx::tma_load_4d_pair(dst, m, bar, d0, head, s0, bat);
    else ptx::tma_load_4d_pair(dst, m, bar, d0, s0, head, bat);
  };
  const int nb_all = (S + KB - 1) / KB;
  auto blocks = [&](int q0) {
    return CAUSAL ? min(nb_all, (q0 + 2 * QT - 1) / KB + 1) : nb_all;
  };
  auto stage_k = [&](int s) { return ring + s * C::STAGE_BYTES; };
  auto stage_v = [&](int s) { return ring + s * C::STAGE_BYTES + C::K_BYTES; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      ptx::mbar_init(&k_full[i], 1);
      ptx::mbar_init(&v_full[i], 1);
      ptx::mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&s_full[i], 1);
      ptx::mbar_init(&p_full[i], 16);  // 8 softmax warps per CTA
    }
    ptx::mbar_init(q_full, 16);      // 8 softmax warps per CTA write Q
    ptx::mbar_init(q_empty, 1);
    ptx::mbar_init(o_done, 1);
    ptx::mbar_init(o_full, 1);
    ptx::mbar_init(o_free, 16);
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // peer barriers initialised, tensor memory allocated
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA --
    if (lane == 0) {
      long long g = 0;
      bool ok = true;
      for (long long t = cluster_id; t < tiles.total && ok; t += n_clusters) {
        int q0, head, bat;
        tiles.get(t, CAUSAL, q0, head, bat);
        const int nb = blocks(q0);
        for (int j = 0; j < nb; ++j, ++g) {
          const int st = (int)(g % STAGES);
          const uint32_t par = (uint32_t)(((g / STAGES) & 1) ^ 1);
          if (!ptx::mbar_wait(&kv_empty[st], par, status, 0x221, abort_flag)) { ok = false; break; }
          if (leader) {
            ptx::mbar_arrive_expect_tx(&k_full[st], 2 * C::K_BYTES);
            ptx::mbar_arrive_expect_tx(&v_full[st], 2 * C::V_BYTES);
          }
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            load(stage_k(st) + c * KH * 128, &tm_k, lead(&k_full[st]), c * 32,
                 j * KB + rank * KH, head, bat, ol.hs & 2);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            load(stage_v(st) + c * KB * 128, &tm_v, lead(&v_full[st]), rank * (D / 2) + c * 32,
                 j * KB, head, bat, ol.hs & 4);
        }
      }
      if (leader) {
        // the leader's full barriers count both CTAs' bytes: wait (bounded)
        // for the last round of each stage so no copy of the pair is in flight
        for (long long i = std::max<long long>(0, g - STAGES); i < g; ++i) {
          const uint32_t par = (uint32_t)((i / STAGES) & 1);
          ptx::mbar_wait(&k_full[i % STAGES], par, status, 0x227, nullptr);
          ptx::mbar_wait(&v_full[i % STAGES], par, status, 0x227, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA --
    if (lane == 0 && leader) {
      constexpr uint32_t idesc_s = ptx::make_idesc_tf32(2 * QT, KB, false, false);
      constexpr uint32_t idesc_o = ptx::make_idesc_tf32(2 * QT, D, false, true);
      bool ok = true;
      int nb_cur = 0;  // blocks of the tile whose S is being issued
      auto issue_s = [&](long long g, int j, int i) -> bool {
        if (j == 0 &&
            !ptx::mbar_wait<true>(q_full, (uint32_t)(i & 1), status, 0x22b, abort_flag))
          return false;
        const int st = (int)(g % STAGES);
        if (!ptx::mbar_wait(&k_full[st], (uint32_t)((g / STAGES) & 1), status, 0x223,
                            abort_flag))
          return false;
        ptx::tc_fence_after();
        // one descriptor per block; a K-slice moves its 14-bit start address
        // (bytes / 16) by a compile-time offset, no carry (smem < 256 KB)
        const uint64_t bd0 = umma::operand_desc<false>(ptx::smem_u32(stage_k(st)));
        const uint32_t d_tmem = tmem + C::S_COL + (uint32_t)(g & 1) * KB;
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
          constexpr int kChunk = KH * 128;  // one 32-dim chunk of the K half
          const uint64_t bd = bd0 + (uint64_t)(((kk / 4) * kChunk + (kk % 4) * 32) >> 4);
          ptx::mma_tf32_ts_pair(d_tmem, tmem + C::Q_COL + kk * 8, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit_pair(&s_full[g & 1], 0x3);
        if (j == nb_cur - 1) ptx::mma_commit_pair(q_empty, 0x3);  // the tile's last S
        return true;
      };
      auto issue_pv = [&](long long g, int j, int i) -> bool {
        const int st = (int)(g % STAGES);
        if (!ptx::mbar_wait<true>(&p_full[g & 1], (uint32_t)((g >> 1) & 1), status, 0x224,
                                  abort_flag))
          return false;
        if (!ptx::mbar_wait(&v_full[st], (uint32_t)((g / STAGES) & 1), status, 0x225,
                            abort_flag))
          return false;
        if (j == 0 && i > 0 &&
            !ptx::mbar_wait<true>(o_free, (uint32_t)((i - 1) & 1), status, 0x22c, abort_flag))
          return false;
        ptx::tc_fence_after();
        // V chunk c (32 head dims x 128 keys, 16 KB) at c * KB * 128; 8 keys = 1024 B
        const uint64_t bd0 = ptx::make_sdesc(ptx::smem_u32(stage_v(st)), KB * 128, 512, 1);
        const uint32_t p_tmem = tmem + C::S_COL + (uint32_t)(g & 1) * KB;
        const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < KB / 8; ++kk)
          ptx::mma_tf32_ts_pair(tmem + C::O_COL, p_tmem + kk * 8, bd0 + (uint64_t)(kk * 64),
                                idesc_o, kk > 0 ? 1u : acc0);
        ptx::mma_commit_pair(&kv_empty[st], 0x3);
        ptx::mma_commit_pair(o_done, 0x3);
        return true;
      };
      long long t = cluster_id, g = 0;
      int i = 0;
      if (t < tiles.total) {
        int q0, head, bat;
        tiles.get(t, CAUSAL, q0, head, bat);
        int nb = blocks(q0);
        nb_cur = nb;
        ok = issue_s(0, 0, 0);
        int j = 0;
        while (ok) {
          if (j + 1 < nb) {
            // S of the next block first: it overlaps this block's softmax
            if (!issue_s(g + 1, j + 1, i) || !issue_pv(g, j, i)) { ok = false; break; }
            ++g;
            ++j;
            continue;
          }
          // last block of the tile: its P V, then the next tile's first S
          // (which waits for the next Q; Q was released after the last S)
          if (!issue_pv(g, j, i)) { ok = false; break; }
          ptx::mma_commit_pair(o_full, 0x3);
          ++g;
          t += n_clusters;
          if (t >= tiles.total) break;
          ++i;
          j = 0;
          tiles.get(t, CAUSAL, q0, head, bat);
          nb = blocks(q0);
          nb_cur = nb;
          if (!issue_s(g, 0, i)) { ok = false; break; }
        }
      }
      ptx::mma_commit_pair(drain, 0x1);
      ptx::mbar_wait(drain, 0, status, 0x226, nullptr);
    }
  } else {
    // ------------------------------------------------------ softmax rows --
    // As in the single-CTA kernel, with 64 of a block's 128 columns per
    // thread (two 32-column TMEM loads).
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;             // column half
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    constexpr int HC = KB / 2, HD = D / 2;
    bool ok = true;
    // This thread's half of its Q row for tile t (local tile i), times
    // scale * log2(e) (scores come out in base 2) and rounded to tf32, into
    // tensor memory -- once the previous tile's S MMAs are done with it.
    auto load_q = [&](long long t, int i) {
      if (ok) ok = __all_sync(0xffffffffu, ptx::mbar_wait(q_empty, (uint32_t)((i & 1) ^ 1),
                                                          status, 0x22d, abort_flag));
      if (!ok) return;
      int q0, head, bat;
      tiles.get(t, CAUSAL, q0, head, bat);
      // 16 rows x 32 columns per store in the 16x256b shape: four lanes
      // read 32 contiguous bytes of a row (a thread per row would touch 32
      // lines per load instruction)
      const int row0 = q0 + rank * QT + q * 32;
      const float* qh = qin.p + (long long)bat * qin.b + (long long)head * qin.h + h * HD +
                        2 * (lane & 3);
#pragma unroll 1
      for (int u = 0; u < 2; ++u) {
        const int r0 = row0 + 16 * u + (lane >> 2), r1 = r0 + 8;
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t r[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int col = c * 32 + 8 * j;
            float2 f0 = make_float2(0.f, 0.f), f1 = f0;
            if (r0 < S) f0 = __ldg(reinterpret_cast<const float2*>(qh + (long long)r0 * qin.s + col));
            if (r1 < S) f1 = __ldg(reinterpret_cast<const float2*>(qh + (long long)r1 * qin.s + col));
            r[4 * j] = round_tf32(f0.x * scale_log2);
            r[4 * j + 1] = round_tf32(f0.y * scale_log2);
            r[4 * j + 2] = round_tf32(f1.x * scale_log2);
            r[4 * j + 3] = round_tf32(f1.y * scale_log2);
          }
          ptx::tmem_st_16x256b_x4(
              tmem + ((uint32_t)(q * 32 + 16 * u) << 16) + C::Q_COL + h * HD + c * 32, r);
        }
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      warp_arrive(q_full);
    };
    long long g = 0;
    int tile_i = 0;
    if (cluster_id < tiles.total) load_q(cluster_id, 0);
    for (long long t = cluster_id; t < tiles.total; t += n_clusters, ++tile_i) {
      int q0, head, bat;
      tiles.get(t, CAUSAL, q0, head, bat);
      const int nb = blocks(q0);
      const int qrow = q0 + rank * QT + row;
      float m_used = -INFINITY, l = 0.f;
      [[maybe_unused]] float lx = 0.f;  // LSE: the sum of P before truncation
      for (int j = 0; j < nb; ++j, ++g) {
        const int sb = (int)(g & 1);
        if (ok) ok = __all_sync(0xffffffffu, ptx::mbar_wait(&s_full[sb], (uint32_t)((g >> 1) & 1),
                                                            status, 0x228, abort_flag));
        // the 64 scores, then in place the 64 P values (one register array)
        uint32_t v[64];
        uint32_t (&v0)[32] = *reinterpret_cast<uint32_t(*)[32]>(v);
        uint32_t (&v1)[32] = *reinterpret_cast<uint32_t(*)[32]>(v + 32);
        const uint32_t sbase = tmem + lane_off + C::S_COL + sb * KB + h * HC;
        float m = -INFINITY;
        if (ok) {
          ptx::tc_fence_after();
          ptx::tmem_ld32(sbase, v0);
          ptx::tmem_ld32(sbase + 32, v1);
          ptx::tmem_wait_ld();
          const int kv0 = j * KB + h * HC;
          if (kv0 + HC > S || (CAUSAL && kv0 + HC - 1 > q0 + rank * QT)) {
#pragma unroll
            for (int k = 0; k < 64; ++k) {
              const int kv = kv0 + k;
              if (kv >= S || (CAUSAL && kv > qrow)) v[k] = __float_as_uint(-INFINITY);
            }
          }
          float mx[8];
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mx[k] = fmaxf(fmaxf(fmaxf(__uint_as_float(v[k]), __uint_as_float(v[k + 8])),
                                fmaxf(__uint_as_float(v[k + 16]), __uint_as_float(v[k + 24]))),
                          fmaxf(fmaxf(__uint_as_float(v[k + 32]), __uint_as_float(v[k + 40])),
                                fmaxf(__uint_as_float(v[k + 48]), __uint_as_float(v[k + 56]))));
#pragma unroll
          for (int k = 0; k < 4; ++k) mx[k] = fmaxf(mx[k], mx[k + 4]);
          m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        }
        float* xm = xmax + sb * 256;
        xm[h * 128 + row] = m;
        ptx::named_bar_sync(1 + q, 64);
        m = fmaxf(m, xm[(h ^ 1) * 128 + row]);
        if (*abort_flag) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          const bool need = m > m_used + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            const float m_new = need ? m : m_used;
            const float alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
            if (j > 0) {
              // exact parity wait: S_g done implies every P V before P V_{g-1}
              // done (issued before S_g), and P V_g needs P_g
              ok = __all_sync(0xffffffffu, ptx::mbar_wait(o_done, (uint32_t)((g - 1) & 1),
                                                          status, 0x229, abort_flag));
              if (ok) {
                ptx::tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                  uint32_t o[32];
                  const uint32_t oaddr = tmem + lane_off + C::O_COL + h * HD + c * 32;
                  ptx::tmem_ld32(oaddr, o);
                  ptx::tmem_wait_ld();
#pragma unroll
                  for (int k = 0; k < 32; ++k)
                    o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                  ptx::tmem_st32(oaddr, o);
                }
                ptx::tmem_wait_st();
              }
            }
            l *= alpha;
            if constexpr (LSE) lx *= alpha;
            m_used = m_new;
          }
        }
        if (ok) {
          // P truncated to tf32 as the tensor core reads it; l sums exactly
          // those values, so P / l sums to one
          float ls[4] = {0.f, 0.f, 0.f, 0.f};
          if constexpr (LSE) {
            float lxs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < 64; ++k) {
              const float e = ex2(__uint_as_float(v[k]) - m_used);
              lxs[k & 3] += e;
              v[k] = __float_as_uint(e) & 0xFFFFE000u;
              ls[k & 3] += __uint_as_float(v[k]);
            }
            lx += (lxs[0] + lxs[1]) + (lxs[2] + lxs[3]);
          } else {
#pragma unroll
            for (int k = 0; k < 64; ++k) {
              v[k] = __float_as_uint(ex2(__uint_as_float(v[k]) - m_used)) & 0xFFFFE000u;
              ls[k & 3] += __uint_as_float(v[k]);
            }
          }
          l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
          ptx::tmem_st32(sbase, v0);
          ptx::tmem_st32(sbase + 32, v1);
          ptx::tmem_wait_st();
          ptx::tc_fence_before();
          warp_arrive(&p_full[sb]);
        }
      }
      // the next tile's Q (the MMA warp can start its S while O drains)
      if (t + n_clusters < tiles.total) load_q(t + n_clusters, tile_i + 1);
      lsum[h * 128 + row] = l;
      ptx::named_bar_sync(1 + q, 64);
      l += lsum[(h ^ 1) * 128 + row];
      if constexpr (LSE) {
        // the row's log-sum-exp of its base-2 scores (P = 2^(s - lse)), from
        // the untruncated sum; lsum is reused once the partner has read l
        ptx::named_bar_sync(1 + q, 64);
        lsum[h * 128 + row] = lx;
        ptx::named_bar_sync(1 + q, 64);
        lx += lsum[(h ^ 1) * 128 + row];
        if (h == 0 && qrow < S) lse[((long long)bat * tiles.H + head) * S + qrow] = m_used + log2f(lx);
      }
      if (ok) ok = __all_sync(0xffffffffu, ptx::mbar_wait(o_full, (uint32_t)(tile_i & 1),
                                                          status, 0x22a, abort_flag));
      if (ok) {
        ptx::tc_fence_after();
        const float inv = 1.0f / l;
        // 16 rows per pass in the 16x256b shape (whole 32-byte sectors per
        // store), each row scaled by its own 1 / l, fetched from the lane
        // that owns the row
        const int row0 = q0 + rank * QT + q * 32;
        float* oh = out + (long long)bat * ol.b + (long long)head * ol.h + h * HD + 2 * (lane & 3);
#pragma unroll 1
        for (int u = 0; u < 2; ++u) {
          const int src = 16 * u + (lane >> 2);
          const float i0 = __shfl_sync(0xffffffffu, inv, src);
          const float i1 = __shfl_sync(0xffffffffu, inv, src + 8);
          const int r0 = row0 + src, r1 = r0 + 8;
          uint32_t o[HD / 32][16];
#pragma unroll
          for (int c = 0; c < HD / 32; ++c)
            ptx::tmem_ld_16x256b_x4(
                tmem + ((uint32_t)(q * 32 + 16 * u) << 16) + C::O_COL + h * HD + c * 32, o[c]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int col = c * 32 + 8 * j;
              if (r0 < S)
                __stcs(reinterpret_cast<float2*>(oh + (long long)r0 * ol.s + col),
                       make_float2(__uint_as_float(o[c][4 * j]) * i0,
                                   __uint_as_float(o[c][4 * j + 1]) * i0));
              if (r1 < S)
                __stcs(reinterpret_cast<float2*>(oh + (long long)r1 * ol.s + col),
                       make_float2(__uint_as_float(o[c][4 * j + 2]) * i1,
                                   __uint_as_float(o[c][4 * j + 3]) * i1));
            }
          }
        }
        ptx::tc_fence_before();
        warp_arrive(o_free);
      }
    }
  }

  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // the pair's MMAs are retired before either CTA frees TMEM
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

// (seq, head, batch) element strides of Q, K, V, O.
struct AttnStrides {
  long long q[3], k[3], v[3], o[3];
};

// ----------------------------------------------------------------- SIMT --
// One warp per query row; keys streamed, online softmax, O in registers
// (lane owns head dims lane, lane+32, ...).  Exact fp32, any head dim <= 256.
template <bool CAUSAL>
__global__ void __launch_bounds__(256) attention_simt_kernel(const float* __restrict__ Q,
                                                             const float* __restrict__ K,
                                                             const float* __restrict__ V,
                                                             float* __restrict__ O, int B, int H,
                                                             int S, int D, float scale,
                                                             AttnStrides st) {
  const long long gw = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= (long long)B * H * S) return;
  const int i = (int)(gw % S);
  const int h = (int)((gw / S) % H);
  const int b = (int)(gw / ((long long)S * H));
  const float* q = Q + b * st.q[2] + h * st.q[1] + i * st.q[0];
  const float* kb = K + b * st.k[2] + h * st.k[1];
  const float* vb = V + b * st.v[2] + h * st.v[1];
  float qr[8], acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int d = lane + 32 * c;
    qr[c] = d < D ? q[d] : 0.f;
    acc[c] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int jend = CAUSAL ? i + 1 : S;
  for (int j = 0; j < jend; ++j) {
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int d = lane + 32 * c;
      if (d < D) s = fmaf(qr[c], kb[j * st.k[0] + d], s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= scale;
    const float mn = fmaxf(m, s);
    const float a = expf(m - mn), p = expf(s - mn);
    l = l * a + p;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int d = lane + 32 * c;
      acc[c] = acc[c] * a + (d < D ? p * vb[j * st.v[0] + d] : 0.f);
    }
    m = mn;
  }
  float* o = O + b * st.o[2] + h * st.o[1] + i * st.o[0];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int d = lane + 32 * c;
    if (d < D) o[d] = acc[c] / l;
  }
}

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

// 4-D map of one attention operand with element strides (seq, head, batch);
// the smaller of the seq / head strides becomes dimension 1.  Elements are
// rounded to tf32 (nearest-even) by the TMA unit.  Sets *hs when dimension 1
// is the head.
agpu_status make_attn_map(CUtensorMap* map, const float* base, int D, int S, int H, int B,
                          const long long (&st)[3], uint32_t rows, bool mn_major, bool* hs) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AGPU_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  *hs = st[1] < st[0];
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4], es[4] = {1, 1, 1, 1};
  dims[0] = D;
  box[0] = 32;
  if (*hs) {
    dims[1] = H; strides[0] = st[1] * 4; box[1] = 1;
    dims[2] = S; strides[1] = st[0] * 4; box[2] = rows;
  } else {
    dims[1] = S; strides[0] = st[0] * 4; box[1] = rows;
    dims[2] = H; strides[1] = st[1] * 4; box[2] = 1;
  }
  dims[3] = B; strides[2] = (B > 1 ? st[2] : (long long)std::max(st[0] * S, st[1] * H)) * 4;
  box[3] = 1;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, 4, const_cast<float*>(base), dims,
                  strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(AGPU_ERR_CUDA, "sdpa: tensor map encode failed (%d); strides must be "
                "multiples of 4 elements", (int)r);
  return AGPU_OK;
}

template <int D, bool CAUSAL>
agpu_status run_attention_tc(agpu_device* dev, const float* q, const float* k, const float* v,
                             float* o, int B, int H, int s, const AttnStrides& sd,
                             cudaStream_t st) {
  using C = AttnCfg<D>;
  CUtensorMap tk, tv;
  bool hk, hv;
  AGPU_TRY(make_attn_map(&tk, k, D, s, H, B, sd.k, KT, false, &hk));
  AGPU_TRY(make_attn_map(&tv, v, D, s, H, B, sd.v, KT, true, &hv));
  AttnOut ol{sd.o[0], sd.o[1], sd.o[2], (hk ? 2 : 0) | (hv ? 4 : 0)};
  AttnQ qin{q, sd.q[0], sd.q[1], sd.q[2]};
  auto kern = attention_tf32_kernel<D, CAUSAL>;
  AGPU_CUDA((set_smem_once<attention_tf32_kernel<D, CAUSAL>>(dev, C::SMEM)));
  AttnTiles tiles;
  tiles.nqt = (int)ceil_div(s, QT);
  tiles.H = H;
  tiles.rows = QT;
  tiles.total = (long long)tiles.nqt * H * B;
  const unsigned grid = (unsigned)std::min<long long>(tiles.total, dev->sm_count);
  const float scale_log2 = (1.0f / sqrtf((float)D)) * kLog2e;
  kern<<<grid, kAttnThreads, C::SMEM, st>>>(tk, tv, qin, o, s, scale_log2, ol, tiles,
                                            dev->d_status);
  return after_launch(dev, "attention_tf32_kernel");
}

template <int D, bool CAUSAL>
agpu_status run_attention_pair(agpu_device* dev, const float* q, const float* k, const float* v,
                               float* o, int B, int H, int s, const AttnStrides& sd,
                               cudaStream_t st, float* lse = nullptr) {
  using C = PairAttnCfg<D>;
  CUtensorMap tk, tv;
  bool hk, hv;
  AGPU_TRY(make_attn_map(&tk, k, D, s, H, B, sd.k, KH, false, &hk));
  AGPU_TRY(make_attn_map(&tv, v, D, s, H, B, sd.v, KB, true, &hv));
  AttnOut ol{sd.o[0], sd.o[1], sd.o[2], (hk ? 2 : 0) | (hv ? 4 : 0)};
  AttnQ qin{q, sd.q[0], sd.q[1], sd.q[2]};
  auto kern = lse ? attention_pair_kernel<D, CAUSAL, true> : attention_pair_kernel<D, CAUSAL, false>;
  AGPU_CUDA(lse ? (set_smem_once<attention_pair_kernel<D, CAUSAL, true>>(dev, C::SMEM))
                : (set_smem_once<attention_pair_kernel<D, CAUSAL, false>>(dev, C::SMEM)));
  AttnTiles tiles;
  tiles.nqt = (int)ceil_div(s, 2 * QT);
  tiles.H = H;
  tiles.rows = 2 * QT;
  tiles.total = (long long)tiles.nqt * H * B;
  const long long pairs = std::min<long long>(tiles.total, dev->sm_count / 2);
  const float scale_log2 = (1.0f / sqrtf((float)D)) * kLog2e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kPairAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AGPU_CUDA(cudaLaunchKernelEx(&cfg, kern, tk, tv, qin, o, s, scale_log2, ol, tiles,
                               dev->d_status, lse));
  return after_launch(dev, "attention_pair_kernel");
}

}  // namespace

agpu_status launch_attention_strided(agpu_device* dev, const float* q, const float* k,
                                     const float* v, float* o, uint32_t B, uint32_t H,
                                     uint32_t s, uint32_t d, const long long (&qs)[3],
                                     const long long (&ks)[3], const long long (&vs)[3],
                                     const long long (&os)[3], bool causal, cudaStream_t st) {
  if ((uint64_t)B * H * s * d == 0) return AGPU_OK;
  AttnStrides sd;
  for (int i = 0; i < 3; ++i) {
    sd.q[i] = qs[i]; sd.k[i] = ks[i]; sd.v[i] = vs[i]; sd.o[i] = os[i];
  }
  bool pitch_ok = true;
  for (int i = 0; i < 3; ++i)
    pitch_ok = pitch_ok && sd.q[i] % 4 == 0 && sd.k[i] % 4 == 0 && sd.v[i] % 4 == 0 &&
               sd.o[i] % 4 == 0;
  const bool aligned = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15u) == 0;
  // fp32-level accuracy modes (3xTF32, FFMA) take the exact SIMT kernel
  const bool tc = effective_precision(dev) == AGPU_PREC_TF32 && aligned && pitch_ok &&
                  (d == 64 || d == 128) && s >= 64 && H <= 65535 && B <= 65535;
  // sequences of >= 256 rows run on CTA pairs (AGPU_SDPA_PAIR=0: single CTAs)
  static const bool pair_ok = [] {
    const char* e = getenv("AGPU_SDPA_PAIR");
    return !(e && e[0] == '0');
  }();
  if (tc && pair_ok && s >= 2 * QT) {
    if (d == 128)
      return causal ? run_attention_pair<128, true>(dev, q, k, v, o, B, H, s, sd, st)
                    : run_attention_pair<128, false>(dev, q, k, v, o, B, H, s, sd, st);
    return causal ? run_attention_pair<64, true>(dev, q, k, v, o, B, H, s, sd, st)
                  : run_attention_pair<64, false>(dev, q, k, v, o, B, H, s, sd, st);
  }
  if (tc) {
    if (d == 128)
      return causal ? run_attention_tc<128, true>(dev, q, k, v, o, B, H, s, sd, st)
                    : run_attention_tc<128, false>(dev, q, k, v, o, B, H, s, sd, st);
    return causal ? run_attention_tc<64, true>(dev, q, k, v, o, B, H, s, sd, st)
                  : run_attention_tc<64, false>(dev, q, k, v, o, B, H, s, sd, st);
  }
  if (d > 256) return fail(AGPU_ERR_UNSUPPORTED, "sdpa: head dim %u > 256", d);
  const long long warps = (long long)B * H * s;
  const unsigned blocks = (unsigned)ceil_div((uint64_t)warps * 32, 256);
  const float scale = 1.0f / sqrtf((float)d);
  if (causal)
    attention_simt_kernel<true><<<blocks, 256, 0, st>>>(q, k, v, o, B, H, s, d, scale, sd);
  else
    attention_simt_kernel<false><<<blocks, 256, 0, st>>>(q, k, v, o, B, H, s, d, scale, sd);
  return after_launch(dev, "attention_simt_kernel");
}

// The forward on CTA pairs with each row's log-sum-exp of its base-2 scores
// (s = q.k / sqrt(d) * log2 e, so P = 2^(s - lse)) into lse [bh, s];
// AGPU_ERR_UNSUPPORTED (nothing launched, no message) where the pair kernel
// does not run: another precision, s < 256, d not 64 or 128, pitches TMA
// cannot address, or AGPU_SDPA_PAIR=0.  Contiguous [bh, s, d] operands.
agpu_status launch_attention_lse(agpu_device* dev, const float* q, const float* k,
                                 const float* v, float* o, float* lse, uint32_t bh, uint32_t s,
                                 uint32_t d, bool causal, cudaStream_t st) {
  static const bool pair_ok = [] {
    const char* e = getenv("AGPU_SDPA_PAIR");
    return !(e && e[0] == '0');
  }();
  const bool aligned = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15u) == 0;
  if (!pair_ok || effective_precision(dev) != AGPU_PREC_TF32 || !aligned ||
      (d != 64 && d != 128) || s < 2 * QT || bh > 65535 || bh == 0)
    return AGPU_ERR_UNSUPPORTED;
  AttnStrides sd;
  const long long c[3] = {(long long)d, (long long)s * d, (long long)bh * s * d};
  for (int i = 0; i < 3; ++i) sd.q[i] = sd.k[i] = sd.v[i] = sd.o[i] = c[i];
  if (d == 128)
    return causal ? run_attention_pair<128, true>(dev, q, k, v, o, 1, bh, s, sd, st, lse)
                  : run_attention_pair<128, false>(dev, q, k, v, o, 1, bh, s, sd, st, lse);
  return causal ? run_attention_pair<64, true>(dev, q, k, v, o, 1, bh, s, sd, st, lse)
                : run_attention_pair<64, false>(dev, q, k, v, o, 1, bh, s, sd, st, lse);
}

// Contiguous [bh, s, d] operands: heads = bh, batch = 1.
agpu_status launch_attention(agpu_device* dev, const float* q, const float* k, const float* v,
                             float* o, uint32_t bh, uint32_t s, uint32_t d, bool causal,
                             cudaStream_t st) {
  const long long c[3] = {(long long)d, (long long)s * d, (long long)bh * s * d};
  return launch_attention_strided(dev, q, k, v, o, 1, bh, s, d, c, c, c, c, causal, st);
}

}  // namespace agpu
