// Fused scaled-dot-product attention on sm_100a (flash-style, fp32 I/O,
// tcgen05 kind::tf32 with fp32 accumulation).
//
// Replaces the reference's unfused composition (src/ops/attention.rs:149-169):
// transpose(K) -> batch_matmul(Q, K^T) -> scale(1/sqrt(d)) -> softmax ->
// batch_matmul(P, V), which writes and re-reads the [BH, S, S] scores three
// times.  Same result, no scores in HBM:
//
//   CTA = one 128-row query tile of one (batch, head); 192 threads.
//   warp 0     TMA: Q tile once (4 boxes of 32 head dims), then K_j and V_j
//              blocks of 64 keys into a 2-deep ring (V with the 32-byte-atom
//              swizzle: it is the MN-major B operand of P V).
//   warp 1     one lane issues the MMAs:
//                S_j  = Q K_j^T   (M 128, N 64, K = d)      -> TMEM S[j%2]
//                O   += P_j V_j   (M 128, N = d, K 64), A = P_j read from TMEM
//              S_{j+1} is issued before waiting for P_j, so it overlaps the
//              softmax of block j.
//   warps 2-5  thread = query row: read its 64 scores from TMEM, online
//              softmax in base 2 (scale*log2 e folded into one multiply), write
//              P_j back over S_j in TMEM; O (in TMEM) is rescaled only when
//              the row max grows by more than 2^8 since the last rescale, so
//              exp2 never exceeds 256 and most blocks skip the rescale.
//              Finally O / l is written to HBM.
// Shapes outside the tensor-core path (head dim not 64/128, unaligned
// pitches) use a warp-per-query SIMT kernel with the same online softmax.
#include <algorithm>

#include "agpu_internal.cuh"
#include "ptx.cuh"
#include "umma_kernel.cuh"

namespace agpu {

namespace {

constexpr int QT = 128;     // query rows per CTA
constexpr int KT = 64;      // keys per block
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;

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
  int hs;  // bit 0: q, bit 1: k, bit 2: v
};

template <int D>
struct AttnCfg {
  static constexpr int Q_BYTES = QT * D * 4;
  static constexpr int K_BYTES = KT * D * 4;
  static constexpr int V_BYTES = KT * D * 4;
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int STAGES = 2;
  static constexpr int SMEM = 1024 + Q_BYTES + STAGES * STAGE_BYTES + 256;
  static constexpr int S_COL = 0;         // S/P buffers: columns [0, 2*KT)
  static constexpr int O_COL = 2 * KT;    // O: columns [2*KT, 2*KT + D)
  static constexpr int TMEM_COLS = (2 * KT + D <= 256) ? 256 : 512;
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(192, 1)
    attention_tf32_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, float* __restrict__ out,
                          int S, float scale_log2, AttnOut ol, unsigned int* status) {
  using C = AttnCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* ring = smem + C::Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + C::STAGES * C::STAGE_BYTES);
  uint64_t* q_full = bars;          // [1]
  uint64_t* k_full = bars + 1;      // [2]
  uint64_t* v_full = bars + 3;      // [2]
  uint64_t* kv_empty = bars + 5;    // [2]
  uint64_t* s_full = bars + 7;      // [2]
  uint64_t* p_full = bars + 9;      // [2]
  uint64_t* o_done = bars + 11;     // [1]
  uint64_t* drain = bars + 12;      // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int head = blockIdx.y, bat = blockIdx.z;
  const int q0 = blockIdx.x * QT;
  // 4-D maps {d, s, h, b}, or {d, h, s, b} when the head stride is the smaller
  // one (e.g. [batch, seq, heads, d] activations); the box is rows x 32 dims.
  auto load = [&](void* dst, const CUtensorMap* m, uint64_t* bar, int d0, int s0, bool hs) {
    if (hs) ptx::tma_load_4d(dst, m, bar, d0, head, s0, bat);
    else ptx::tma_load_4d(dst, m, bar, d0, s0, head, bat);
  };
  const int nb_all = (S + KT - 1) / KT;
  const int nb = CAUSAL ? min(nb_all, (q0 + QT - 1) / KT + 1) : nb_all;

  auto stage_k = [&](int s) { return ring + s * C::STAGE_BYTES; };
  auto stage_v = [&](int s) { return ring + s * C::STAGE_BYTES + C::K_BYTES; };

  if (threadIdx.x == 0) {
    ptx::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&k_full[i], 1);
      ptx::mbar_init(&v_full[i], 1);
      ptx::mbar_init(&kv_empty[i], 1);
      ptx::mbar_init(&s_full[i], 1);
      ptx::mbar_init(&p_full[i], 128);
    }
    ptx::mbar_init(o_done, 1);
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
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < D / 32; ++c)
        load(sq + c * QT * 128, &tm_q, q_full, c * 32, q0, ol.hs & 1);
      long long issued = 0;
      for (int j = 0; j < nb; ++j) {
        const int st = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        if (!ptx::mbar_wait(&kv_empty[st], par, status, 0x201, abort_flag)) break;
        ptx::mbar_arrive_expect_tx(&k_full[st], C::K_BYTES);
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          load(stage_k(st) + c * KT * 128, &tm_k, &k_full[st], c * 32, j * KT, ol.hs & 2);
        ptx::mbar_arrive_expect_tx(&v_full[st], C::V_BYTES);
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          load(stage_v(st) + c * KT * 128, &tm_v, &v_full[st], c * 32, j * KT, ol.hs & 4);
        ++issued;
      }
      // never exit with loads in flight into this CTA's shared memory
      ptx::mbar_wait(q_full, 0, status, 0x207, nullptr);
      for (long long j = std::max<long long>(0, issued - 2); j < issued; ++j) {
        ptx::mbar_wait(&k_full[j & 1], (uint32_t)((j >> 1) & 1), status, 0x207, nullptr);
        ptx::mbar_wait(&v_full[j & 1], (uint32_t)((j >> 1) & 1), status, 0x207, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = ptx::make_idesc_tf32(QT, KT, false, false);
      constexpr uint32_t idesc_o = ptx::make_idesc_tf32(QT, D, false, true);
      const uint32_t q_addr = ptx::smem_u32(sq);
      bool ok = ptx::mbar_wait(q_full, 0, status, 0x202, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!ptx::mbar_wait(&k_full[st], (j >> 1) & 1, status, 0x203, abort_flag)) return false;
        ptx::tc_fence_after();
        const uint32_t k_addr = ptx::smem_u32(stage_k(st));
        const uint32_t d_tmem = tmem + C::S_COL + st * KT;
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
          const uint32_t off = (kk % 4) * 32;  // 8 fp32 inside the 128-byte row
          const uint64_t ad = umma::operand_desc<false>(q_addr + (kk / 4) * QT * 128 + off);
          const uint64_t bd = umma::operand_desc<false>(k_addr + (kk / 4) * KT * 128 + off);
          ptx::mma_tf32_ss(d_tmem, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(&s_full[st]);
        return true;
      };
      if (ok && nb > 0) ok = issue_s(0);
      for (int j = 0; j < nb && ok; ++j) {
        const int st = j & 1;
        if (j + 1 < nb && !issue_s(j + 1)) { ok = false; break; }
        if (!ptx::mbar_wait(&p_full[st], (j >> 1) & 1, status, 0x204, abort_flag)) { ok = false; break; }
        if (!ptx::mbar_wait(&v_full[st], (j >> 1) & 1, status, 0x205, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t v_addr = ptx::smem_u32(stage_v(st));
        const uint32_t p_tmem = tmem + C::S_COL + st * KT;
#pragma unroll
        for (int kk = 0; kk < KT / 8; ++kk) {
          // V chunk c (32 head dims x 64 keys, 8 KB) at c * KT * 128; 8 keys = 1024 B
          const uint64_t bd = ptx::make_sdesc(v_addr + kk * 1024, KT * 128, 512, 1);
          ptx::mma_tf32_ts(tmem + C::O_COL, p_tmem + kk * 8, bd, idesc_o,
                           (j > 0 || kk > 0) ? 1u : 0u);
        }
        ptx::mma_commit(&kv_empty[st]);
        ptx::mma_commit(o_done);
      }
      ptx::mma_commit(drain);
      ptx::mbar_wait(drain, 0, status, 0x206, nullptr);
    }
  } else {
    // ------------------------------------------------------ softmax rows --
    const int q = warp & 3;
    const int row = q * 32 + lane;            // accumulator lane = query row in tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int qrow = q0 + row;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      const int st = j & 1;
      if (!ptx::mbar_wait(&s_full[st], (j >> 1) & 1, status, 0x208, abort_flag)) { ok = false; break; }
      ptx::tc_fence_after();
      uint32_t s0[32], s1[32];
      const uint32_t sbase = tmem + lane_off + C::S_COL + st * KT;
      ptx::tmem_ld32(sbase, s0);
      ptx::tmem_ld32(sbase + 32, s1);
      ptx::tmem_wait_ld();
      float t[64];
      const int kv0 = j * KT;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        t[i] = __uint_as_float(s0[i]) * scale_log2;
        t[32 + i] = __uint_as_float(s1[i]) * scale_log2;
      }
      if (kv0 + KT > S || (CAUSAL && kv0 + KT - 1 > q0)) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const int kv = kv0 + i;
          if (kv >= S || (CAUSAL && kv > qrow)) t[i] = -INFINITY;
        }
      }
      float mx = t[0];
#pragma unroll
      for (int i = 1; i < 64; ++i) mx = fmaxf(mx, t[i]);
      const bool need = mx > m_used + kRescaleLog2;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mx : m_used;
        const float alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_new);
        if (j > 0) {
          // O holds P_0..P_{j-1} V; wait for PV_{j-1}, then rescale in place.
          if (!ptx::mbar_wait(o_done, (j - 1) & 1, status, 0x209, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            const uint32_t oaddr = tmem + lane_off + C::O_COL + c * 32;
            ptx::tmem_ld32(oaddr, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            ptx::tmem_st32(oaddr, o);
          }
          ptx::tmem_wait_st();
        }
        l *= alpha;
        m_used = m_new;
      }
      float ls = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = ex2(t[i] - m_used), p1 = ex2(t[32 + i] - m_used);
        ls += p0 + p1;
        s0[i] = round_tf32(p0);
        s1[i] = round_tf32(p1);
      }
      l += ls;
      ptx::tmem_st32(sbase, s0);
      ptx::tmem_st32(sbase + 32, s1);
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&p_full[st]);
    }
    if (ok && nb > 0 && ptx::mbar_wait(o_done, (nb - 1) & 1, status, 0x20a, abort_flag)) {
      ptx::tc_fence_after();
      const float inv = 1.0f / l;
      float* orow = out + (long long)bat * ol.b + (long long)head * ol.h + (long long)qrow * ol.s;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        ptx::tmem_ld32(tmem + lane_off + C::O_COL + c * 32, o);
        ptx::tmem_wait_ld();
        if (qrow < S) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            __stcs(reinterpret_cast<float4*>(orow + c * 32) + i,
                   make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                               __uint_as_float(o[4 * i + 2]) * inv,
                               __uint_as_float(o[4 * i + 3]) * inv));
        }
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
  CUtensorMap tq, tk, tv;
  bool hq, hk, hv;
  AGPU_TRY(make_attn_map(&tq, q, D, s, H, B, sd.q, QT, false, &hq));
  AGPU_TRY(make_attn_map(&tk, k, D, s, H, B, sd.k, KT, false, &hk));
  AGPU_TRY(make_attn_map(&tv, v, D, s, H, B, sd.v, KT, true, &hv));
  AttnOut ol{sd.o[0], sd.o[1], sd.o[2], (hq ? 1 : 0) | (hk ? 2 : 0) | (hv ? 4 : 0)};
  auto kern = attention_tf32_kernel<D, CAUSAL>;
  AGPU_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
  dim3 grid((unsigned)ceil_div(s, QT), (unsigned)H, (unsigned)B);
  const float scale_log2 = (1.0f / sqrtf((float)D)) * kLog2e;
  kern<<<grid, 192, C::SMEM, st>>>(tq, tk, tv, o, s, scale_log2, ol, dev->d_status);
  return after_launch(dev, "attention_tf32_kernel");
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
  const bool tc = dev->precision == AGPU_PREC_TF32 && aligned && pitch_ok &&
                  (d == 64 || d == 128) && s >= 64 && H <= 65535 && B <= 65535;
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

// Contiguous [bh, s, d] operands: heads = bh, batch = 1.
agpu_status launch_attention(agpu_device* dev, const float* q, const float* k, const float* v,
                             float* o, uint32_t bh, uint32_t s, uint32_t d, bool causal,
                             cudaStream_t st) {
  const long long c[3] = {(long long)d, (long long)s * d, (long long)bh * s * d};
  return launch_attention_strided(dev, q, k, v, o, 1, bh, s, d, c, c, c, c, causal, st);
}

}  // namespace agpu
