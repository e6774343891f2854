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
//     apply the epilogue in registers and write each 32x32 block through a
//     swizzled staging buffer with a TMA bulk tensor store (read-modify-write
//     segments transpose through shared memory and store coalesced rows);
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
#include <atomic>
#include <climits>
#include <cstdlib>
#include <cstring>

#include "agpu_internal.cuh"
#include "ptx.cuh"
#include "umma_kernel.cuh"
#include "umma2_kernel.cuh"
#include "umma2_splitk_kernel.cuh"
#include "umma2_x3_kernel.cuh"
#include "pair_launch.cuh"

namespace agpu {

using umma::BK;
using umma::BM;
using umma::kEpiStride;

namespace {

__device__ __forceinline__ float epi_act(float x, int act) {
  if (act == 1) return x / (1.0f + expf(-x));  // swish, src/ops/elementwise.rs:87
  if (act == 2) return fmaxf(x, 0.0f);         // relu
  return x;
}

// Row-major (batched) GEMM: tiles 128 x BN walk batch-major with a 16-row-
// block group swizzle (L2 reuse of the B column block across the group).
template <int BN_, bool A_MN_, bool B_MN_, bool ROWVEC_ = false>
struct GemmPolicy {
  static constexpr int BN = BN_;
  static constexpr bool A_MN = A_MN_, B_MN = B_MN_;
  // the row-vector modes' whole-tile epilogue (store_tile), compiled into
  // the pair kernel only for these instantiations, with a 13 KB slice of
  // extra epilogue memory per warp: three 4 KB blocks of P in flight (TMA
  // loads through C's map) and their mbarriers
  static constexpr bool TILE_EPILOGUE = ROWVEC_;
  static constexpr int kPBufs = 3;
  static constexpr int EPI_EXTRA = ROWVEC_ ? umma::kEpiWarps * 13 * 1024 : 0;
  int M, N, K, tiles_m, tiles_n;
  long long tiles;
  float* C;
  long long c_batch;  // M * N
  // fused epilogue (applied once): C = act(A*B + bias[col] + resid[row, col])
  const float* bias;   // [N] or null (Linear bias, the reference's add_per_col)
  const float* resid;  // [batch, M, N] or null (residual add)
  int act;             // 0 none, 1 swish, 2 relu
  // row-vector modes (GemmEpilogue::mode; TMA-store path only)
  int mode = 0;
  const float* rowvec = nullptr;  // [batch, M]
  float ep_scale = 1.0f;
  bool causal = false;
  // MN-major operand loaded through the 4-D chunked view, one TMA box per
  // stage (else one box per 32-column chunk)
  bool a_chunked = false, b_chunked = false;
  // C written by TMA bulk stores (store_tma) through this map {N, M, batch},
  // box 32 x 32, 128-byte swizzle; else by the transposing store
  bool c_tma = false;
  CUtensorMap tmap_c;

  struct Tile { int b, m0, n0; };

  __device__ long long num_tiles() const { return tiles; }
  __device__ int num_k() const { return (K + BK - 1) / BK; }

  __device__ Tile tile(long long t) const {
    const long long per_batch = (long long)tiles_m * tiles_n;
    Tile r;
    r.b = (int)(t / per_batch);
    const int q = (int)(t % per_batch);
    constexpr int G = 16;
    const int span = G * tiles_n;
    const int first_m = (q / span) * G;
    const int gsize = min(tiles_m - first_m, G);
    const int in_group = q % span;
    r.m0 = (first_m + in_group % gsize) * BM;
    r.n0 = (in_group / gsize) * BN;
    return r;
  }

  __device__ void load(const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* sa, uint8_t* sb,
                       uint64_t* bar, const Tile& t, int kb) const {
    const int k0 = kb * BK;
    if (!A_MN) {
      ptx::tma_load_3d(sa, ta, bar, k0, t.m0, t.b);
    } else if (a_chunked) {
      ptx::tma_load_4d(sa, ta, bar, 0, k0, t.m0 / 32, t.b);
    } else {
#pragma unroll
      for (int j = 0; j < BM / 32; ++j)
        ptx::tma_load_3d(sa + j * BK * 128, ta, bar, t.m0 + 32 * j, k0, t.b);
    }
    if (!B_MN) {
      ptx::tma_load_3d(sb, tb, bar, k0, t.n0, t.b);
    } else if (b_chunked) {
      ptx::tma_load_4d(sb, tb, bar, 0, k0, t.n0 / 32, t.b);
    } else {
#pragma unroll
      for (int j = 0; j < BN / 32; ++j)
        ptx::tma_load_3d(sb + j * BK * 128, tb, bar, t.n0 + 32 * j, k0, t.b);
    }
  }

  __device__ bool col_live(const Tile& t, int col0) const { return t.n0 + col0 < N; }

  // SwiGLU epilogue (act 3): B's columns come in 32-column blocks, gate block
  // j = columns [64j, 64j+32), up block j = [64j+32, 64j+64); C is [M, N/2]
  // with C[:, 32j + i] = swish(gate) * up.  The pair kernel hands both blocks
  // of a pair to store_swiglu.
  __device__ bool paired() const { return act == 3; }

  __device__ void store_swiglu(const Tile& t, int row, int col0, const uint32_t (&g)[32],
                               const uint32_t (&u)[32], float* stg, int lane) const {
    float4* srow = reinterpret_cast<float4*>(stg + lane * kEpiStride);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float gv = __uint_as_float(g[4 * j + e]);
        a[e] = gv / (1.0f + expf(-gv)) * __uint_as_float(u[4 * j + e]);
      }
      srow[j] = make_float4(a[0], a[1], a[2], a[3]);
    }
    __syncwarp();
    const int no = N / 2;
    const int row_base = t.m0 + row - lane;
    const int col = (t.n0 + col0) / 2 + (lane & 7) * 4;
    float* Cb = C + (long long)t.b * c_batch;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = i * 4 + (lane >> 3);
      const int grow = row_base + r;
      const float4 val = *reinterpret_cast<const float4*>(stg + r * kEpiStride + (lane & 7) * 4);
      if (grow < M && col < no)
        *reinterpret_cast<float4*>(Cb + (long long)grow * no + col) = val;
    }
    __syncwarp();
  }

  // Mode 2 runs a whole-tile epilogue (TILE_EPILOGUE instantiations: the
  // pair kernel calls store_tile instead of store per chunk): the warp walks
  // the tile's live 32-column chunks itself, so it can overlap across chunks
  // -- the next chunk's tensor-memory load is issued while this one is staged
  // and stored, and the blocks of P up to kPBufs chunks ahead are in flight.
  // (Mode 1 measured faster per chunk, in store_tma.)
  __device__ bool whole_tile() const { return mode == 2; }

  // Warp slice of the extra epilogue memory: kPBufs blocks of P (4 KB
  // each, 1024-aligned, the 128-byte swizzle of C's map), then kPBufs
  // mbarriers, then the count of blocks this warp has loaded so far (which
  // fixes each buffer's phase across tiles).
  __device__ static uint64_t* pbar(float* xtra) {
    return reinterpret_cast<uint64_t*>(xtra + kPBufs * 1024);
  }
  __device__ static unsigned int* pcount(float* xtra) {
    return reinterpret_cast<unsigned int*>(pbar(xtra) + kPBufs);
  }
  __device__ void init_extra(float* xtra) const {
    for (int k = 0; k < kPBufs; ++k) ptx::mbar_init(pbar(xtra) + k, 1);
    *pcount(xtra) = 0u;
  }

  // Thread `lane` owns row t.m0 + row; trow addresses the warp's TMEM lanes
  // at the tile's first accumulator column.  Block c of P (the warp's 32
  // rows, the tile's columns 32 c ..) is the warp's load number g + c, into
  // buffer (g + c) % kPBufs; lane 0 keeps kPBufs loads in flight, issuing
  // block c + kPBufs as soon as block c has been read.  Every wait is
  // bounded; after an expired one the warp waits (bounded) for its loads
  // still in flight and returns false.
  __device__ bool store_tile(const Tile& t, int row, uint32_t trow, float* stg, float* xtra,
                             int lane, unsigned int* status, volatile int* abort_flag) const {
    const int grow = t.m0 + row, row_base = grow - lane;
    const float rv = grow < M ? __ldg(rowvec + (long long)t.b * M + grow) : 0.f;
    const int nch = min(BN / 32, (N - t.n0 + 31) / 32);
    uint64_t* bars = pbar(xtra);
    const unsigned int g = *reinterpret_cast<volatile unsigned int*>(pcount(xtra));
    auto issue = [&](int c) {  // lane 0
      const int k = (int)((g + c) % kPBufs);
      ptx::mbar_arrive_expect_tx(bars + k, 4096);
      ptx::tma_load_3d(xtra + k * 1024, &tmap_c, bars + k, t.n0 + 32 * c, row_base, t.b);
    };
    if (lane == 0)
      for (int c = 0; c < min(kPBufs, nch); ++c) issue(c);
    bool ok = true;
    int c = 0;
    uint32_t v[32];
    ptx::tmem_ld32(trow, v);
#pragma unroll 1
    for (; c < nch; ++c) {
      const int col = t.n0 + 32 * c;
      float* buf = stg + (c & 1) * 1024;
      const unsigned int gc = g + c;
      float* pb = xtra + (gc % kPBufs) * 1024;
      if (lane == 0) ptx::bulk_wait_read1();  // the store two chunks back has read `buf`
      ptx::tmem_wait_ld();
      __syncwarp();
      uint8_t* rowp = reinterpret_cast<uint8_t*>(buf) + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4)) =
            make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                        __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
      if (c + 1 < nch) ptx::tmem_ld32(trow + 32 * (c + 1), v);  // lands while this chunk stores
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(bars + gc % kPBufs, (gc / kPBufs) & 1,
                                                  status, 0x309, abort_flag));
      if (!ok) break;
      __syncwarp();
      // dS = P o (dP - D[row]) * scale, row 4 i + lane / 8 of both blocks
      // (the same swizzled positions)
      const int jj = lane & 7;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = 4 * i + (lane >> 3);
        const float d = __shfl_sync(0xffffffffu, rv, r);
        const int off = r * 128 + ((jj ^ (r & 7)) << 4);
        float4* cell = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(buf) + off);
        const float4 pv = *reinterpret_cast<const float4*>(reinterpret_cast<uint8_t*>(pb) + off);
        const float4 a = *cell;
        float4 o;
        o.x = pv.x * (a.x - d) * ep_scale;
        o.y = pv.y * (a.y - d) * ep_scale;
        o.z = pv.z * (a.z - d) * ep_scale;
        o.w = pv.w * (a.w - d) * ep_scale;
        *cell = o;
      }
      // the async proxy sees the staged block; and pb's generic reads come
      // before the TMA load that refills it
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (c + kPBufs < nch) issue(c + kPBufs);
        if (row_base < M) {
          ptx::tma_store_3d(&tmap_c, buf, col, row_base, t.b);
          ptx::bulk_commit();
        }
      }
    }
    if (!ok) {
      // loads c .. min(c + kPBufs, nch) - 1 may still be in flight
      if (c + 1 < nch) ptx::tmem_wait_ld();
      for (int e = c; e < min(c + kPBufs, nch); ++e)
        ptx::mbar_wait_for(bars + (g + e) % kPBufs, ((g + e) / kPBufs) & 1, nullptr, 0, nullptr,
                           ptx::kWaitLimitNs);
    }
    __syncwarp();
    if (lane == 0) {
      *pcount(xtra) = g + (unsigned int)nch;
      ptx::bulk_wait_read0();  // the next tile starts again at buffer 0
    }
    __syncwarp();
    return ok;
  }

  // TMA store of one 32 x 32 block (c_tma): thread `lane` holds row m0 + row,
  // columns n0 + col0 .. +31, applies the epilogue in registers and writes
  // its row into one of the warp's two 4 KB staging buffers in the 128-byte
  // swizzle the map expects (16-byte chunk j of row r at position j ^ r % 8,
  // so the warp's writes spread over all banks); one lane then issues the
  // bulk tensor store and moves on.  A buffer is rewritten two blocks later,
  // once the store that read it has (cp.async.bulk.wait_group.read 1); the
  // TMA unit clips rows past M and columns past N.  Blocks alternate buffers
  // by column-chunk parity; a tile whose last live chunk is even (an edge
  // tile with an odd chunk count) drains its stores before the next tile
  // starts again at buffer 0.
  __device__ void store_tma(const Tile& t, int row, int col0, const uint32_t (&v)[32],
                            float* stg, int lane) const {
    float* buf = stg + ((col0 >> 5) & 1) * 1024;
    if (lane == 0) ptx::bulk_wait_read1();
    __syncwarp();
    const int grow = t.m0 + row, col = t.n0 + col0;
    float4 w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      w[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                         __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
    if (bias) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (col + 4 * j < N) {
          const float4 bb = __ldg(reinterpret_cast<const float4*>(bias + col + 4 * j));
          w[j].x += bb.x; w[j].y += bb.y; w[j].z += bb.z; w[j].w += bb.w;
        }
    }
    if (resid && grow < M) {
      const float* rp = resid + (long long)t.b * c_batch + (long long)grow * N + col;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (col + 4 * j < N) {
          const float4 rr = __ldg(reinterpret_cast<const float4*>(rp + 4 * j));
          w[j].x += rr.x; w[j].y += rr.y; w[j].z += rr.z; w[j].w += rr.w;
        }
    }
    if (act) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        w[j].x = epi_act(w[j].x, act); w[j].y = epi_act(w[j].y, act);
        w[j].z = epi_act(w[j].z, act); w[j].w = epi_act(w[j].w, act);
      }
    }
    if (mode == 1) {  // P = 2^(S * scale - L[row]), 0 above the diagonal if causal
      const float rv = grow < M ? __ldg(rowvec + (long long)t.b * M + grow) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int cc = col + 4 * j;
        w[j].x = (causal && cc > grow) ? 0.f : ptx::ex2_approx(fmaf(w[j].x, ep_scale, -rv));
        w[j].y = (causal && cc + 1 > grow) ? 0.f : ptx::ex2_approx(fmaf(w[j].y, ep_scale, -rv));
        w[j].z = (causal && cc + 2 > grow) ? 0.f : ptx::ex2_approx(fmaf(w[j].z, ep_scale, -rv));
        w[j].w = (causal && cc + 3 > grow) ? 0.f : ptx::ex2_approx(fmaf(w[j].w, ep_scale, -rv));
      }
    }
    uint8_t* rowp = reinterpret_cast<uint8_t*>(buf) + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4)) = w[j];
    ptx::fence_proxy_async_smem();  // the async proxy (TMA) sees the staged block
    __syncwarp();
    const int row_base = grow - lane;
    if (lane == 0) {
      if (row_base < M && col < N) {
        ptx::tma_store_3d(&tmap_c, buf, col, row_base, t.b);
        ptx::bulk_commit();
      }
      if (((col0 >> 5) & 1) == 0 && (col0 + 32 >= BN || col + 32 >= N)) ptx::bulk_wait_read0();
    }
  }

  // Thread `lane` holds row (row_base + lane), columns n0+col0 .. +31.  The
  // warp transposes its 32x32 block through shared memory so that each
  // store instruction writes four full 128-byte row segments.  A tile's only
  // (last, not accumulating) write goes through store_tma when the map is set.
  __device__ void store(const Tile& t, int row, int col0, const uint32_t (&v)[32], float* stg,
                        int lane, bool accumulate, bool last) const {
    if (c_tma && last && !accumulate) {
      store_tma(t, row, col0, v, stg, lane);
      return;
    }
    float4* srow = reinterpret_cast<float4*>(stg + lane * kEpiStride);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      srow[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                            __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
    __syncwarp();
    const int row_base = t.m0 + row - lane;
    const int col = t.n0 + col0 + (lane & 7) * 4;
    float* Cb = C + (long long)t.b * c_batch;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = i * 4 + (lane >> 3);
      const int grow = row_base + r;
      float4 val = *reinterpret_cast<const float4*>(stg + r * kEpiStride + (lane & 7) * 4);
      if (grow < M && col < N) {
        const long long off = (long long)grow * N + col;
        float4* dst = reinterpret_cast<float4*>(Cb + off);
        if (accumulate) {
          const float4 o = *dst;
          val.x += o.x; val.y += o.y; val.z += o.z; val.w += o.w;
        } else {
          if (bias) {
            const float4 bb = __ldg(reinterpret_cast<const float4*>(bias + col));
            val.x += bb.x; val.y += bb.y; val.z += bb.z; val.w += bb.w;
          }
          if (resid) {
            const float4 rr =
                __ldg(reinterpret_cast<const float4*>(resid + (long long)t.b * c_batch + off));
            val.x += rr.x; val.y += rr.y; val.z += rr.z; val.w += rr.w;
          }
        }
        if (last && act) {
          val.x = epi_act(val.x, act); val.y = epi_act(val.y, act);
          val.z = epi_act(val.z, act); val.w = epi_act(val.w, act);
        }
        *dst = val;
      }
    }
    __syncwarp();
  }
};

// CTA-pair GEMM tile: 256 x BN (BN = 256, or 512 as two MMAs of N 256);
// CTA `rank` of the pair stages rows m0 + 128*rank .. +127 of A and, per
// MMA sub-block s, columns n0 + s*MMA_N + rank*MMA_N/2 .. of B.
template <int BN_, bool A_MN_, bool B_MN_, bool ROWVEC_ = false>
struct GemmPairPolicy : GemmPolicy<BN_, A_MN_, B_MN_, ROWVEC_> {
  using Base = GemmPolicy<BN_, A_MN_, B_MN_, ROWVEC_>;
  using Tile = typename Base::Tile;
  using Cfg = umma::PairCfg<BN_>;
  static constexpr int PM = 2 * BM;  // tile rows of the pair
  static constexpr int HALF = Cfg::MMA_N / 2;  // B columns per CTA per sub-block

  __device__ Tile tile(long long t) const {
    const long long per_batch = (long long)this->tiles_m * this->tiles_n;
    Tile r;
    r.b = (int)(t / per_batch);
    const int q = (int)(t % per_batch);
    constexpr int G = 8;
    const int span = G * this->tiles_n;
    const int first_m = (q / span) * G;
    const int gsize = min(this->tiles_m - first_m, G);
    const int in_group = q % span;
    r.m0 = (first_m + in_group % gsize) * PM;
    r.n0 = (in_group / gsize) * BN_;
    return r;
  }

  __device__ Tile rank_tile(const Tile& t, int rank) const {
    Tile r = t;
    r.m0 += BM * rank;
    return r;
  }

  __device__ void load(const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* sa, uint8_t* sb,
                       uint32_t lbar, const Tile& t, int kb, int rank) const {
    const int k0 = kb * BK;
    const int m = t.m0 + BM * rank;
    if (!A_MN_) {
      ptx::tma_load_3d_pair(sa, ta, lbar, k0, m, t.b);
    } else if (this->a_chunked) {
      ptx::tma_load_4d_pair(sa, ta, lbar, 0, k0, m / 32, t.b);
    } else {
#pragma unroll
      for (int j = 0; j < BM / 32; ++j)
        ptx::tma_load_3d_pair(sa + j * BK * 128, ta, lbar, m + 32 * j, k0, t.b);
    }
#pragma unroll
    for (int sub = 0; sub < Cfg::NMMA; ++sub) {
      const int n = t.n0 + sub * Cfg::MMA_N + HALF * rank;
      if (!B_MN_) {
        ptx::tma_load_3d_pair(sb + sub * HALF * 128, tb, lbar, k0, n, t.b);
      } else if (this->b_chunked) {
        ptx::tma_load_4d_pair(sb + sub * (HALF / 32) * BK * 128, tb, lbar, 0, k0, n / 32, t.b);
      } else {
#pragma unroll
        for (int j = 0; j < HALF / 32; ++j)
          ptx::tma_load_3d_pair(sb + (sub * (HALF / 32) + j) * BK * 128, tb, lbar, n + 32 * j,
                                k0, t.b);
      }
    }
  }
};

// 3xTF32 on CTA pairs (umma2_x3_kernel.cuh): the pair tile plus the number
// of K-blocks each accumulator segment sums before the epilogue folds it into
// the running sum in tensor memory.
template <int BN_, bool A_MN_, bool B_MN_>
struct GemmPairX3Policy : GemmPairPolicy<BN_, A_MN_, B_MN_> {
  int seg = 16;
};

// ------------------------------------------------------------ SIMT FFMA --
// Exact fp32 GEMM, 64x64 tile per 256 threads, 4x4 outputs per thread,
// arbitrary strides/alignment.  a_trans: A stored [K,M]; b_trans: B stored [N,K].
template <bool AT, bool BT>
__global__ void __launch_bounds__(256) gemm_ffma_kernel(const float* __restrict__ A,
                                                        const float* __restrict__ B,
                                                        float* __restrict__ C, int M, int N,
                                                        int K, GemmEpilogue ep) {
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
      if (gn < N) {
        float v = acc[i][j];
        if (ep.bias) v += ep.bias[gn];
        if (ep.resid) v += ep.resid[(long long)b * M * N + (long long)gm * N + gn];
        C[(long long)gm * N + gn] = epi_act(v, ep.act);
      }
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
// otherwise the plain 128-byte swizzle.  `round_tf32` makes the TMA unit
// round every element to tf32 (nearest, ties to even) on its way into shared
// memory; the tensor core itself truncates fp32 operands to tf32, so rounding
// first halves the conversion error and removes its bias.
agpu_status make_tmap_f32_3d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer,
                             uint64_t batch, uint64_t batch_stride_elems, uint32_t box_inner,
                             uint32_t box_outer, bool mn_major, bool round_tf32) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AGPU_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {inner * 4, batch_stride_elems * 4};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      round_tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(map, dt, 3, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(AGPU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) inner=%llu outer=%llu", (int)r,
                (unsigned long long)inner, (unsigned long long)outer);
  return AGPU_OK;
}

// 4-D fp32 view {32, K, MN/32, batch} of an MN-major operand stored
// [batch][K][MN] with MN % 32 == 0: the third dimension steps 32-element
// chunks (128 bytes), so one box {32, BK, chunks, 1} lands as `chunks`
// consecutive BK x 128-byte MN-major swizzle atoms -- the same shared-memory
// image as `chunks` boxes of the 3-D view, from one TMA instruction.
static agpu_status make_tmap_f32_chunked(CUtensorMap* map, const float* base, uint64_t mn,
                                         uint64_t k, uint64_t batch, uint32_t chunks,
                                         bool round_tf32) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AGPU_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[4] = {32, k, mn / 32, batch};
  cuuint64_t strides[3] = {mn * 4, 128, k * mn * 4};
  cuuint32_t box[4] = {32, BK, chunks, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      round_tf32 ? CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(map, dt, 4, const_cast<float*>(base), dims,
                  strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(AGPU_ERR_CUDA, "cuTensorMapEncodeTiled (chunked) failed (%d) mn=%llu k=%llu",
                (int)r, (unsigned long long)mn, (unsigned long long)k);
  return AGPU_OK;
}

// Tensor maps of both operands of the tensor-core GEMMs; `b_box` = B rows
// (K-major) or columns (MN-major) one CTA stages per stage.  MN-major
// operands whose MN extent is a multiple of 32 take the chunked view (one
// TMA instruction per operand per stage instead of one per 32 columns);
// AGPU_GEMM_CHUNKED=0 keeps the per-chunk loads.  `round` = TFLOAT32 maps
// (round to nearest on the way in); 3xTF32 splits exact FLOAT32 operands.
template <class P>
static agpu_status make_gemm_maps(CUtensorMap* ta, CUtensorMap* tb, P* pol, const float* a,
                                  const float* b, uint32_t batch, uint32_t m, uint32_t n,
                                  uint32_t k, uint32_t b_box, bool round) {
  static const bool chunk_ok = [] {
    const char* e = getenv("AGPU_GEMM_CHUNKED");
    return !(e && e[0] == '0');
  }();
  pol->a_chunked = P::A_MN && chunk_ok && m % 32 == 0;
  pol->b_chunked = P::B_MN && chunk_ok && n % 32 == 0;
  if (!P::A_MN)
    AGPU_TRY(make_tmap_f32_3d(ta, a, k, m, batch, (uint64_t)m * k, BK, BM, false, round));
  else if (pol->a_chunked)
    AGPU_TRY(make_tmap_f32_chunked(ta, a, m, k, batch, BM / 32, round));
  else
    AGPU_TRY(make_tmap_f32_3d(ta, a, m, k, batch, (uint64_t)m * k, 32, BK, true, round));
  if (!P::B_MN)
    AGPU_TRY(make_tmap_f32_3d(tb, b, k, n, batch, (uint64_t)k * n, BK, b_box, false, round));
  else if (pol->b_chunked)
    AGPU_TRY(make_tmap_f32_chunked(tb, b, n, k, batch, b_box / 32, round));
  else
    AGPU_TRY(make_tmap_f32_3d(tb, b, n, k, batch, (uint64_t)k * n, 32, BK, true, round));
  return AGPU_OK;
}

// The map of C for the TMA-store epilogue: {N, M, batch}, 32 x 32 boxes,
// 128-byte swizzle (AGPU_GEMM_TMA_STORE=0: the transposing store instead).
// SwiGLU writes an N/2-wide C through its own store.
bool tma_store_enabled() {
  static const bool enabled = [] {
    const char* e = getenv("AGPU_GEMM_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  return enabled;
}

template <class P>
static agpu_status make_c_map(P* pol, float* c, uint32_t batch, uint32_t m, uint32_t n, int act) {
  pol->c_tma = false;
  if (!tma_store_enabled() || act == 3 || n % 4 != 0 || (reinterpret_cast<uintptr_t>(c) & 15) != 0)
    return AGPU_OK;
  AGPU_TRY(make_tmap_f32_3d(&pol->tmap_c, c, n, m, batch, (uint64_t)m * n, 32, 32, false, false));
  pol->c_tma = true;
  return AGPU_OK;
}

template <int BN, bool A_MN, bool B_MN, bool X3>
static agpu_status run_tc(agpu_device* dev, const float* a, const float* b, float* c,
                          uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                          const GemmEpilogue& ep, cudaStream_t s) {
  using P = GemmPolicy<BN, A_MN, B_MN>;
  using Cfg = umma::Cfg<BN, X3>;
  CUtensorMap ta, tb;
  P pol;
  // A: K-major stored [M,K] -> dims {K, M}; MN-major stored [K,M] -> dims {M, K}.
  // B: MN-major stored [K,N] -> dims {N, K}; K-major stored [N,K] -> dims {K, N}.
  AGPU_TRY(make_gemm_maps(&ta, &tb, &pol, a, b, batch, m, n, k, BN, !X3));
  pol.M = m; pol.N = n; pol.K = k;
  pol.tiles_m = (int)ceil_div(m, BM);
  pol.tiles_n = (int)ceil_div(n, BN);
  pol.tiles = (long long)pol.tiles_m * pol.tiles_n * batch;
  pol.C = c;
  pol.c_batch = (long long)m * n;
  pol.bias = ep.bias;
  pol.resid = ep.resid;
  pol.act = ep.act;
  AGPU_TRY(make_c_map(&pol, c, batch, m, n, ep.act));
  auto kern = umma::umma_tf32_kernel<P, X3>;
  AGPU_CUDA((set_smem_once<umma::umma_tf32_kernel<P, X3>>(dev, Cfg::SMEM)));
  const long long grid = std::min<long long>(pol.tiles, dev->sm_count);
  kern<<<(unsigned)grid, Cfg::THREADS, Cfg::SMEM, s>>>(ta, tb, pol, dev->d_status);
  return after_launch(dev, "gemm_tf32 (umma_tf32_kernel)");
}

template <int BN, bool A_MN, bool B_MN, bool ROWVEC = false>
static agpu_status run_tc_pair(agpu_device* dev, const float* a, const float* b, float* c,
                               uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                               const GemmEpilogue& ep, cudaStream_t s) {
  using P = GemmPairPolicy<BN, A_MN, B_MN, ROWVEC>;
  CUtensorMap ta, tb;
  P pol;
  AGPU_TRY(make_gemm_maps(&ta, &tb, &pol, a, b, batch, m, n, k, P::HALF, true));
  pol.M = m; pol.N = n; pol.K = k;
  pol.tiles_m = (int)ceil_div(m, P::PM);
  pol.tiles_n = (int)ceil_div(n, BN);
  pol.tiles = (long long)pol.tiles_m * pol.tiles_n * batch;
  pol.C = c;
  pol.c_batch = (long long)m * (ep.act == 3 ? n / 2 : n);
  pol.bias = ep.bias;
  pol.resid = ep.resid;
  pol.act = ep.act;
  pol.mode = ep.mode;
  pol.rowvec = ep.rowvec;
  pol.ep_scale = ep.scale;
  pol.causal = ep.causal;
  AGPU_TRY(make_c_map(&pol, c, batch, m, n, ep.act));
  if (ep.mode != 0 && !pol.c_tma) return fail(AGPU_ERR_CUDA, "gemm: row-vector mode without a C map");
  return launch_pair(dev, ta, tb, pol, pol.tiles, s,
                     "gemm_tf32 (umma_tf32_pair_kernel)");
}

// K-blocks (of 32) per accumulator segment of the 3xTF32 pair kernel:
// AGPU_X3_SEG in the environment, default 16 (K = 512); 0 = no segments.
static int x3_seg() {
  static const int v = [] {
    const char* e = getenv("AGPU_X3_SEG");
    return e ? std::max(0, atoi(e)) : 16;
  }();
  return v;
}

// 3xTF32 GEMM on 256 x 256 CTA-pair tiles: lo(A), lo(B) into pool scratch by
// one elementwise pass, then the pair kernel reads each operand twice (as
// stored: its hi part; and its lo part) and sums three products per slice.
template <bool A_MN, bool B_MN>
static agpu_status run_tc_pair_x3(agpu_device* dev, const float* a, const float* b, float* c,
                                  uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                                  const GemmEpilogue& ep, cudaStream_t s) {
  using P = GemmPairX3Policy<256, A_MN, B_MN>;
  using Cfg = umma::PairX3Cfg<256>;
  const uint64_t na = (uint64_t)batch * m * k, nb = (uint64_t)batch * k * n;
  void* scratch = nullptr;
  AGPU_TRY(pool_alloc(dev, (na + nb) * sizeof(float), &scratch, s));
  float* alo = static_cast<float*>(scratch);
  float* blo = alo + na;  // na % 4 == 0 (k % 4 == 0): 16-byte aligned
  const long long n4 = (long long)((na + nb) / 4);
  const long long grid = std::min<long long>((n4 + 255) / 256, 8LL * dev->sm_count);
  umma::tf32_lo_kernel<<<(unsigned)std::max<long long>(grid, 1), 256, 0, s>>>(
      reinterpret_cast<const float4*>(a), reinterpret_cast<float4*>(alo), (long long)(na / 4),
      reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(blo), (long long)(nb / 4));
  agpu_status st = after_launch(dev, "tf32_lo_kernel");
  CUtensorMap ta, tb, tal, tbl;
  P pol, pol_lo;
  if (st == AGPU_OK)
    st = make_gemm_maps(&ta, &tb, &pol, a, b, batch, m, n, k, P::HALF, false);
  if (st == AGPU_OK)
    st = make_gemm_maps(&tal, &tbl, &pol_lo, alo, blo, batch, m, n, k, P::HALF, false);
  if (st == AGPU_OK) {
    pol.M = m; pol.N = n; pol.K = k;
    pol.tiles_m = (int)ceil_div(m, P::PM);
    pol.tiles_n = (int)ceil_div(n, 256);
    pol.tiles = (long long)pol.tiles_m * pol.tiles_n * batch;
    pol.C = c;
    pol.c_batch = (long long)m * n;
    pol.bias = ep.bias;
    pol.resid = ep.resid;
    pol.act = ep.act;
    pol.seg = x3_seg();
    st = make_c_map(&pol, c, batch, m, n, ep.act);
  }
  if (st == AGPU_OK) {
    auto kern = umma::umma_x3_pair_kernel<P>;
    cudaError_t e = set_smem_once<umma::umma_x3_pair_kernel<P>>(dev, Cfg::SMEM);
    if (e == cudaSuccess) {
      const long long clusters = std::min<long long>(pol.tiles, std::max(1, dev->sm_count / 2));
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
      cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
      cfg.dynamicSmemBytes = Cfg::SMEM;
      cfg.stream = s;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tal, tbl, pol, dev->d_status);
    }
    st = e == cudaSuccess ? after_launch(dev, "gemm_3xtf32 (umma_x3_pair_kernel)")
                          : cuda_status(e, "gemm_3xtf32 (umma_x3_pair_kernel)");
  }
  pool_free(dev, scratch, s);
  return st;
}

// Split-K over a cluster of S CTA pairs per 256 x BN tile (S = 2 or 4,
// BN = 256 or 128).
template <int BN, bool A_MN, bool B_MN, int S>
static agpu_status run_tc_pair_splitk(agpu_device* dev, const float* a, const float* b, float* c,
                                      uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                                      const GemmEpilogue& ep, cudaStream_t s) {
  using P = GemmPairPolicy<BN, A_MN, B_MN>;
  using Cfg = umma::PairCfg<BN>;
  CUtensorMap ta, tb;
  P pol;
  AGPU_TRY(make_gemm_maps(&ta, &tb, &pol, a, b, batch, m, n, k, P::HALF, true));
  pol.M = m; pol.N = n; pol.K = k;
  pol.tiles_m = (int)ceil_div(m, P::PM);
  pol.tiles_n = (int)ceil_div(n, BN);
  pol.tiles = (long long)pol.tiles_m * pol.tiles_n * batch;
  pol.C = c;
  pol.c_batch = (long long)m * n;
  pol.bias = ep.bias;
  pol.resid = ep.resid;
  pol.act = ep.act;
  auto kern = umma::umma_tf32_pair_splitk_kernel<P, S>;
  AGPU_CUDA((set_smem_once<umma::umma_tf32_pair_splitk_kernel<P, S>>(dev, Cfg::SMEM)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * S * pol.tiles), 1, 1);
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2 * S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  AGPU_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, pol, dev->d_status));
  return after_launch(dev, "gemm_tf32 (umma_tf32_pair_splitk_kernel)");
}

// Clusters of 2*S CTAs of the split-K kernel that fit on the device at once
// (a cluster occupies 2*S SMs of one GPC: 15 of 8 CTAs on a B200).
template <int BN, int S>
static int splitk_max_clusters(agpu_device* dev) {
  static std::atomic<int> cached{-1};
  int v = cached.load(std::memory_order_acquire);
  if (v >= 0) return v;
  using P = GemmPairPolicy<BN, false, true>;
  using Cfg = umma::PairCfg<BN>;
  int n = 0;
  if (set_smem_once<umma::umma_tf32_pair_splitk_kernel<P, S>>(dev, Cfg::SMEM) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * S, 1, 1);
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2 * S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, umma::umma_tf32_pair_splitk_kernel<P, S>, &cfg) !=
        cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  cached.store(n, std::memory_order_release);
  return n;
}

// Split-K plan for a pair GEMM whose 256 x 256 tiles leave most SM pairs
// idle (fewer tiles than half the pairs): among 256 x 256 and 256 x 128 tiles
// with S = 4 or 2 K slices -- all S * tiles pairs busy at once, every tile's
// cluster resident at once, >= 2 K-blocks per slice -- the one with the least
// MMA work per pair (tile columns x K-blocks per slice), wider tiles first on
// a tie (fewer operand bytes per FLOP); else s = 1, no split.
// AGPU_GEMM_SPLITK=0 disables, =256 keeps 256-column tiles.
struct SplitK {
  int bn, s;
};

static SplitK splitk_plan(agpu_device* dev, uint32_t batch, uint32_t m, uint32_t n, uint32_t k) {
  static const int mode = [] {
    const char* e = getenv("AGPU_GEMM_SPLITK");
    if (e && e[0] == '0') return 0;
    if (e && strcmp(e, "256") == 0) return 2;
    return 1;
  }();
  SplitK best{256, 1};
  if (mode == 0) return best;
  const long long pairs = std::max(1, dev->sm_count / 2);
  const long long nk = ceil_div(k, BK);
  if (2 * (long long)ceil_div(m, 256) * ceil_div(n, 256) * batch > pairs) return best;
  long long best_work = LLONG_MAX;
  const SplitK cand[4] = {{256, 4}, {256, 2}, {128, 4}, {128, 2}};
  for (const SplitK& c : cand) {
    if (c.bn == 128 && mode == 2) continue;
    const long long tiles = (long long)ceil_div(m, 256) * ceil_div(n, c.bn) * batch;
    if (tiles * c.s > pairs || nk < 2 * c.s) continue;
    const int fit = c.bn == 256 ? (c.s == 4 ? splitk_max_clusters<256, 4>(dev)
                                            : splitk_max_clusters<256, 2>(dev))
                                : (c.s == 4 ? splitk_max_clusters<128, 4>(dev)
                                            : splitk_max_clusters<128, 2>(dev));
    if (tiles > fit) continue;
    const long long work = (long long)c.bn * ceil_div(nk, c.s);
    if (work < best_work) {
      best = c;
      best_work = work;
    }
  }
  return best;
}

template <int BN, int S>
static agpu_status run_splitk_layout(agpu_device* dev, const float* a, const float* b, float* c,
                                     uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool at,
                                     bool bt, const GemmEpilogue& ep, cudaStream_t s) {
  if (!at && !bt) return run_tc_pair_splitk<BN, false, true, S>(dev, a, b, c, batch, m, n, k, ep, s);
  if (!at && bt) return run_tc_pair_splitk<BN, false, false, S>(dev, a, b, c, batch, m, n, k, ep, s);
  if (at && !bt) return run_tc_pair_splitk<BN, true, true, S>(dev, a, b, c, batch, m, n, k, ep, s);
  return run_tc_pair_splitk<BN, true, false, S>(dev, a, b, c, batch, m, n, k, ep, s);
}

// The CTA-pair kernel serves TF32 GEMMs with at least one full 256 x 256 tile;
// AGPU_GEMM_PAIR=0 in the environment selects the single-CTA kernel instead.
static bool use_pair(uint32_t m, uint32_t n) {
  static const bool enabled = [] {
    const char* e = getenv("AGPU_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return enabled && m >= 256 && n >= 256;
}

// 256 x 512 pair tiles move a third fewer TMA bytes per FLOP than 256 x 256
// but have half as many tiles and a single-buffered accumulator, so the
// tensor core idles while a tile's 128 x 512 fp32 per CTA drains (about
// 12k SM cycles when every SM writes at once, against 46 cycles per unit of
// K of MMA work).  Take them when the estimated throughput -- tile-wave fill
// x column fill x that drain factor x the kernel efficiency measured for
// each width (0.99 wide at 8192^3, 0.88 for 256 x 256) -- is higher.
// AGPU_GEMM_WIDE=0 disables them.
static bool use_wide(const agpu_device* dev, uint32_t batch, uint32_t m, uint32_t n,
                     uint32_t k) {
  static const int mode = [] {
    const char* e = getenv("AGPU_GEMM_WIDE");
    return e ? (e[0] == '0' ? 0 : e[0] == '2' ? 2 : 1) : 1;
  }();
  if (mode == 0 || n < 512) return false;
  if (mode == 2) return true;
  const long long pairs = std::max(1, dev->sm_count / 2);
  const long long tm = ceil_div(m, 256);
  auto score = [&](long long bn, double eff) {
    const long long tn = ceil_div(n, bn);
    const long long tiles = tm * tn * batch;
    const double waves = (double)tiles / (double)(ceil_div(tiles, pairs) * pairs);
    return eff * waves * (double)n / (double)(tn * bn);
  };
  const double mma = 46.4 * (double)k, drain = 12000.0;
  return score(512, 0.99 * mma / (mma + drain)) > score(256, 0.88);
}

template <bool X3>
static agpu_status dispatch_tc(agpu_device* dev, const float* a, const float* b, float* c,
                               uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool at,
                               bool bt, const GemmEpilogue& ep, cudaStream_t s) {
  const bool wide = n > 128;
  if (X3 && use_pair(m, n)) {
    if (!at && !bt) return run_tc_pair_x3<false, true>(dev, a, b, c, batch, m, n, k, ep, s);
    if (!at && bt) return run_tc_pair_x3<false, false>(dev, a, b, c, batch, m, n, k, ep, s);
    if (at && !bt) return run_tc_pair_x3<true, true>(dev, a, b, c, batch, m, n, k, ep, s);
    return run_tc_pair_x3<true, false>(dev, a, b, c, batch, m, n, k, ep, s);
  }
  if (!X3 && use_pair(m, n)) {
    const SplitK sk = splitk_plan(dev, batch, m, n, k);
    if (sk.s == 4 && sk.bn == 256)
      return run_splitk_layout<256, 4>(dev, a, b, c, batch, m, n, k, at, bt, ep, s);
    if (sk.s == 2 && sk.bn == 256)
      return run_splitk_layout<256, 2>(dev, a, b, c, batch, m, n, k, at, bt, ep, s);
    if (sk.s == 4 && sk.bn == 128)
      return run_splitk_layout<128, 4>(dev, a, b, c, batch, m, n, k, at, bt, ep, s);
    if (sk.s == 2 && sk.bn == 128)
      return run_splitk_layout<128, 2>(dev, a, b, c, batch, m, n, k, at, bt, ep, s);
    if (use_wide(dev, batch, m, n, k)) {
      if (!at && !bt) return run_tc_pair<512, false, true>(dev, a, b, c, batch, m, n, k, ep, s);
      if (!at && bt) return run_tc_pair<512, false, false>(dev, a, b, c, batch, m, n, k, ep, s);
      if (at && !bt) return run_tc_pair<512, true, true>(dev, a, b, c, batch, m, n, k, ep, s);
      return run_tc_pair<512, true, false>(dev, a, b, c, batch, m, n, k, ep, s);
    }
    if (!at && !bt) return run_tc_pair<256, false, true>(dev, a, b, c, batch, m, n, k, ep, s);
    if (!at && bt) return run_tc_pair<256, false, false>(dev, a, b, c, batch, m, n, k, ep, s);
    if (at && !bt) return run_tc_pair<256, true, true>(dev, a, b, c, batch, m, n, k, ep, s);
    return run_tc_pair<256, true, false>(dev, a, b, c, batch, m, n, k, ep, s);
  }
  // B is MN-major unless stored transposed ([N,K]).
  if (wide) {
    if (!at && !bt) return run_tc<256, false, true, X3>(dev, a, b, c, batch, m, n, k, ep, s);
    if (!at && bt) return run_tc<256, false, false, X3>(dev, a, b, c, batch, m, n, k, ep, s);
    if (at && !bt) return run_tc<256, true, true, X3>(dev, a, b, c, batch, m, n, k, ep, s);
    return run_tc<256, true, false, X3>(dev, a, b, c, batch, m, n, k, ep, s);
  }
  if (!at && !bt) return run_tc<128, false, true, X3>(dev, a, b, c, batch, m, n, k, ep, s);
  if (!at && bt) return run_tc<128, false, false, X3>(dev, a, b, c, batch, m, n, k, ep, s);
  if (at && !bt) return run_tc<128, true, true, X3>(dev, a, b, c, batch, m, n, k, ep, s);
  return run_tc<128, true, false, X3>(dev, a, b, c, batch, m, n, k, ep, s);
}

static agpu_status run_ffma(agpu_device* dev, const float* a, const float* b, float* c,
                            uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool at, bool bt,
                            const GemmEpilogue& ep, cudaStream_t s) {
  dim3 grid((unsigned)ceil_div(n, 64), (unsigned)ceil_div(m, 64), batch);
  if (!at && !bt) gemm_ffma_kernel<false, false><<<grid, 256, 0, s>>>(a, b, c, m, n, k, ep);
  else if (!at && bt) gemm_ffma_kernel<false, true><<<grid, 256, 0, s>>>(a, b, c, m, n, k, ep);
  else if (at && !bt) gemm_ffma_kernel<true, false><<<grid, 256, 0, s>>>(a, b, c, m, n, k, ep);
  else gemm_ffma_kernel<true, true><<<grid, 256, 0, s>>>(a, b, c, m, n, k, ep);
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

bool gemm_rowvec_mode_ok(agpu_device* dev, const float* a, const float* b, const float* c,
                         uint32_t batch, uint32_t m, uint32_t n, uint32_t k) {
  return batch > 0 && effective_precision(dev) == AGPU_PREC_TF32 && use_pair(m, n) &&
         gemm_tc_eligible(a, b, c, m, n, k) && tma_store_enabled() &&
         splitk_plan(dev, batch, m, n, k).s == 1;
}

agpu_status launch_gemm_ex(agpu_device* dev, const float* a, const float* b, float* c,
                           uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool a_trans,
                           bool b_trans, const GemmEpilogue& ep, cudaStream_t s) {
  if (batch == 0 || m == 0 || n == 0) return AGPU_OK;
  const bool has_ep = ep.bias || ep.resid || ep.act;
  if (k == 0 && !has_ep) {
    AGPU_CUDA(cudaMemsetAsync(c, 0, (size_t)batch * m * n * sizeof(float), s));
    return AGPU_OK;
  }
  const agpu_precision p = effective_precision(dev);
  if (ep.mode != 0) {
    // C = A B^T only (the attention backward's S and dP products)
    if (ep.bias || ep.resid || ep.act || !ep.rowvec || k == 0 || a_trans || !b_trans ||
        !gemm_rowvec_mode_ok(dev, a, b, c, batch, m, n, k))
      return AGPU_ERR_UNSUPPORTED;
    return run_tc_pair<256, false, false, true>(dev, a, b, c, batch, m, n, k, ep, s);
  }
  if (ep.act == 3) {
    // SwiGLU: fused into the CTA-pair kernel's epilogue when that kernel runs
    // the GEMM whole; otherwise the plain GEMM into scratch, then swish * up
    // over the 32-column block pairs (rows of 64: gate 32 | up 32)
    const bool fused = p == AGPU_PREC_TF32 && !ep.bias && !ep.resid && n % 64 == 0 &&
                       use_pair(m, n) && gemm_tc_eligible(a, b, c, m, n, k) &&
                       splitk_plan(dev, batch, m, n, k).s == 1;
    if (fused) {
      if (use_wide(dev, batch, m, n, k)) {
        if (!a_trans && !b_trans) return run_tc_pair<512, false, true>(dev, a, b, c, batch, m, n, k, ep, s);
        if (!a_trans && b_trans) return run_tc_pair<512, false, false>(dev, a, b, c, batch, m, n, k, ep, s);
        if (a_trans && !b_trans) return run_tc_pair<512, true, true>(dev, a, b, c, batch, m, n, k, ep, s);
        return run_tc_pair<512, true, false>(dev, a, b, c, batch, m, n, k, ep, s);
      }
      if (!a_trans && !b_trans) return run_tc_pair<256, false, true>(dev, a, b, c, batch, m, n, k, ep, s);
      if (!a_trans && b_trans) return run_tc_pair<256, false, false>(dev, a, b, c, batch, m, n, k, ep, s);
      if (a_trans && !b_trans) return run_tc_pair<256, true, true>(dev, a, b, c, batch, m, n, k, ep, s);
      return run_tc_pair<256, true, false>(dev, a, b, c, batch, m, n, k, ep, s);
    }
    void* tmp = nullptr;
    AGPU_TRY(pool_alloc(dev, (size_t)batch * m * n * sizeof(float), &tmp, s));
    float* t = static_cast<float*>(tmp);
    GemmEpilogue plain;
    plain.bias = ep.bias;
    plain.resid = ep.resid;
    agpu_status st = launch_gemm_ex(dev, a, b, t, batch, m, n, k, a_trans, b_trans, plain, s);
    if (st == AGPU_OK)
      st = launch_swish_mul(dev, t, t + 32, c, (uint64_t)batch * m * n / 64, 32, 64, 64, 32, s);
    pool_free(dev, tmp, s);
    return st;
  }
  const bool tiny = (uint64_t)m * n * k * batch < (1ull << 15);
  const bool vec_ep = (reinterpret_cast<uintptr_t>(ep.bias) |
                       reinterpret_cast<uintptr_t>(ep.resid)) % 16 == 0;
  if (p == AGPU_PREC_FFMA || tiny || k == 0 || !vec_ep || !gemm_tc_eligible(a, b, c, m, n, k))
    return run_ffma(dev, a, b, c, batch, m, n, k, a_trans, b_trans, ep, s);
  if (p == AGPU_PREC_TF32X3)
    return dispatch_tc<true>(dev, a, b, c, batch, m, n, k, a_trans, b_trans, ep, s);
  return dispatch_tc<false>(dev, a, b, c, batch, m, n, k, a_trans, b_trans, ep, s);
}

agpu_status launch_gemm(agpu_device* dev, const float* a, const float* b, float* c,
                        uint32_t batch, uint32_t m, uint32_t n, uint32_t k, bool a_trans,
                        bool b_trans, cudaStream_t s) {
  return launch_gemm_ex(dev, a, b, c, batch, m, n, k, a_trans, b_trans, GemmEpilogue{}, s);
}

}  // namespace agpu
