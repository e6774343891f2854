// conv2d on sm_100a: implicit GEMM on tcgen05 tensor cores, plus the SIMT
// kernels for the shapes that path does not take and for the backward ops.
//
// Replaces the reference's one-thread-per-output direct convolution
// SHADER_CONV2D (src/ops/conv.rs:173-220; API :437-480): NCHW input,
// weight [Cout, Cin/groups, kh, kw], bias (None -> zeros), stride, padding,
// dilation, groups; out = (H + 2p - d(k-1) - 1)/s + 1.
//
// Tensor-core path (groups == 1, stride 1):
//   1. stage the input NCHW -> NHWC with channels padded to Cs = ceil4(Cin)
//      (one read + one write; makes every (pixel, 32-channel) run a
//      128-byte row a TMA box can fetch);
//   2. re-lay the weight to [Cout, kh, kw, Cw] with Cw = ceil32(Cin), zeros in
//      the padding, so each (tap, 32-channel block) is one K-block;
//   3. GEMM D[pixel, oc] = sum_k A[pixel, k] W2[oc, k], k = (kh, kw, c):
//      M tile = 128 output pixels = BH rows x BW columns of one image,
//      A K-block = a 4-D TMA box {32 channels, BW, BH, 1} of the NHWC input at
//      (c0, ow0 + kw*d - p, oh0 + kh*d - p, n): out-of-range (padding)
//      coordinates read as zeros, so no bounds checks run in the mainloop;
//      N tile = BN output channels; the epilogue adds the bias and writes
//      NCHW rows (lanes = consecutive output pixels -> coalesced stores).
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "agpu_internal.cuh"
#include "ptx.cuh"
#include "umma_kernel.cuh"
#include "umma2_kernel.cuh"
#include "pair_launch.cuh"

namespace agpu {

agpu_status make_tmap_f32_3d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer,
                             uint64_t batch, uint64_t batch_stride_elems, uint32_t box_inner,
                             uint32_t box_outer, bool mn_major, bool round_tf32);
bool tma_store_enabled();

using umma::BK;
using umma::BM;

namespace {

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

template <int BN_>
struct ConvPolicy {
  static constexpr int BN = BN_;
  static constexpr bool A_MN = false, B_MN = false;
  int n_img, cout, KW, ph, pw, dh, dw, Ho, Wo, BW, BH;
  int tiles_w, tiles_h, tiles_n, cblocks, taps, cw;
  long long tiles;
  const float* bias;  // may be null
  float* out;
  // output by TMA bulk stores (store_tma) through the map {Wo, Ho, Cout, N}
  // with 32 x 1 x 32 boxes; needs BW >= 32, so that a warp's 32 tile rows
  // are 32 consecutive pixels of one output row
  bool c_tma = false;
  CUtensorMap tmap_y;

  struct Tile { int n, oh0, ow0, oc0; };

  __device__ long long num_tiles() const { return tiles; }
  __device__ int num_k() const { return taps * cblocks; }

  // oc tiles innermost: consecutive CTAs reuse the same input tile from L2.
  __device__ Tile tile(long long t) const {
    Tile r;
    r.oc0 = (int)(t % tiles_n) * BN;
    long long q = t / tiles_n;
    r.ow0 = (int)(q % tiles_w) * BW;
    q /= tiles_w;
    r.oh0 = (int)(q % tiles_h) * BH;
    r.n = (int)(q / tiles_h);
    return r;
  }

  __device__ void load(const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* sa, uint8_t* sb,
                       uint64_t* bar, const Tile& t, int kb) const {
    const int tap = kb / cblocks, cb = kb % cblocks;
    const int kh = tap / KW, kw = tap % KW;
    ptx::tma_load_4d(sa, ta, bar, cb * BK, t.ow0 + kw * dw - pw, t.oh0 + kh * dh - ph, t.n);
    // the weight map is 3-D {K, Cout, 1} (make_tmap_f32_3d): load with a 3-D box
    ptx::tma_load_3d(sb, tb, bar, tap * cw + cb * BK, t.oc0, 0);
  }

  __device__ bool col_live(const Tile& t, int col0) const { return t.oc0 + col0 < cout; }
  // no paired (SwiGLU) epilogue for convolutions
  __device__ bool paired() const { return false; }
  static constexpr bool TILE_EPILOGUE = false;  // per-chunk stores
  static constexpr int EPI_EXTRA = 0;
  __device__ void store_swiglu(const Tile&, int, int, const uint32_t (&)[32],
                               const uint32_t (&)[32], float*, int) const {}

  // Thread `lane` holds pixel (oh, ow0 + lane) of the warp's output row,
  // channels oc0 + col0 .. +31; it writes column `lane` of a [32 channels]
  // [32 pixels] block (conflict-free: one bank per lane) into one of the
  // warp's two 4 KB staging buffers, and one lane issues the bulk tensor
  // store (clipped at Wo, Ho and Cout by the map).  Buffers alternate by
  // column-chunk parity as in the GEMM's store_tma.
  __device__ void store_tma(const Tile& t, int row, int col0, const uint32_t (&v)[32],
                            float* stg, int lane) const {
    float* buf = stg + ((col0 >> 5) & 1) * 1024;
    if (lane == 0) ptx::bulk_wait_read1();
    __syncwarp();
    const int oc_lane = t.oc0 + col0 + lane;
    const float b_lane = (bias && oc_lane < cout) ? __ldg(bias + oc_lane) : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      buf[j * 32 + lane] = __uint_as_float(v[j]) + __shfl_sync(0xffffffffu, b_lane, j);
    ptx::fence_proxy_async_smem();  // the async proxy (TMA) sees the staged block
    __syncwarp();
    if (lane == 0) {
      const int r0 = row - lane;  // the warp's first tile row
      const int oh = t.oh0 + r0 / BW, ow = t.ow0 + r0 % BW;
      if (oh < Ho && ow < Wo) {
        ptx::tma_store_4d(&tmap_y, buf, ow, oh, t.oc0 + col0, t.n);
        ptx::bulk_commit();
      }
      if (((col0 >> 5) & 1) == 0 && (col0 + 32 >= BN || t.oc0 + col0 + 32 >= cout))
        ptx::bulk_wait_read0();
    }
  }

  __device__ void store(const Tile& t, int row, int col0, const uint32_t (&v)[32], float* stg,
                        int lane, bool accumulate, bool last) const {
    if (c_tma && last && !accumulate) {
      store_tma(t, row, col0, v, stg, lane);
      return;
    }
    const int oh = t.oh0 + row / BW, ow = t.ow0 + row % BW;
    if (oh >= Ho || ow >= Wo) return;
    const long long plane = (long long)Ho * Wo;
    float* o = out + ((long long)t.n * cout) * plane + (long long)oh * Wo + ow;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int oc = t.oc0 + col0 + j;
      if (oc < cout) {
        float* dst = o + (long long)oc * plane;
        if (accumulate) {
          *dst += __uint_as_float(v[j]);
        } else {
          const float bb = bias ? __ldg(bias + oc) : 0.0f;
          __stcs(dst, __uint_as_float(v[j]) + bb);
        }
      }
    }
  }
};

// CTA-pair conv tile: 256 output pixels (2*BH rows x BW columns) x BN output
// channels; CTA `rank` stages rows oh0 + rank*BH .. of the pixels and, per MMA
// sub-block s (two for BN > 256), weight rows oc0 + s*MMA_N + rank*MMA_N/2 ..
template <int BN_>
struct ConvPairPolicy : ConvPolicy<BN_> {
  using Base = ConvPolicy<BN_>;
  using Tile = typename Base::Tile;

  __device__ Tile tile(long long t) const {
    Tile r;
    r.oc0 = (int)(t % this->tiles_n) * BN_;
    long long q = t / this->tiles_n;
    r.ow0 = (int)(q % this->tiles_w) * this->BW;
    q /= this->tiles_w;
    r.oh0 = (int)(q % this->tiles_h) * 2 * this->BH;
    r.n = (int)(q / this->tiles_h);
    return r;
  }

  __device__ Tile rank_tile(const Tile& t, int rank) const {
    Tile r = t;
    r.oh0 += rank * this->BH;
    return r;
  }

  __device__ void load(const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* sa, uint8_t* sb,
                       uint32_t lbar, const Tile& t, int kb, int rank) const {
    const int tap = kb / this->cblocks, cb = kb % this->cblocks;
    const int kh = tap / this->KW, kw = tap % this->KW;
    ptx::tma_load_4d_pair(sa, ta, lbar, cb * BK, t.ow0 + kw * this->dw - this->pw,
                          t.oh0 + rank * this->BH + kh * this->dh - this->ph, t.n);
    constexpr int HALF = umma::PairCfg<BN_>::MMA_N / 2;
#pragma unroll
    for (int sub = 0; sub < umma::PairCfg<BN_>::NMMA; ++sub)
      ptx::tma_load_3d_pair(sb + sub * HALF * 128, tb, lbar, tap * this->cw + cb * BK,
                            t.oc0 + sub * 2 * HALF + rank * HALF, 0);
  }
};

// Weight gradient (conv2d_grad_weight, stride 1) as implicit GEMMs, one per
// kernel tap: dW_tap[oc, ic] = sum over pixels of gy[oc, pix] * x_tap[pix, ic]
// with x_tap the input shifted by the tap.  A = gy read in place (K-major:
// 32 consecutive output pixels of one row per K-block), B = the NHWC-staged
// input (MN-major: 32 channels x the same 32 pixels, shifted by the tap, the
// halo zero-filled by TMA).  The pixel sum (N*Ho*Wo long) is split into
// `segs` K ranges so the few output tiles fill the GPU; each range writes its
// partial tile to a workspace [seg][Cout][tap][Cin] and a second kernel sums
// the ranges in order into dW [Cout][Cin][KH][KW].
template <int BN_>
struct WgradPolicy {
  static constexpr int BN = BN_;
  static constexpr bool A_MN = false, B_MN = true;
  int cout, cin, kw, ph, pw, dh, dw, wo;
  int bpr, bpi, n_img;           // K-blocks per output row / per image, images
  int tiles_m, tiles_n, taps, segs, kper;
  long long tiles;
  float* ws;                     // [segs][cout][taps][cin]

  struct Tile { int oc0, tap, ic0, seg; };

  __device__ long long num_tiles() const { return tiles; }
  __device__ int num_k() const { return kper; }

  // output-channel tiles innermost: consecutive CTAs share the shifted input
  __device__ Tile tile(long long t) const {
    Tile r;
    r.oc0 = (int)(t % tiles_m) * BM;
    long long q = t / tiles_m;
    r.ic0 = (int)(q % tiles_n) * BN;
    q /= tiles_n;
    r.tap = (int)(q % taps);
    r.seg = (int)(q / taps);
    return r;
  }

  __device__ void load(const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* sa, uint8_t* sb,
                       uint64_t* bar, const Tile& t, int kb) const {
    // blocks past the last image read out of range: TMA fills zeros
    const long long g = (long long)t.seg * kper + kb;
    const int img = (int)(g / bpi), rem = (int)(g % bpi);
    const int oh = rem / bpr, ow0 = (rem % bpr) * 32;
    ptx::tma_load_3d(sa, ta, bar, oh * wo + ow0, t.oc0, img);
    const int kh_i = t.tap / kw, kw_i = t.tap % kw;
#pragma unroll
    for (int j = 0; j < BN / 32; ++j)
      ptx::tma_load_4d(sb + j * BK * 128, tb, bar, t.ic0 + 32 * j, ow0 + kw_i * dw - pw,
                       oh + kh_i * dh - ph, img);
  }

  __device__ bool col_live(const Tile& t, int col0) const { return t.ic0 + col0 < cin; }

  __device__ void store(const Tile& t, int row, int col0, const uint32_t (&v)[32], float*, int,
                        bool accumulate, bool) const {
    const int oc = t.oc0 + row;
    if (oc >= cout) return;
    float* dst = ws + (((long long)t.seg * cout + oc) * taps + t.tap) * cin + t.ic0 + col0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (t.ic0 + col0 + j < cin) {
        if (accumulate) dst[j] += __uint_as_float(v[j]);
        else dst[j] = __uint_as_float(v[j]);
      }
    }
  }
};

// dW[oc][ic][kh][kw] = sum over seg of ws[seg][oc][tap][ic], in seg order.
__global__ void wgrad_reduce_kernel(const float* __restrict__ ws, float* __restrict__ gw, int segs,
                                    int cout, int cin, int taps) {
  const long long total = (long long)cout * cin * taps;
  const long long plane = total;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int tap = (int)(i % taps);
    const long long r = i / taps;
    const int ic = (int)(r % cin);
    const int oc = (int)(r / cin);
    const long long src = ((long long)oc * taps + tap) * cin + ic;
    float sum = 0.f;
    for (int sg = 0; sg < segs; ++sg) sum += __ldg(ws + sg * plane + src);
    gw[i] = sum;
  }
}

// Staging for the implicit-GEMM convolutions, in one launch:
//   blocks [0, wblocks): W [Cout, Cin, taps] -> W2 [Cout, taps, Cw]
//     (channels >= Cin zero), a grid-stride loop over W2 (coalesced writes);
//   the rest: NCHW [N, C, HW] -> NHWC [N, HW, Cs] (channels >= C zero), one
//     32-channel x 128-pixel tile per CTA: 16 loads in flight per thread
//     (each warp instruction reads 128 contiguous bytes of one channel), a
//     shared-memory transpose with row pitch 129 (conflict-free both ways),
//     float4 stores (8 lanes write one pixel's 32 channels, 128 B).
// The weight blocks come first in the grid, so they overlap the transpose.
constexpr int kStageP = 128, kStageC = 32;

__global__ void __launch_bounds__(256) conv_stage_kernel(
    const float* __restrict__ x, float* __restrict__ xs, int C, int HW, int Cs, int ptiles,
    int ctiles, const float* __restrict__ w, float* __restrict__ w2, int cin, int taps, int Cw,
    long long w2_elems, int wblocks) {
  __shared__ float tile[kStageC][kStageP + 1];
  if ((int)blockIdx.x < wblocks) {
    for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < w2_elems;
         i += (long long)wblocks * 256) {
      const int c = (int)(i % Cw);
      const long long r = i / Cw;
      const int t = (int)(r % taps);
      const long long oc = r / taps;
      w2[i] = c < cin ? __ldg(w + (oc * cin + c) * taps + t) : 0.0f;
    }
    return;
  }
  long long b = (long long)blockIdx.x - wblocks;
  const int pt = (int)(b % ptiles);
  b /= ptiles;
  const int ct = (int)(b % ctiles);
  const long long n = b / ctiles;
  const int p0 = pt * kStageP, c0 = ct * kStageC;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float* xn = x + n * C * HW;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int cl = warp + 8 * k, c = c0 + cl;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int p = p0 + lane + 32 * i;
      tile[cl][lane + 32 * i] = (c < C && p < HW) ? __ldcs(xn + (long long)c * HW + p) : 0.0f;
    }
  }
  __syncthreads();
  float* yn = xs + n * HW * Cs;
  const int c4 = lane % 8;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int pl = warp * 16 + k * 4 + lane / 8;
    const int p = p0 + pl, c = c0 + 4 * c4;
    if (p < HW && c < Cs)
      *reinterpret_cast<float4*>(yn + (long long)p * Cs + c) =
          make_float4(tile[4 * c4][pl], tile[4 * c4 + 1][pl], tile[4 * c4 + 2][pl],
                      tile[4 * c4 + 3][pl]);
  }
}

// Enqueue conv_stage_kernel: x (NCHW, C channels) -> xs (NHWC, Cs channels);
// with w != nullptr also W -> W2 as above.
void launch_conv_stage(const agpu_device* dev, const float* x, float* xs, int n, int C, int HW,
                       int Cs, const float* w, float* w2, int cout, int cin, int taps, int Cw,
                       cudaStream_t s) {
  const int ptiles = (int)ceil_div(HW, kStageP), ctiles = (int)ceil_div(Cs, kStageC);
  const long long w2_elems = w ? (long long)cout * taps * Cw : 0;
  const int wblocks = (int)std::min<long long>(ceil_div(w2_elems, 256 * 8), 4LL * dev->sm_count);
  const long long blocks = wblocks + (long long)n * ctiles * ptiles;
  conv_stage_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, xs, C, HW, Cs, ptiles, ctiles, w, w2, cin,
                                                     taps, Cw, w2_elems, wblocks);
}

// conv_transpose2d weight W [Cin, Cout, KH, KW] -> the equivalent conv2d
// weight W' [Cout, Cin, KH, KW] with both taps reversed:
// W'[o, i, a, b] = W[i, o, KH-1-a, KW-1-b].
__global__ void weight_flip_kernel(const float* __restrict__ w, float* __restrict__ w2, int cin,
                                   int cout, int kh, int kw) {
  const long long total = (long long)cin * cout * kh * kw;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i % kw);
    long long r = i / kw;
    const int a = (int)(r % kh);
    r /= kh;
    const int ic = (int)(r % cin);
    const int oc = (int)(r / cin);
    w2[i] = w[(((long long)ic * cout + oc) * kh + (kh - 1 - a)) * kw + (kw - 1 - b)];
  }
}

// Direct convolution, one thread per output (exact fp32; any stride,
// dilation, groups) -- same arithmetic order as the reference shader.
__global__ void conv2d_direct_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                     const float* __restrict__ bias, float* __restrict__ y,
                                     int N, int Cin, int H, int W, int Cout, int KH, int KW,
                                     int sh, int sw, int ph, int pw, int dh, int dw, int groups,
                                     int Ho, int Wo) {
  const long long total = (long long)N * Cout * Ho * Wo;
  const int gin = Cin / groups, gout = Cout / groups;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int ow = (int)(idx % Wo);
    const int oh = (int)((idx / Wo) % Ho);
    const int oc = (int)((idx / ((long long)Wo * Ho)) % Cout);
    const int n = (int)(idx / ((long long)Wo * Ho * Cout));
    const int g = oc / gout;
    float sum = bias ? bias[oc] : 0.0f;
    for (int ic = 0; ic < gin; ++ic)
      for (int kh = 0; kh < KH; ++kh) {
        const int ih = oh * sh + kh * dh - ph;
        if (ih < 0 || ih >= H) continue;
        for (int kw = 0; kw < KW; ++kw) {
          const int iw = ow * sw + kw * dw - pw;
          if (iw < 0 || iw >= W) continue;
          sum = fmaf(x[(((long long)n * Cin + g * gin + ic) * H + ih) * W + iw],
                     w[(((long long)oc * gin + ic) * KH + kh) * KW + kw], sum);
        }
      }
    y[idx] = sum;
  }
}

// Transposed convolution (SHADER_CONV_TRANSPOSE2D, src/ops/conv.rs:245-296):
// weight [Cin, Cout/groups, kh, kw].
__global__ void conv_transpose2d_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                        const float* __restrict__ bias, float* __restrict__ y,
                                        int N, int Cin, int H, int W, int Cout, int KH, int KW,
                                        int sh, int sw, int ph, int pw, int dh, int dw,
                                        int groups, int Ho, int Wo) {
  const long long total = (long long)N * Cout * Ho * Wo;
  const int gin = Cin / groups, gout = Cout / groups;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int ow = (int)(idx % Wo);
    const int oh = (int)((idx / Wo) % Ho);
    const int oc = (int)((idx / ((long long)Wo * Ho)) % Cout);
    const int n = (int)(idx / ((long long)Wo * Ho * Cout));
    const int g = oc / gout, ocl = oc % gout;
    float sum = bias ? bias[oc] : 0.0f;
    for (int ic = 0; ic < gin; ++ic)
      for (int kh = 0; kh < KH; ++kh) {
        const int ohf = oh + ph - kh * dh;
        if (ohf < 0 || ohf % sh) continue;
        const int ih = ohf / sh;
        if (ih >= H) continue;
        for (int kw = 0; kw < KW; ++kw) {
          const int owf = ow + pw - kw * dw;
          if (owf < 0 || owf % sw) continue;
          const int iw = owf / sw;
          if (iw >= W) continue;
          sum = fmaf(x[(((long long)n * Cin + g * gin + ic) * H + ih) * W + iw],
                     w[(((long long)(g * gin + ic) * gout + ocl) * KH + kh) * KW + kw], sum);
        }
      }
    y[idx] = sum;
  }
}

// grad_weight (SHADER_CONV2D_GRAD_WEIGHT, src/ops/conv.rs:337-385): one CTA
// per weight element, the N*Ho*Wo reduction split over 256 threads.
__global__ void __launch_bounds__(256) conv2d_grad_weight_kernel(
    const float* __restrict__ x, const float* __restrict__ gy, float* __restrict__ gw, int N,
    int Cin, int H, int W, int Cout, int Ho, int Wo, int KH, int KW, int sh, int sw, int ph,
    int pw, int dh, int dw, int groups) {
  __shared__ float red[8];
  const int gin = Cin / groups, gout = Cout / groups;
  const long long idx = blockIdx.x;
  const int kw = (int)(idx % KW);
  const int kh = (int)((idx / KW) % KH);
  const int ic = (int)((idx / ((long long)KW * KH)) % gin);
  const int oc = (int)(idx / ((long long)KW * KH * gin));
  const int g = oc / gout;
  const long long P = (long long)N * Ho * Wo;
  float sum = 0.f;
  for (long long p = threadIdx.x; p < P; p += blockDim.x) {
    const int ow = (int)(p % Wo);
    const int oh = (int)((p / Wo) % Ho);
    const int n = (int)(p / ((long long)Wo * Ho));
    const int ih = oh * sh + kh * dh - ph, iw = ow * sw + kw * dw - pw;
    if (ih < 0 || iw < 0 || ih >= H || iw >= W) continue;
    sum = fmaf(gy[(((long long)n * Cout + oc) * Ho + oh) * Wo + ow],
               x[(((long long)n * Cin + g * gin + ic) * H + ih) * W + iw], sum);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += red[i];
    gw[idx] = s;
  }
}

// grad_bias (SHADER_CONV2D_GRAD_BIAS, src/ops/conv.rs:390-410): one CTA per channel.
__global__ void __launch_bounds__(256) conv2d_grad_bias_kernel(const float* __restrict__ gy,
                                                               float* __restrict__ gb, int N,
                                                               int Cout, long long HW) {
  __shared__ float red[8];
  const int oc = blockIdx.x;
  float sum = 0.f;
  for (int n = 0; n < N; ++n) {
    const float* p = gy + ((long long)n * Cout + oc) * HW;
    for (long long i = threadIdx.x; i < HW; i += blockDim.x) sum += p[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += red[i];
    gb[oc] = s;
  }
}

unsigned grid_for(const agpu_device* dev, long long work) {
  const long long want = (work + 255) / 256;
  return (unsigned)std::max<long long>(1, std::min<long long>(want, (long long)dev->sm_count * 16));
}

// The implicit-GEMM conv of images [0, p.n) of a staged NHWC input `xs` and
// tap-major weights `w2` (both from conv_stage_kernel), output NCHW `y`.
template <int BN, bool X3, bool PAIR>
agpu_status conv_tc_staged(agpu_device* dev, const ConvParams& p, const float* xs,
                           const float* w2, const float* bias, float* y, cudaStream_t s) {
  using P = typename std::conditional<PAIR, ConvPairPolicy<BN>, ConvPolicy<BN>>::type;
  const int Cs = (p.cin + 3) / 4 * 4;
  const int Cw = (p.cin + BK - 1) / BK * BK;
  agpu_status st = AGPU_OK;
  P pol;
  pol.n_img = p.n; pol.cout = p.cout; pol.KW = p.kw;
  pol.ph = p.ph; pol.pw = p.pw; pol.dh = p.dh; pol.dw = p.dw;
  pol.Ho = p.ho; pol.Wo = p.wo;
  int bw = 1;
  while (bw < p.wo && bw < 128) bw *= 2;
  pol.BW = bw;
  pol.BH = 128 / bw;
  pol.tiles_w = (int)ceil_div(p.wo, pol.BW);
  pol.tiles_h = (int)ceil_div(p.ho, (PAIR ? 2 : 1) * pol.BH);
  pol.tiles_n = (int)ceil_div(p.cout, BN);
  pol.cblocks = Cw / BK;
  pol.taps = p.kh * p.kw;
  pol.cw = Cw;
  pol.tiles = (long long)p.n * pol.tiles_h * pol.tiles_w * pol.tiles_n;
  pol.bias = bias;
  pol.out = y;

  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(AGPU_ERR_CUDA, "no cuTensorMapEncodeTiled");
  pol.c_tma = false;
  if (tma_store_enabled() && pol.BW >= 32 && p.wo % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    cuuint64_t dims[4] = {(cuuint64_t)p.wo, (cuuint64_t)p.ho, (cuuint64_t)p.cout,
                          (cuuint64_t)p.n};
    cuuint64_t strides[3] = {(cuuint64_t)p.wo * 4, (cuuint64_t)p.ho * p.wo * 4,
                             (cuuint64_t)p.cout * p.ho * p.wo * 4};
    cuuint32_t box[4] = {32, 1, 32, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc(&pol.tmap_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(AGPU_ERR_CUDA, "conv2d: output tensor map encode failed (%d)", (int)r);
    pol.c_tma = true;
  }
  CUtensorMap ta, tb;
  {
    cuuint64_t dims[4] = {(cuuint64_t)Cs, (cuuint64_t)p.w, (cuuint64_t)p.h, (cuuint64_t)p.n};
    cuuint64_t strides[3] = {(cuuint64_t)Cs * 4, (cuuint64_t)p.w * Cs * 4,
                             (cuuint64_t)p.h * p.w * Cs * 4};
    cuuint32_t box[4] = {BK, (cuuint32_t)pol.BW, (cuuint32_t)pol.BH, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    // TF32 mode: the TMA unit rounds to tf32 (nearest-even); 3xTF32 needs raw fp32
    CUresult r = enc(&ta, X3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_TFLOAT32,
                     4, const_cast<float*>(xs), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(AGPU_ERR_CUDA, "conv2d: input tensor map encode failed (%d)", (int)r);
  }
  AGPU_TRY(make_tmap_f32_3d(&tb, w2, (uint64_t)p.kh * p.kw * Cw, p.cout, 1,
                            (uint64_t)p.kh * p.kw * Cw * p.cout, BK,
                            PAIR ? umma::PairCfg<BN>::MMA_N / 2 : BN, false, !X3));
  if constexpr (PAIR) {
    st = launch_pair(dev, ta, tb, pol, pol.tiles, s,
                     "conv2d_tf32 (umma_tf32_pair_kernel)");
  } else {
    using Cfg = umma::Cfg<BN, X3>;
    auto kern = umma::umma_tf32_kernel<P, X3>;
    cudaError_t e = set_smem_once<umma::umma_tf32_kernel<P, X3>>(dev, Cfg::SMEM);
    if (e != cudaSuccess) return cuda_status(e, "conv attr");
    const long long grid = std::min<long long>(pol.tiles, dev->sm_count);
    kern<<<(unsigned)grid, Cfg::THREADS, Cfg::SMEM, s>>>(ta, tb, pol, dev->d_status);
    st = after_launch(dev, "conv2d_tf32 (umma_tf32_kernel)");
  }
  return st;
}

// Stage, then convolve.  With the CTA-pair kernel and >= 4 images the batch
// runs as two halves: the weights and the first half's input are staged on
// `s`; the second half's input is staged on the device's auxiliary stream
// while the first half's conv runs (the staging kernel's CTAs fit beside the
// conv's on each SM), and its conv fills the SMs the first half's last wave
// leaves idle; `s` then waits for the auxiliary stream.
// AGPU_CONV_OVERLAP=0 keeps one stage and one conv launch.
template <int BN, bool X3, bool PAIR>
agpu_status run_conv_tc(agpu_device* dev, const ConvParams& p, const float* x, const float* w,
                        const float* bias, float* y, cudaStream_t s, const GnEpilogue* gn) {
  static_assert(!(X3 && PAIR), "the CTA-pair kernel is TF32 only");
  // the fused group norm (+ swish) of images [0, n) of y, in place, on `st`
  auto norm = [&](const ConvParams& q, float* yq, cudaStream_t st) {
    return gn ? launch_group_norm(dev, yq, gn->gamma, gn->beta, yq, q.n, q.cout, q.ho * q.wo,
                                  gn->groups, gn->eps, gn->swish, st)
              : AGPU_OK;
  };
  const int Cs = (p.cin + 3) / 4 * 4;
  const int Cw = (p.cin + BK - 1) / BK * BK;
  const uint64_t img_elems = (uint64_t)p.h * p.w * Cs;
  const uint64_t xs_elems = (uint64_t)p.n * img_elems;
  const uint64_t w2_elems = (uint64_t)p.cout * p.kh * p.kw * Cw;
  void* scratch = nullptr;
  AGPU_TRY(pool_alloc(dev, (xs_elems + w2_elems) * sizeof(float) + 256, &scratch, s));
  float* xs = static_cast<float*>(scratch);
  float* w2 = xs + (xs_elems + 63) / 64 * 64;
  static const bool overlap_ok = [] {
    const char* e = getenv("AGPU_CONV_OVERLAP");
    return !(e && e[0] == '0');
  }();
  cudaStream_t s2 = (PAIR && overlap_ok && p.n >= 4) ? aux_stream(dev) : nullptr;
  const int na = s2 ? p.n / 2 : p.n;
  launch_conv_stage(dev, x, xs, na, p.cin, p.h * p.w, Cs, w, w2, p.cout, p.cin, p.kh * p.kw, Cw,
                    s);
  agpu_status st = after_launch(dev, "conv_stage_kernel");
  if (st != AGPU_OK) { pool_free(dev, scratch, s); return st; }
  if (!s2) {
    st = conv_tc_staged<BN, X3, PAIR>(dev, p, xs, w2, bias, y, s);
    pool_free(dev, scratch, s);
    if (st == AGPU_OK) st = norm(p, y, s);
    return st;
  }
  ConvParams pa = p, pb = p;
  pa.n = na;
  pb.n = p.n - na;
  const uint64_t x_img = (uint64_t)p.cin * p.h * p.w, y_img = (uint64_t)p.cout * p.ho * p.wo;
  cudaEvent_t forked = nullptr, joined = nullptr;
  if (cudaEventCreateWithFlags(&forked, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&joined, cudaEventDisableTiming) != cudaSuccess) {
    if (forked) cudaEventDestroy(forked);
    pool_free(dev, scratch, s);
    return cuda_status(cudaGetLastError(), "conv2d: event create");
  }
  cudaError_t e = cudaEventRecord(forked, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s2, forked, 0);
  if (e == cudaSuccess) {
    launch_conv_stage(dev, x + na * x_img, xs + na * img_elems, pb.n, p.cin, p.h * p.w, Cs,
                      nullptr, nullptr, 0, 0, 0, 0, s2);
    st = after_launch(dev, "conv_stage_kernel");
    if (st == AGPU_OK) st = conv_tc_staged<BN, X3, PAIR>(dev, pa, xs, w2, bias, y, s);
    if (st == AGPU_OK)
      st = conv_tc_staged<BN, X3, PAIR>(dev, pb, xs + na * img_elems, w2, bias, y + na * y_img,
                                        s2);
    // a fused group norm of the first half runs beside the second half's conv
    if (st == AGPU_OK) st = norm(pa, y, s);
    if (st == AGPU_OK) st = norm(pb, y + na * y_img, s2);
    // join in every case, so that the scratch is freed after both streams
    e = cudaEventRecord(joined, s2);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, joined, 0);
  }
  cudaEventDestroy(forked);
  cudaEventDestroy(joined);
  pool_free(dev, scratch, s);
  if (e != cudaSuccess && st == AGPU_OK) st = cuda_status(e, "conv2d: stream fork/join");
  return st;
}

// BN: output-channel tile minimising padding (N of the MMA, multiple of 32).
template <bool X3>
agpu_status dispatch_conv_tc(agpu_device* dev, const ConvParams& p, const float* x,
                             const float* w, const float* bias, float* y, cudaStream_t s,
                             const GnEpilogue* gn = nullptr) {
  // TF32 convs with at least two 128-pixel tiles per image run on CTA pairs;
  // output-channel counts that are multiples of 320 take 256 x 320 tiles (two
  // MMAs of N 160: fewer TMA bytes per FLOP than 256 x 160).
  // AGPU_CONV_WIDE=0 keeps them on 256 x 160 tiles.
  constexpr bool PAIR = !X3;
  static const bool wide = [] {
    const char* e = getenv("AGPU_CONV_WIDE");
    return !(e && e[0] == '0');
  }();
  if constexpr (PAIR) {
    if ((long long)p.ho * p.wo >= 256) {
      if (wide && p.cout % 320 == 0) return run_conv_tc<320, X3, true>(dev, p, x, w, bias, y, s, gn);
      if (p.cout % 160 == 0 && p.cout % 256 != 0)
        return run_conv_tc<160, X3, true>(dev, p, x, w, bias, y, s, gn);
      if (p.cout >= 256) return run_conv_tc<256, X3, true>(dev, p, x, w, bias, y, s, gn);
      if (p.cout > 96) return run_conv_tc<128, X3, true>(dev, p, x, w, bias, y, s, gn);
      return run_conv_tc<64, X3, true>(dev, p, x, w, bias, y, s, gn);
    }
  }
  if (p.cout % 160 == 0 && p.cout % 256 != 0) return run_conv_tc<160, X3, false>(dev, p, x, w, bias, y, s, gn);
  if (p.cout >= 256) return run_conv_tc<256, X3, false>(dev, p, x, w, bias, y, s, gn);
  if (p.cout > 96) return run_conv_tc<128, X3, false>(dev, p, x, w, bias, y, s, gn);
  return run_conv_tc<64, X3, false>(dev, p, x, w, bias, y, s, gn);
}

template <int BN, bool X3>
agpu_status run_wgrad_tc(agpu_device* dev, const ConvParams& p, const float* x, const float* gy,
                         float* gw, cudaStream_t s) {
  using P = WgradPolicy<BN>;
  using Cfg = umma::Cfg<BN, X3>;
  P pol;
  pol.cout = p.cout; pol.cin = p.cin; pol.kw = p.kw;
  pol.ph = p.ph; pol.pw = p.pw; pol.dh = p.dh; pol.dw = p.dw; pol.wo = p.wo;
  pol.bpr = p.wo / 32;
  pol.bpi = p.ho * pol.bpr;
  pol.n_img = p.n;
  pol.tiles_m = (int)ceil_div(p.cout, BM);
  pol.tiles_n = (int)ceil_div(p.cin, BN);
  pol.taps = p.kh * p.kw;
  // K split: the fewest ranges (each at least 32 K-blocks) whose tiles fill
  // the SMs' waves to 90 %; every range adds a partial weight-sized tensor of
  // workspace traffic.
  const long long base = (long long)pol.tiles_m * pol.tiles_n * pol.taps;
  const long long kblocks = (long long)p.n * pol.bpi;
  int best = 1;
  double best_eff = 0.0;
  for (int sg = 1; sg <= 64; ++sg) {
    if (sg > 1 && kblocks / sg < 32) break;
    const long long units = base * sg;
    const long long waves = (units + dev->sm_count - 1) / dev->sm_count;
    const double eff = (double)units / (double)(waves * dev->sm_count);
    if (eff > best_eff + 1e-9) { best_eff = eff; best = sg; }
    if (eff >= 0.9) break;
  }
  pol.segs = best;
  pol.kper = (int)ceil_div(kblocks, best);
  pol.tiles = base * best;
  const int Cs = (p.cin + 3) / 4 * 4;
  const uint64_t xs_elems = (uint64_t)p.n * p.h * p.w * Cs;
  const uint64_t ws_elems = (uint64_t)best * p.cout * pol.taps * p.cin;
  void* scratch = nullptr;
  AGPU_TRY(pool_alloc(dev, (xs_elems + ws_elems) * sizeof(float) + 256, &scratch, s));
  float* xs = static_cast<float*>(scratch);
  pol.ws = xs + (xs_elems + 63) / 64 * 64;
  launch_conv_stage(dev, x, xs, p.n, p.cin, p.h * p.w, Cs, nullptr, nullptr, 0, 0, 0, 0, s);
  agpu_status st = after_launch(dev, "conv_stage_kernel");
  CUtensorMap ta, tb;
  if (st == AGPU_OK)
    st = make_tmap_f32_3d(&ta, gy, (uint64_t)p.ho * p.wo, p.cout, p.n,
                          (uint64_t)p.cout * p.ho * p.wo, 32, BM, false, !X3);
  if (st == AGPU_OK) {
    EncodeTiledFn enc = encode_fn();
    cuuint64_t dims[4] = {(cuuint64_t)Cs, (cuuint64_t)p.w, (cuuint64_t)p.h, (cuuint64_t)p.n};
    cuuint64_t strides[3] = {(cuuint64_t)Cs * 4, (cuuint64_t)p.w * Cs * 4,
                             (cuuint64_t)p.h * p.w * Cs * 4};
    cuuint32_t box[4] = {32, 32, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = enc ? enc(&tb, X3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : CU_TENSOR_MAP_DATA_TYPE_TFLOAT32,
                           4, xs, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)
                     : CUDA_ERROR_NOT_FOUND;
    if (r != CUDA_SUCCESS) st = fail(AGPU_ERR_CUDA, "conv2d_grad_weight: input map (%d)", (int)r);
  }
  if (st == AGPU_OK) {
    auto kern = umma::umma_tf32_kernel<P, X3>;
    cudaError_t e = set_smem_once<umma::umma_tf32_kernel<P, X3>>(dev, Cfg::SMEM);
    if (e != cudaSuccess) {
      st = cuda_status(e, "wgrad attr");
    } else {
      const long long grid = std::min<long long>(pol.tiles, dev->sm_count);
      kern<<<(unsigned)grid, Cfg::THREADS, Cfg::SMEM, s>>>(ta, tb, pol, dev->d_status);
      st = after_launch(dev, "conv2d_grad_weight (umma_tf32_kernel)");
    }
  }
  if (st == AGPU_OK) {
    const long long total = (long long)p.cout * p.cin * pol.taps;
    wgrad_reduce_kernel<<<grid_for(dev, total), 256, 0, s>>>(pol.ws, gw, best, p.cout, p.cin,
                                                             pol.taps);
    st = after_launch(dev, "wgrad_reduce_kernel");
  }
  pool_free(dev, scratch, s);
  return st;
}

}  // namespace

bool conv_tc_eligible(const ConvParams& p) {
  return p.groups == 1 && p.sh == 1 && p.sw == 1 && p.cout >= 16 &&
         (long long)p.n * p.cout * p.ho * p.wo * p.cin * p.kh * p.kw >= (1LL << 22) &&
         p.n <= 65535;
}

agpu_status launch_conv2d(agpu_device* dev, const ConvParams& p, const float* x, const float* w,
                          const float* bias, float* y, cudaStream_t s) {
  const long long total = (long long)p.n * p.cout * p.ho * p.wo;
  if (total == 0) return AGPU_OK;
  const agpu_precision prec = effective_precision(dev);
  if (prec != AGPU_PREC_FFMA && conv_tc_eligible(p)) {
    if (prec == AGPU_PREC_TF32X3) return dispatch_conv_tc<true>(dev, p, x, w, bias, y, s);
    return dispatch_conv_tc<false>(dev, p, x, w, bias, y, s);
  }
  conv2d_direct_kernel<<<grid_for(dev, total), 256, 0, s>>>(
      x, w, bias, y, p.n, p.cin, p.h, p.w, p.cout, p.kh, p.kw, p.sh, p.sw, p.ph, p.pw, p.dh, p.dw,
      p.groups, p.ho, p.wo);
  return after_launch(dev, "conv2d_direct_kernel");
}

agpu_status launch_conv2d_gn(agpu_device* dev, const ConvParams& p, const float* x,
                             const float* w, const float* bias, float* y, const GnEpilogue& gn,
                             cudaStream_t s) {
  const long long total = (long long)p.n * p.cout * p.ho * p.wo;
  if (total == 0) return AGPU_OK;
  const agpu_precision prec = effective_precision(dev);
  if (prec != AGPU_PREC_FFMA && conv_tc_eligible(p)) {
    if (prec == AGPU_PREC_TF32X3)
      return dispatch_conv_tc<true>(dev, p, x, w, bias, y, s, &gn);
    return dispatch_conv_tc<false>(dev, p, x, w, bias, y, s, &gn);
  }
  AGPU_TRY(launch_conv2d(dev, p, x, w, bias, y, s));
  return launch_group_norm(dev, y, gn.gamma, gn.beta, y, p.n, p.cout, p.ho * p.wo, gn.groups,
                           gn.eps, gn.swish, s);
}

agpu_status launch_conv_transpose2d(agpu_device* dev, const ConvParams& p, const float* x,
                                    const float* w, const float* bias, float* y,
                                    cudaStream_t s) {
  const long long total = (long long)p.n * p.cout * p.ho * p.wo;
  if (total == 0) return AGPU_OK;
  // Stride 1, one group, no output padding: conv_transpose2d(x, W, pad p) is
  // conv2d(x, W', pad d*(k-1) - p) with W' the channel-swapped, tap-reversed
  // weight (src/ops/conv.rs:277-290: oh = ih - p + kh*d, so ih = oh + p - kh*d
  // = oh - p' + (k-1-kh)*d), which runs on the tensor-core implicit GEMM.
  // The exact fp32 mode keeps the direct kernel (the reference's sum order).
  const int php = p.dh * (p.kh - 1) - p.ph, pwp = p.dw * (p.kw - 1) - p.pw;
  ConvParams q{p.n, p.cin, p.h, p.w, p.cout, p.kh, p.kw, 1, 1, php, pwp, p.dh, p.dw, 1, p.ho,
               p.wo};
  if (effective_precision(dev) != AGPU_PREC_FFMA && p.sh == 1 && p.sw == 1 && p.groups == 1 &&
      php >= 0 &&
      pwp >= 0 && p.ho == p.h + p.dh * (p.kh - 1) - 2 * p.ph &&
      p.wo == p.w + p.dw * (p.kw - 1) - 2 * p.pw && conv_tc_eligible(q)) {
    const long long wn = (long long)p.cin * p.cout * p.kh * p.kw;
    void* buf = nullptr;
    AGPU_TRY(pool_alloc(dev, (uint64_t)wn * sizeof(float), &buf, s));
    float* w2 = static_cast<float*>(buf);
    weight_flip_kernel<<<grid_for(dev, wn), 256, 0, s>>>(w, w2, p.cin, p.cout, p.kh, p.kw);
    agpu_status st = after_launch(dev, "weight_flip_kernel");
    if (st == AGPU_OK) st = launch_conv2d(dev, q, x, w2, bias, y, s);
    pool_free(dev, buf, s);
    return st;
  }
  conv_transpose2d_kernel<<<grid_for(dev, total), 256, 0, s>>>(
      x, w, bias, y, p.n, p.cin, p.h, p.w, p.cout, p.kh, p.kw, p.sh, p.sw, p.ph, p.pw, p.dh, p.dw,
      p.groups, p.ho, p.wo);
  return after_launch(dev, "conv_transpose2d_kernel");
}

agpu_status launch_conv2d_grad_weight(agpu_device* dev, const ConvParams& p, const float* x,
                                      const float* gy, float* gw, cudaStream_t s) {
  const long long nw = (long long)p.cout * (p.cin / p.groups) * p.kh * p.kw;
  if (nw == 0) return AGPU_OK;
  // tensor cores: stride 1, one group, output rows in whole 32-pixel blocks
  const agpu_precision prec = effective_precision(dev);
  if (prec != AGPU_PREC_FFMA && p.groups == 1 && p.sh == 1 && p.sw == 1 &&
      p.wo % 32 == 0 && p.n > 0 && p.n <= 65535 &&
      (long long)p.n * p.cout * p.ho * p.wo * p.cin * p.kh * p.kw >= (1LL << 22)) {
    if (prec == AGPU_PREC_TF32X3) {
      if (p.cin > 128) return run_wgrad_tc<256, true>(dev, p, x, gy, gw, s);
      return run_wgrad_tc<128, true>(dev, p, x, gy, gw, s);
    }
    if (p.cin % 160 == 0 && p.cin % 256 != 0) return run_wgrad_tc<160, false>(dev, p, x, gy, gw, s);
    if (p.cin > 128) return run_wgrad_tc<256, false>(dev, p, x, gy, gw, s);
    return run_wgrad_tc<128, false>(dev, p, x, gy, gw, s);
  }
  if (nw > 0x7fffffffLL) return fail(AGPU_ERR_UNSUPPORTED, "conv2d_grad_weight: too many weights");
  conv2d_grad_weight_kernel<<<(unsigned)nw, 256, 0, s>>>(x, gy, gw, p.n, p.cin, p.h, p.w, p.cout,
                                                         p.ho, p.wo, p.kh, p.kw, p.sh, p.sw, p.ph,
                                                         p.pw, p.dh, p.dw, p.groups);
  return after_launch(dev, "conv2d_grad_weight_kernel");
}

agpu_status launch_conv2d_grad_bias(agpu_device* dev, const float* gy, float* gb, int n, int cout,
                                    long long hw, cudaStream_t s) {
  if (cout == 0) return AGPU_OK;
  conv2d_grad_bias_kernel<<<(unsigned)cout, 256, 0, s>>>(gy, gb, n, cout, hw);
  return after_launch(dev, "conv2d_grad_bias_kernel");
}

}  // namespace agpu
