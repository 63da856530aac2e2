// Page-level kernels of the end-to-end det+rec path on B200:
//
//   stem_kernel        det preprocessing of 960x960 pages (scale 1, so the
//                      reference's bilinear resize is the identity) fused with
//                      the backbone stem, a 3x3 stride-2 conv 3->32 + folded BN
//                      + hardswish, written fp16 NHWC for the DW+PW blocks.
//                      Normalisation as preprocess_kernels.cu:169-177
//                      ((v * 1/255 - mean_c) * inv_std_c, channel-positional).
//   ink_kernel         the probability map the DB stage consumes in the
//                      synthetic end-to-end run (no trained DB head exists):
//                      sigmoid(k * (dilated ink - 0.5)) at full resolution.
//   head_kernel        the backbone's 1x1 256->1 head + sigmoid (DB logit map at
//                      the backbone's resolution), computed and written.
//   roi_warp_kernel    batch_roi_warp_kernel (src/kernels/preprocess_kernels.cu:211-344):
//                      inverse-perspective bilinear crop, BGR->RGB, rec
//                      normalisation, zero beyond the crop width; fp16 out.
//
// Default nvcc contraction (as the reference kernels are built): the ROI warp
// keeps batch_roi_warp_kernel's expressions, so it rounds the same way.
#include "tocr_common.cuh"
#include "tc_ptx.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace tocr {
namespace {

// ---------------------------------------------------------------- stem -------
constexpr int kStemCo = 32;

// The det normalisation (b / 255 - mean) * inv_std is folded into the conv:
// conv = (sum_k w_k inv_std_c b_k) / 255 + bias - sum_k w_k inv_std_c mean_c
// over the taps inside the image. Taps outside the image are zero in the
// normalised tensor, so their share of the constant comes back through corr.
struct StemParams {
  float w[kStemCo][27];      // w * inv_std[ci], taps [ky][kx][ci], BN folded
  float b0[kStemCo];         // bias - sum over all 27 taps of w * inv_std * mean
  float corr[9][kStemCo];    // per tap position (ky, kx): sum_ci w * inv_std * mean
};

__device__ __forceinline__ float hswish(float v) {
  return v * fminf(fmaxf(v + 3.f, 0.f), 6.f) * (1.f / 6.f);
}
// The same function as v * clamp(v / 6 + 1/2, 0, 1): one saturating FMA and
// one multiply.
__device__ __forceinline__ float hswish_sat(float v) {
  return v * __saturatef(fmaf(v, 1.f / 6.f, 0.5f));
}

// The stem as an implicit GEMM on the tensor cores: M = 128 output pixels
// (a 4 x 32 tile), N = 32 channels, K = the 27 taps (ky, kx, ci) padded to
// 32, on the raw bytes (exact in fp16) against the normalisation-folded
// weights. fp16 weights alone would lose too much of the fp32 conv, so each
// is split into fp16 hi + lo (w = hi + lo to about 2^-22): an A row is the
// tap bytes twice, [b(32) | b(32)], one 128-byte K-major row, and a B row is
// [w_hi(32) | w_lo(32)], so four MMAs of K = 16 over the row accumulate
// sum b (w_hi + w_lo) in fp32. The epilogue scales by 1/255 and adds the
// folded bias (and, on the image border, the correction of the taps that
// fall outside).
// A persistent CTA of 128 threads loops over tiles. The bytes of the 9 x 65
// input window arrive as one 16-byte chunk per thread, loaded a tile ahead
// (in flight while the current tile runs) and parked in shared memory; each
// thread (= pixel = TMEM lane) normalises its 27 taps from there (zero
// outside the image: the conv pads the normalised tensor) into its A row,
// one thread issues the six MMAs into 32 TMEM columns, then every thread
// reads its pixel's 32 accumulators (tcgen05.ld), adds the bias, applies
// hardswish and stores 64 bytes.
namespace stc {
constexpr int TR = 4, TC = 32, TPX = TR * TC;   // output tile = MMA M
constexpr int WR = 2 * TR + 1, WC = 2 * TC + 1; // input window
constexpr int WB = 224;                         // window row bytes: 14 chunks of 16
constexpr int kThreads = 128;
static_assert(WR * (WB / 16) <= kThreads, "one window chunk per thread");
constexpr int OFF_A = 0, A_BYTES = TPX * 128;
constexpr int B_BYTES = kStemCo * 128;
constexpr int OFF_B = OFF_A + A_BYTES;
constexpr int OFF_WIN = OFF_B + B_BYTES;
constexpr int OFF_BIAS = OFF_WIN + WR * WB;      // b0 [32] then corr [9][32]
constexpr int OFF_BAR = (OFF_BIAS + 10 * kStemCo * 4 + 7) / 8 * 8;
constexpr int OFF_MISC = OFF_BAR + 8;           // TMEM address, abort flag
constexpr int SMEM_ALLOC = OFF_MISC + 16 + 1024;  // + runtime 1024 alignment
constexpr int TMEM_COLS = 32;
static_assert(OFF_B % 1024 == 0, "UMMA operand alignment");
}  // namespace stc

__device__ int g_stem_err;  // first bounded-wait timeout code, 0 if none

// Byte offset of 16-byte chunk `chunk` of row `row` in a K-major tile with
// 128-byte rows in the 128B-swizzle layout (8-row groups 1024 bytes apart).
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  const __half2 h = __halves2half2(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

__global__ void __launch_bounds__(stc::kThreads, 6)
stem_tc_kernel(const uint8_t *__restrict__ pages, int H, int W, long long page_stride,
               __half *__restrict__ out, const StemParams sp, int tiles_x, int tiles_y,
               int ntiles) {
  using namespace ptx;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sa = smem + stc::OFF_A, *sb = smem + stc::OFF_B;
  uint8_t *win = smem + stc::OFF_WIN;
  float *sbias = reinterpret_cast<float *>(smem + stc::OFF_BIAS);
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + stc::OFF_BAR);
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + stc::OFF_MISC);
  volatile int *s_abort = reinterpret_cast<volatile int *>(smem + stc::OFF_MISC + 4);
  const int tid = threadIdx.x, warp = tid >> 5;

  // ---- setup: split weights into the B tile [hi | lo], bias, barrier, TMEM ----
  for (int i = tid; i < kStemCo * 8; i += stc::kThreads) {
    const int co = i >> 3, j = i & 7;
    uint32_t h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __half v[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int k = 8 * (j & 3) + 2 * e + q;
        const float w = k < 27 ? sp.w[co][k] : 0.f;
        const __half hi = __float2half_rn(w);
        v[q] = j < 4 ? hi : __float2half_rn(w - __half2float(hi));
      }
      h[e] = pack_h2(v[0], v[1]);
    }
    *reinterpret_cast<uint4 *>(sb + sw128_off(co, j)) = make_uint4(h[0], h[1], h[2], h[3]);
  }
  for (int i = tid; i < 10 * kStemCo; i += stc::kThreads)
    sbias[i] = i < kStemCo ? sp.b0[i] : sp.corr[(i - kStemCo) / kStemCo][i % kStemCo];
  if (tid == 0) {
    mbar_init(bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(s_tmem, stc::TMEM_COLS);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  const int Ho = (H - 1) / 2 + 1, Wo = (W - 1) / 2 + 1;
  const int tiles_per_img = tiles_x * tiles_y;
  const long long row_bytes = 3ll * W;
  const int py = tid / stc::TC, px = tid % stc::TC;  // this thread's pixel in the tile
  constexpr uint32_t kIdesc = idesc_f16(stc::TPX, kStemCo);
  const bool vec_ok = (row_bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(pages) & 15) == 0 &&
                      (page_stride & 15) == 0;
  // this thread's window chunk of tile t: row tid / 14, bytes [a0 + 16 k, +16)
  const int crow = tid / (stc::WB / 16), ck = tid % (stc::WB / 16);
  auto load_chunk = [&](int t) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t >= ntiles || crow >= stc::WR) return v;
    const int n = t / tiles_per_img, r = t % tiles_per_img;
    const int y = 2 * (r / tiles_x) * stc::TR - 1 + crow;
    const long long b0 = 3ll * (2 * (r % tiles_x) * stc::TC - 1);
    const long long a0 = b0 >= 0 ? (b0 & ~15ll) : -16;
    const long long b = a0 + 16 * ck;
    if (y < 0 || y >= H || b < 0 || b >= row_bytes) return v;
    const uint8_t *q = pages + (long long)n * page_stride + (long long)y * row_bytes + b;
    if (vec_ok) return __ldg(reinterpret_cast<const uint4 *>(q));
    uint8_t tmp[16];
    for (int j = 0; j < 16; ++j) tmp[j] = b + j < row_bytes ? __ldg(q + j) : 0;
    memcpy(&v, tmp, 16);
    return v;
  };
  uint4 chunk = load_chunk(blockIdx.x);
  uint32_t it = 0;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
    const int n = t / tiles_per_img, r = t % tiles_per_img;
    const int oy0 = (r / tiles_x) * stc::TR, ox0 = (r % tiles_x) * stc::TC;
    const int iy0 = 2 * oy0 - 1, ix0 = 2 * ox0 - 1;
    const long long b0 = 3ll * ix0;
    const long long a0 = b0 >= 0 ? (b0 & ~15ll) : -16;
    if (crow < stc::WR) *reinterpret_cast<uint4 *>(win + crow * stc::WB + 16 * ck) = chunk;
    __syncthreads();
    chunk = load_chunk(t + gridDim.x);  // next tile's window, in flight meanwhile
    {  // A row of this pixel: tap bytes in (ky, kx, ci) order, twice. A tap
       // outside the image reads a zero: load_chunk leaves the window's rows
       // above / below the image and its 16-byte chunks left / right of a row
       // at zero, so no per-tap bounds test is needed.
      uint32_t pk[16];
      __half prev = __ushort2half_rn(0);
      const int off0 = (int)(3ll * (ix0 + 2 * px) - a0);
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
        const uint8_t *wr = win + (2 * py + ky) * stc::WB + off0;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
#pragma unroll
          for (int ci = 0; ci < 3; ++ci) {
            const int k = (ky * 3 + kx) * 3 + ci;
            const __half v = __ushort2half_rn(wr[3 * kx + ci]);
            if (k & 1) pk[k >> 1] = pack_h2(prev, v);
            else prev = v;
          }
        }
      }
      pk[13] = pack_h2(prev, __ushort2half_rn(0));  // tap 26, then zero padding
      pk[14] = pk[15] = 0u;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 c = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        *reinterpret_cast<uint4 *>(sa + sw128_off(tid, j)) = c;
        *reinterpret_cast<uint4 *>(sa + sw128_off(tid, j + 4)) = c;
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    bool waited = true;
    if (tid == 0) {  // the other threads wait at the barrier below, not spinning
      tc_fence_after();
      const uint32_t a = smem_u32(sa), b = smem_u32(sb);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_f16(tmem, sw128_kmajor_desc(a + 32 * k), sw128_kmajor_desc(b + 32 * k), kIdesc,
                k > 0 ? 1u : 0u);
      mma_commit(bar);
      waited = mbar_wait_bounded(bar, it & 1, s_abort, &g_stem_err, 41);
    }
    const bool ok = __syncthreads_and(waited);
    if (!ok) break;
    tc_fence_after();
    uint32_t v[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
    tmem_ld_wait(v);
    const int oy = oy0 + py, ox = ox0 + px;
    if (oy < Ho && ox < Wo) {
      // the folded bias straight from the parameter bank (FMA operand)
      float f[kStemCo];
#pragma unroll
      for (int c = 0; c < kStemCo; ++c) f[c] = fmaf(__uint_as_float(v[c]), 1.0f / 255.0f, sp.b0[c]);
      const int y0 = 2 * oy - 1, x0 = 2 * ox - 1;
      if (y0 < 0 || x0 < 0 || y0 + 2 >= H || x0 + 2 >= W) {  // taps outside the image
        for (int pos = 0; pos < 9; ++pos) {
          const int yy = y0 + pos / 3, xx = x0 + pos % 3;
          if (yy >= 0 && yy < H && xx >= 0 && xx < W) continue;
#pragma unroll
          for (int c = 0; c < kStemCo; ++c) f[c] += sbias[kStemCo * (1 + pos) + c];
        }
      }
      uint4 packed[kStemCo / 8];
      uint32_t *pw = reinterpret_cast<uint32_t *>(packed);
#pragma unroll
      for (int c = 0; c < kStemCo; c += 2) {
        const __half2 h = __floats2half2_rn(hswish_sat(f[c]), hswish_sat(f[c + 1]));
        pw[c / 2] = *reinterpret_cast<const uint32_t *>(&h);
      }
      uint4 *dst = reinterpret_cast<uint4 *>(out + (((long long)n * Ho + oy) * Wo + ox) * kStemCo);
#pragma unroll
      for (int k = 0; k < kStemCo / 8; ++k) dst[k] = packed[k];
    }
    tc_fence_before();
    __syncthreads();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, stc::TMEM_COLS);
  }
}

// ------------------------------------------------------------- ink map -------
constexpr int kInkRadius = 7;     // horizontal dilation: merges the glyphs of a line
constexpr int kInkTile = 256;

// grid (ceil(W/256), H, n), 256 threads: one row segment per CTA.
__global__ void __launch_bounds__(kInkTile)
ink_kernel(const uint8_t *__restrict__ pages, int H, int W, long long page_stride,
           float *__restrict__ prob, float gain) {
  __shared__ float s_ink[kInkTile + 2 * kInkRadius];
  const int n = blockIdx.z, y = blockIdx.y;
  const int x0 = blockIdx.x * kInkTile;
  const uint8_t *row = pages + (long long)n * page_stride + (long long)y * W * 3;
  for (int i = threadIdx.x; i < kInkTile + 2 * kInkRadius; i += blockDim.x) {
    const int x = x0 - kInkRadius + i;
    float v = 0.f;
    if (x >= 0 && x < W) {
      const uint8_t *p = row + x * 3;
      v = 1.f - ((float)p[0] + (float)p[1] + (float)p[2]) * (1.0f / 765.0f);
    }
    s_ink[i] = v;
  }
  __syncthreads();
  const int x = x0 + threadIdx.x;
  if (x >= W) return;
  float m = 0.f;
#pragma unroll
  for (int d = 0; d <= 2 * kInkRadius; ++d) m = fmaxf(m, s_ink[threadIdx.x + d]);
  prob[((long long)n * H + y) * W + x] = 1.f / (1.f + __expf(-gain * (m - 0.5f)));
}

// Rows up to kInkMaxW pixels: one CTA per row, the row's bytes staged with
// 16-byte loads, four outputs per thread written as a float4. Same values as
// ink_kernel. grid (H, n), 256 threads.
constexpr int kInkMaxW = 4096;

__global__ void __launch_bounds__(256)
ink_row_kernel(const uint8_t *__restrict__ pages, int H, int W, long long page_stride,
               float *__restrict__ prob, float gain) {
  __shared__ __align__(16) uint8_t s_b[3 * kInkMaxW];
  __shared__ float s_ink[kInkMaxW + 2 * kInkRadius + 4];
  const int y = blockIdx.x, n = blockIdx.y;
  const uint8_t *row = pages + (long long)n * page_stride + (long long)y * W * 3;
  const int nb = 3 * W;
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0 && (nb & 15) == 0) {
    for (int i = threadIdx.x; i < (nb >> 4); i += blockDim.x)
      reinterpret_cast<uint4 *>(s_b)[i] = __ldg(reinterpret_cast<const uint4 *>(row) + i);
  } else {
    for (int i = threadIdx.x; i < nb; i += blockDim.x) s_b[i] = __ldg(row + i);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < W + 2 * kInkRadius + 4; i += blockDim.x) {
    const int x = i - kInkRadius;
    float v = 0.f;
    if (x >= 0 && x < W)
      v = 1.f - ((float)s_b[3 * x] + (float)s_b[3 * x + 1] + (float)s_b[3 * x + 2]) * (1.0f / 765.0f);
    s_ink[i] = v;
  }
  __syncthreads();
  float *o = prob + ((long long)n * H + y) * W;
  const bool vec = (W & 3) == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0;
  for (int x = 4 * threadIdx.x; x < W; x += 4 * blockDim.x) {
    float win[2 * kInkRadius + 4];
#pragma unroll
    for (int d = 0; d < 2 * kInkRadius + 4; ++d) win[d] = s_ink[x + d];
    float r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float m = 0.f;
#pragma unroll
      for (int d = 0; d <= 2 * kInkRadius; ++d) m = fmaxf(m, win[j + d]);
      r[j] = 1.f / (1.f + __expf(-gain * (m - 0.5f)));
    }
    if (vec) {
      *reinterpret_cast<float4 *>(o + x) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
      for (int j = 0; j < 4 && x + j < W; ++j) o[x + j] = r[j];
    }
  }
}

// ---------------------------------------------------------------- head -------
// 1x1 conv C->1 + bias + sigmoid over fp16 NHWC. One warp per pixel.
__global__ void __launch_bounds__(256)
head_kernel(const __half *__restrict__ x, long long npix, int C, const float *__restrict__ w,
            float bias, float *__restrict__ out) {
  const long long p = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (p >= npix) return;
  const __half *px = x + p * C;
  float acc = 0.f;
  for (int c = lane * 2; c < C; c += 64) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(px + c));
    acc = fmaf(v.x, w[c], fmaf(v.y, w[c + 1], acc));
  }
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) out[p] = 1.f / (1.f + __expf(-(acc + bias)));
}

// ------------------------------------------------------------ ROI warp -------
struct RecNorm {
  float mean[3], inv_std[3], inv_scale;
};

// One output pixel of crop b (r, g, b planes), arithmetic as
// batch_roi_warp_kernel: zero beyond the crop width or for a non-finite
// source position.
__device__ __forceinline__ void roi_warp_px(const uint8_t *src, int src_h, int src_w, int src_step,
                                            const float *M, int cw, int x, int y,
                                            const RecNorm &nm, float o[3]) {
  o[0] = o[1] = o[2] = 0.f;
  if (x >= cw) return;
  float denom = M[6] * x + M[7] * y + M[8];
  denom = copysignf(fmaxf(fabsf(denom), 1e-7f), denom);
  const float inv_denom = 1.0f / denom;
  float sx = (M[0] * x + M[1] * y + M[2]) * inv_denom;
  float sy = (M[3] * x + M[4] * y + M[5]) * inv_denom;
  if (!isfinite(sx) || !isfinite(sy)) return;
  sx = fminf(fmaxf(sx, -1.0f), (float)(src_w + 1));
  sy = fminf(fmaxf(sy, -1.0f), (float)(src_h + 1));
  int xl = (int)floorf(sx), yl = (int)floorf(sy);
  int xh = xl + 1, yh = yl + 1;
  const float dx = sx - xl, dy = sy - yl;
  xl = min(max(xl, 0), src_w - 1); xh = min(max(xh, 0), src_w - 1);
  yl = min(max(yl, 0), src_h - 1); yh = min(max(yh, 0), src_h - 1);
  auto pix = [&](int px, int py) {
    const uint8_t *p = src + (long long)py * src_step + px * 3;
    return make_float3((float)__ldg(p + 2), (float)__ldg(p + 1), (float)__ldg(p));
  };
  const float3 p00 = pix(xl, yl), p10 = pix(xh, yl), p01 = pix(xl, yh), p11 = pix(xh, yh);
  const float w00 = (1.0f - dx) * (1.0f - dy), w10 = dx * (1.0f - dy);
  const float w01 = (1.0f - dx) * dy, w11 = dx * dy;
  const float r = w00 * p00.x + w10 * p10.x + w01 * p01.x + w11 * p11.x;
  const float g = w00 * p00.y + w10 * p10.y + w01 * p01.y + w11 * p11.y;
  const float bl = w00 * p00.z + w10 * p10.z + w01 * p01.z + w11 * p11.z;
  o[0] = (r * nm.inv_scale - nm.mean[0]) * nm.inv_std[0];
  o[1] = (g * nm.inv_scale - nm.mean[1]) * nm.inv_std[1];
  o[2] = (bl * nm.inv_scale - nm.mean[2]) * nm.inv_std[2];
}

template <typename OutT>
struct WarpStore;
template <>
struct WarpStore<__half> {
  static __device__ __forceinline__ void one(__half *p, float v) { *p = __float2half_rn(v); }
  static __device__ __forceinline__ void two(__half *p, float a, float b) {
    *reinterpret_cast<__half2 *>(p) = __floats2half2_rn(a, b);
  }
};
template <>
struct WarpStore<float> {
  static __device__ __forceinline__ void one(float *p, float v) { *p = v; }
  static __device__ __forceinline__ void two(float *p, float a, float b) {
    *reinterpret_cast<float2 *>(p) = make_float2(a, b);
  }
};

// grid (ceil(dst_w/64), ceil(dst_h/8), z), block (32, 8): the z slices stride
// over the crops that exist (*n_crops when given, else n_crops_value, at most
// max_crops), so no CTA is spent on empty crop slots. crop_page NULL: every
// crop comes from page 0. A thread writes two neighbouring pixels (one
// 2-element store per plane when the width is even).
template <typename OutT>
__global__ void __launch_bounds__(256)
roi_warp_kernel(const uint8_t *__restrict__ pages, long long page_stride, int src_h, int src_w,
                int src_step, const float *__restrict__ minv, const int *__restrict__ crop_w,
                const int *__restrict__ crop_page, const int *__restrict__ n_crops,
                int n_crops_value, int max_crops, OutT *__restrict__ dst, int dst_h, int dst_w,
                RecNorm nm) {
  __shared__ float s_M[9];
  __shared__ int s_crop_w, s_page;
  const int nc = min(n_crops ? *n_crops : n_crops_value, max_crops);
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  const int x0 = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  const int y = blockIdx.y * blockDim.y + threadIdx.y;
  const long long plane = (long long)dst_h * dst_w;
  const bool pair = (dst_w & 1) == 0 && (reinterpret_cast<uintptr_t>(dst) & (2 * sizeof(OutT) - 1)) == 0;
  for (int b = blockIdx.z; b < nc; b += gridDim.z) {
    __syncthreads();
    if (tid < 9) s_M[tid] = minv[(long long)b * 9 + tid];
    if (tid == 0) { s_crop_w = crop_w[b]; s_page = crop_page ? crop_page[b] : 0; }
    __syncthreads();
    if (x0 >= dst_w || y >= dst_h) continue;
    const uint8_t *src = pages + (long long)s_page * page_stride;
    float v0[3], v1[3];
    roi_warp_px(src, src_h, src_w, src_step, s_M, s_crop_w, x0, y, nm, v0);
    OutT *o = dst + (long long)b * 3 * plane + (long long)y * dst_w + x0;
    if (pair) {
      roi_warp_px(src, src_h, src_w, src_step, s_M, s_crop_w, x0 + 1, y, nm, v1);
#pragma unroll
      for (int c = 0; c < 3; ++c) WarpStore<OutT>::two(o + c * plane, v0[c], v1[c]);
    } else {
#pragma unroll
      for (int c = 0; c < 3; ++c) WarpStore<OutT>::one(o + c * plane, v0[c]);
      if (x0 + 1 < dst_w) {
        roi_warp_px(src, src_h, src_w, src_step, s_M, s_crop_w, x0 + 1, y, nm, v1);
#pragma unroll
        for (int c = 0; c < 3; ++c) WarpStore<OutT>::one(o + c * plane + 1, v1[c]);
      }
    }
  }
}

// ---------------------------------------------------- stand-in network heads --
// The trained detection and recognition networks are not available, so the
// modules (PaddleDet / PaddleRec) run these stand-ins where the reference
// runs its TensorRT engines:
//   det: the synthetic page's DB probability map computed from the
//        normalised canvas: ink = 1 - mean of the de-normalised channels
//        (0 outside the letterbox content), 15-pixel horizontal max,
//        sigmoid(gain * (max - 0.5));
//   rec: CTC logits [n][T][V] fp16, 0 except 16.0 at one class per step, the
//        class of crop id and step t being hash-drawn per 3 steps (blank with
//        probability 1/2, else uniform over 1..V-1).
constexpr int kHeadTile = 256, kHeadRadius = 7;

__global__ void __launch_bounds__(kHeadTile)
det_standin_kernel(const float *__restrict__ chw, int H, int W, const int *__restrict__ content,
                   float s0, float s1, float s2, float m0, float m1, float m2, float gain,
                   float *__restrict__ prob) {
  __shared__ float s_ink[kHeadTile + 2 * kHeadRadius];
  const int b = blockIdx.z, y = blockIdx.y, x0 = blockIdx.x * kHeadTile;
  const int ch = content ? content[2 * b] : H, cw = content ? content[2 * b + 1] : W;
  const long long plane = (long long)H * W;
  const float *img = chw + (long long)b * 3 * plane + (long long)y * W;
  for (int i = threadIdx.x; i < kHeadTile + 2 * kHeadRadius; i += blockDim.x) {
    const int x = x0 - kHeadRadius + i;
    float v = 0.f;
    if (x >= 0 && x < W && x < cw && y < ch) {
      const float r = img[x] * s0 + m0, g = img[plane + x] * s1 + m1, bl = img[2 * plane + x] * s2 + m2;
      v = 1.f - (r + g + bl) * (1.f / 3.f);
    }
    s_ink[i] = v;
  }
  __syncthreads();
  const int x = x0 + threadIdx.x;
  if (x >= W) return;
  float m = 0.f;
#pragma unroll
  for (int d = 0; d <= 2 * kHeadRadius; ++d) m = fmaxf(m, s_ink[threadIdx.x + d]);
  prob[(long long)b * plane + (long long)y * W + x] = 1.f / (1.f + __expf(-gain * (m - 0.5f)));
}

__device__ __forceinline__ uint64_t standin_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ int standin_token(uint64_t seed, long long id, int t, int V) {
  const uint64_t h = standin_mix(seed + 0x9E3779B97F4A7C15ULL *
                                 (standin_mix(7000 + (uint64_t)id) + (uint64_t)(t / 3) + 1));
  return (h & 1) ? 0 : 1 + (int)((h >> 32) % (uint64_t)(V - 1));
}

// grid-stride over the n*T rows; one warp per row: zero the row,
// then plant 16.0 (p_max near 1, so results pass the drop score).
__global__ void __launch_bounds__(256)
rec_standin_kernel(__half *__restrict__ logits, const int *__restrict__ ids, long long rows, int T,
                   int V, uint64_t seed) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    __half *row = logits + r * V;
    for (int j = lane; j < V; j += 32) row[j] = __float2half_rn(0.f);
    __syncwarp();
    if (lane == 0) {
      const long long c = r / T;
      const int t = (int)(r % T);
      row[standin_token(seed, ids ? ids[c] : c, t, V)] = __float2half_rn(16.f);
    }
  }
}

RecNorm rec_norm(const float *mean3, const float *inv_std3, float inv_scale) {
  RecNorm nm;
  for (int c = 0; c < 3; ++c) {
    nm.mean[c] = mean3 ? mean3[c] : 0.5f;
    nm.inv_std[c] = inv_std3 ? inv_std3[c] : 2.0f;
  }
  nm.inv_scale = inv_scale;
  return nm;
}

template <typename OutT>
int launch_roi_warp(const uint8_t *d_pages, long long page_stride, int src_h, int src_w,
                    int src_step, const float *d_minv, const int *d_crop_w, const int *d_crop_page,
                    const int *d_n_crops, int n_crops_value, int max_crops, int dst_h, int dst_w,
                    const RecNorm &nm, OutT *d_dst, void *stream, const char *name) {
  TOCR_REQUIRE(max_crops >= 0 && dst_h > 0 && dst_w > 0 && src_h > 0 && src_w > 0,
               "%s: bad sizes", name);
  if (max_crops == 0) return TOCR_OK;
  TOCR_REQUIRE(d_pages && d_minv && d_crop_w && d_dst, "%s: null pointer", name);
  const dim3 block(32, 8);
  const unsigned gx = (dst_w + 63) / 64, gy = (dst_h + 7) / 8;
  // about 16 CTAs per SM in flight; each z slice strides over the crops
  const unsigned zmax = (unsigned)std::max(1, sm_count() * 16 / (int)(gx * gy));
  const dim3 grid(gx, gy, std::min<unsigned>((unsigned)max_crops, std::min(zmax, 65535u)));
  roi_warp_kernel<OutT><<<grid, block, 0, as_stream(stream)>>>(
      d_pages, page_stride, src_h, src_w, src_step, d_minv, d_crop_w, d_crop_page, d_n_crops,
      n_crops_value, max_crops, d_dst, dst_h, dst_w, nm);
  return check_launch(name);
}

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API size_t tocr_stem_params_bytes(void) { return sizeof(StemParams); }

TOCR_API int tocr_stem_pack(const float *w /* [32][3][3][3] co,ci,ky,kx */, const float *b,
                            const float *mean3, const float *inv_std3, void *out,
                            size_t out_bytes) {
  TOCR_REQUIRE(w && b && out && out_bytes >= sizeof(StemParams), "tocr_stem_pack: bad arguments");
  StemParams p{};
  const double dm[3] = {0.485, 0.456, 0.406};
  const double ds[3] = {1.0 / 0.229, 1.0 / 0.224, 1.0 / 0.225};
  double mean[3], inv[3];
  for (int c = 0; c < 3; ++c) {
    mean[c] = mean3 ? (double)mean3[c] : (double)(float)dm[c];
    inv[c] = inv_std3 ? (double)inv_std3[c] : (double)(float)ds[c];
  }
  for (int co = 0; co < kStemCo; ++co) {
    double total = 0.;
    for (int ky = 0; ky < 3; ++ky)
      for (int kx = 0; kx < 3; ++kx) {
        double cpos = 0.;
        for (int ci = 0; ci < 3; ++ci) {
          const double wv = w[((co * 3 + ci) * 3 + ky) * 3 + kx];
          p.w[co][(ky * 3 + kx) * 3 + ci] = (float)(wv * inv[ci]);
          cpos += wv * inv[ci] * mean[ci];
        }
        p.corr[ky * 3 + kx][co] = (float)cpos;
        total += cpos;
      }
    p.b0[co] = (float)((double)b[co] - total);
  }
  memcpy(out, &p, sizeof(p));
  return TOCR_OK;
}

TOCR_API int tocr_stem_f16(const uint8_t *d_pages, int n, int h, int w, long long page_stride,
                           const void *h_params, void *d_out, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && h > 0 && w > 0, "tocr_stem_f16: bad sizes n=%d h=%d w=%d", n, h, w);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_pages && h_params && d_out && aligned(d_out, 16), "tocr_stem_f16: bad pointer");
  const int Ho = (h - 1) / 2 + 1, Wo = (w - 1) / 2 + 1;
  StemParams sp;
  memcpy(&sp, h_params, sizeof(sp));
  const int tiles_x = (Wo + stc::TC - 1) / stc::TC, tiles_y = (Ho + stc::TR - 1) / stc::TR;
  const long long ntiles = (long long)n * tiles_x * tiles_y;
  TOCR_REQUIRE(ntiles < (1ll << 31), "tocr_stem_f16: too many tiles");
  cudaError_t e = cudaFuncSetAttribute(stem_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       stc::SMEM_ALLOC);
  if (e != cudaSuccess) return set_error(TOCR_ERR_CUDA, "stem smem attribute: %s", cudaGetErrorString(e));
  // persistent CTAs: as many as fit per SM (6 by shared memory; 6 x 32 TMEM columns)
  const long long grid = std::min<long long>(ntiles, (long long)sm_count() * 6);
  stem_tc_kernel<<<(unsigned)grid, stc::kThreads, stc::SMEM_ALLOC, as_stream(stream)>>>(
      d_pages, h, w, page_stride, (__half *)d_out, sp, tiles_x, tiles_y, (int)ntiles);
  return check_launch("stem_tc_kernel");
}

// The stem's bounded waits record the first timeout in a device word: this
// writes it to *out_code (0: none), clears it, and synchronises the current
// device.
TOCR_API int tocr_stem_take_error(int *out_code) {
  TOCR_ENTRY();
  TOCR_REQUIRE(out_code, "tocr_stem_take_error: null pointer");
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_stem_err, sizeof(int));
  if (e == cudaSuccess) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_stem_err, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return set_error(TOCR_ERR_CUDA, "tocr_stem_take_error: %s", cudaGetErrorString(e));
  *out_code = v;
  return TOCR_OK;
}

TOCR_API int tocr_ink_map(const uint8_t *d_pages, int n, int h, int w, long long page_stride,
                          float gain, float *d_prob, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && h > 0 && w > 0, "tocr_ink_map: bad sizes");
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_pages && d_prob, "tocr_ink_map: null pointer");
  if (w <= kInkMaxW) {
    ink_row_kernel<<<dim3(h, n), 256, 0, as_stream(stream)>>>(d_pages, h, w, page_stride, d_prob,
                                                             gain);
  } else {
    const dim3 grid((w + kInkTile - 1) / kInkTile, h, n);
    ink_kernel<<<grid, kInkTile, 0, as_stream(stream)>>>(d_pages, h, w, page_stride, d_prob, gain);
  }
  return check_launch("ink_kernel");
}

TOCR_API int tocr_head_sigmoid(const void *d_x, long long npix, int c, const float *d_w,
                               float bias, float *d_out, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(npix >= 0 && c > 0 && c % 64 == 0, "tocr_head_sigmoid: bad sizes");
  if (npix == 0) return TOCR_OK;
  const unsigned grid = (unsigned)((npix * 32 + 255) / 256);
  head_kernel<<<grid, 256, 0, as_stream(stream)>>>((const __half *)d_x, npix, c, d_w, bias, d_out);
  return check_launch("head_kernel");
}

TOCR_API int tocr_roi_warp_f16(const uint8_t *d_pages, long long page_stride, int src_h,
                               int src_w, int src_step, const float *d_minv, const int *d_crop_w,
                               const int *d_crop_page, const int *d_n_crops, int max_crops,
                               int dst_h, int dst_w, const float *mean3, const float *inv_std3,
                               float inv_scale, void *d_dst, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(max_crops >= 0, "tocr_roi_warp_f16: bad sizes");
  if (max_crops == 0) return TOCR_OK;
  TOCR_REQUIRE(d_crop_page && d_n_crops, "tocr_roi_warp_f16: null pointer");
  return launch_roi_warp<__half>(d_pages, page_stride, src_h, src_w, src_step, d_minv, d_crop_w,
                                 d_crop_page, d_n_crops, 0, max_crops, dst_h, dst_w,
                                 rec_norm(mean3, inv_std3, inv_scale),
                                 static_cast<__half *>(d_dst), stream, "tocr_roi_warp_f16");
}

TOCR_API int tocr_det_standin_prob_f32(const float *d_chw, int n, int h, int w,
                                       const int *d_content_hw, const float *mean3,
                                       const float *inv_std3, float gain, float *d_prob,
                                       void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && h > 0 && w > 0 && h <= 65535 && n <= 65535,
               "tocr_det_standin_prob_f32: bad sizes n=%d h=%d w=%d", n, h, w);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_chw && d_prob, "tocr_det_standin_prob_f32: null pointer");
  const float dm[3] = {0.485f, 0.456f, 0.406f}, ds[3] = {0.229f, 0.224f, 0.225f};
  float m[3], sd[3];
  for (int c = 0; c < 3; ++c) {
    m[c] = mean3 ? mean3[c] : dm[c];
    sd[c] = inv_std3 ? 1.f / inv_std3[c] : ds[c];
  }
  const dim3 grid((w + kHeadTile - 1) / kHeadTile, h, n);
  det_standin_kernel<<<grid, kHeadTile, 0, as_stream(stream)>>>(d_chw, h, w, d_content_hw, sd[0],
                                                                 sd[1], sd[2], m[0], m[1], m[2],
                                                                 gain, d_prob);
  return check_launch("det_standin_kernel");
}

TOCR_API int tocr_rec_standin_logits_f16(void *d_logits, const int *d_ids, int n, int seq_len,
                                         int num_classes, uint64_t seed, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && seq_len > 0 && num_classes > 1,
               "tocr_rec_standin_logits_f16: bad sizes n=%d T=%d V=%d", n, seq_len, num_classes);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_logits, "tocr_rec_standin_logits_f16: null pointer");
  const long long rows = (long long)n * seq_len;
  const unsigned grid = (unsigned)std::min<long long>((rows + 7) / 8, (long long)sm_count() * 16);
  rec_standin_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<__half *>(d_logits), d_ids,
                                                          rows, seq_len, num_classes, seed);
  return check_launch("rec_standin_kernel");
}

TOCR_API int tocr_roi_warp_f32(const uint8_t *d_src, int src_h, int src_w, int src_step,
                               const float *d_minv, const int *d_crop_w, int batch_size,
                               int dst_h, int dst_w, const float *mean3, const float *inv_std3,
                               float inv_scale, float *d_dst, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(batch_size >= 0, "tocr_roi_warp_f32: bad batch size %d", batch_size);
  return launch_roi_warp<float>(d_src, 0, src_h, src_w, src_step, d_minv, d_crop_w, nullptr,
                                nullptr, batch_size, batch_size, dst_h, dst_w,
                                rec_norm(mean3, inv_std3, inv_scale), d_dst, stream,
                                "tocr_roi_warp_f32");
}

}  // extern "C"
