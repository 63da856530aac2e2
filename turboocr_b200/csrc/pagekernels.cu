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

#include <algorithm>
#include <cmath>
#include <cstring>

namespace tocr {
namespace {

// ---------------------------------------------------------------- stem -------
constexpr int kStemCo = 32;

struct StemParams {
  float w[kStemCo][27];  // [co][ky][kx][ci], BN folded
  float b[kStemCo];
  float mean[3], inv_std[3];
};

__device__ __forceinline__ float hswish(float v) {
  return v * fminf(fmaxf(v + 3.f, 0.f), 6.f) * (1.f / 6.f);
}

// A CTA computes an 8 x 64 tile of output pixels. The 17 x 129-pixel input
// window is staged once in shared memory, already normalised (zero outside
// the image: the conv pads the normalised tensor), channel planes apart; the
// weights go to shared memory as [tap][co]. Each thread then accumulates a
// 4-pixel x 16-channel block in registers: per tap, four window reads (the
// thread's pixels are 16 columns apart, so a warp reads 16 consecutive even
// columns: no bank conflicts) and four float4 weight broadcasts feed 64 FMAs.
// Every output keeps the tap order (ky, kx, ci) of the accumulation.
// grid (tiles_x, tiles_y, n), 256 threads.
constexpr int kStemTH = 8, kStemTW = 64;
constexpr int kStemIH = 2 * kStemTH + 1, kStemIW = 2 * kStemTW + 1;
constexpr int kStemPitch = kStemIW + 3;  // row pitch of a channel plane (floats)

__global__ void __launch_bounds__(256, 2)
stem_kernel(const uint8_t *__restrict__ pages, int H, int W, long long page_stride,
            __half *__restrict__ out, const StemParams sp) {
  __shared__ float s_in[3][kStemIH][kStemPitch];
  __shared__ __align__(16) float s_w[27][kStemCo];
  const int Ho = (H - 1) / 2 + 1, Wo = (W - 1) / 2 + 1;
  const int n = blockIdx.z;
  const int oy0 = blockIdx.y * kStemTH, ox0 = blockIdx.x * kStemTW;
  const int iy0 = 2 * oy0 - 1, ix0 = 2 * ox0 - 1;
  const uint8_t *pg = pages + (long long)n * page_stride;
  for (int i = threadIdx.x; i < 27 * kStemCo; i += blockDim.x) {
    const int k = i / kStemCo, co = i - k * kStemCo;
    s_w[k][co] = sp.w[co][k];
  }
  // one window pixel per item: its three bytes, normalised (0 outside)
  const long long row_bytes = 3ll * W;
  for (int i = threadIdx.x; i < kStemIH * kStemIW; i += blockDim.x) {
    const int row = i / kStemIW, col = i - row * kStemIW;
    const int y = iy0 + row, x = ix0 + col;
    float v0 = 0.f, v1 = 0.f, v2 = 0.f;
    if (y >= 0 && y < H && x >= 0 && x < W) {
      const uint8_t *px = pg + (long long)y * row_bytes + 3ll * x;
      v0 = ((float)__ldg(px) * (1.0f / 255.0f) - sp.mean[0]) * sp.inv_std[0];
      v1 = ((float)__ldg(px + 1) * (1.0f / 255.0f) - sp.mean[1]) * sp.inv_std[1];
      v2 = ((float)__ldg(px + 2) * (1.0f / 255.0f) - sp.mean[2]) * sp.inv_std[2];
    }
    s_in[0][row][col] = v0;
    s_in[1][row][col] = v1;
    s_in[2][row][col] = v2;
  }
  __syncthreads();
  const int half = threadIdx.x & 1;          // output channels 16 * half .. + 15
  const int g = threadIdx.x >> 1;            // 128 pixel groups
  const int ty = g >> 4, gx = g & 15;        // pixels (ty, gx + 16 j), j = 0..3
  float acc[4][16];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int c = 0; c < 16; ++c) acc[j][c] = sp.b[16 * half + c];
#pragma unroll
  for (int ky = 0; ky < 3; ++ky)
#pragma unroll
    for (int kx = 0; kx < 3; ++kx)
#pragma unroll
      for (int ci = 0; ci < 3; ++ci) {
        const int k = (ky * 3 + kx) * 3 + ci;
        float t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] = s_in[ci][2 * ty + ky][2 * (gx + 16 * j) + kx];
        const float4 *wv = reinterpret_cast<const float4 *>(&s_w[k][16 * half]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 w4 = wv[q];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[j][4 * q + 0] = fmaf(w4.x, t[j], acc[j][4 * q + 0]);
            acc[j][4 * q + 1] = fmaf(w4.y, t[j], acc[j][4 * q + 1]);
            acc[j][4 * q + 2] = fmaf(w4.z, t[j], acc[j][4 * q + 2]);
            acc[j][4 * q + 3] = fmaf(w4.w, t[j], acc[j][4 * q + 3]);
          }
        }
      }
  const int oy = oy0 + ty;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int ox = ox0 + gx + 16 * j;
    if (oy >= Ho || ox >= Wo) continue;
    uint4 packed[2];
    uint32_t *pw = reinterpret_cast<uint32_t *>(packed);
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
      const __half2 h = __floats2half2_rn(hswish(acc[j][c]), hswish(acc[j][c + 1]));
      pw[c / 2] = *reinterpret_cast<const uint32_t *>(&h);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out + (((long long)n * Ho + oy) * Wo + ox) * kStemCo +
                                           16 * half);
    dst[0] = packed[0];
    dst[1] = packed[1];
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

// One output pixel of crop b (r, g, b planes as fp16), arithmetic as
// batch_roi_warp_kernel: zero beyond the crop width or for a non-finite
// source position.
__device__ __forceinline__ void roi_warp_px(const uint8_t *src, int src_h, int src_w, int src_step,
                                            const float *M, int cw, int x, int y,
                                            const RecNorm &nm, __half o[3]) {
  o[0] = o[1] = o[2] = __float2half_rn(0.f);
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
  o[0] = __float2half_rn((r * nm.inv_scale - nm.mean[0]) * nm.inv_std[0]);
  o[1] = __float2half_rn((g * nm.inv_scale - nm.mean[1]) * nm.inv_std[1]);
  o[2] = __float2half_rn((bl * nm.inv_scale - nm.mean[2]) * nm.inv_std[2]);
}

// grid (ceil(dst_w/64), ceil(dst_h/8), z), block (32, 8): the z slices stride
// over the crops that exist (*n_crops, at most max_crops), so no CTA is spent
// on empty crop slots. A thread writes two neighbouring pixels (half2 per
// plane when the width is even).
__global__ void __launch_bounds__(256)
roi_warp_kernel(const uint8_t *__restrict__ pages, long long page_stride, int src_h, int src_w,
                int src_step, const float *__restrict__ minv, const int *__restrict__ crop_w,
                const int *__restrict__ crop_page, const int *__restrict__ n_crops, int max_crops,
                __half *__restrict__ dst, int dst_h, int dst_w, RecNorm nm) {
  __shared__ float s_M[9];
  __shared__ int s_crop_w, s_page;
  const int nc = min(*n_crops, max_crops);
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  const int x0 = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  const int y = blockIdx.y * blockDim.y + threadIdx.y;
  const long long plane = (long long)dst_h * dst_w;
  const bool pair = (dst_w & 1) == 0 && (reinterpret_cast<uintptr_t>(dst) & 3) == 0;
  for (int b = blockIdx.z; b < nc; b += gridDim.z) {
    __syncthreads();
    if (tid < 9) s_M[tid] = minv[(long long)b * 9 + tid];
    if (tid == 0) { s_crop_w = crop_w[b]; s_page = crop_page[b]; }
    __syncthreads();
    if (x0 >= dst_w || y >= dst_h) continue;
    const uint8_t *src = pages + (long long)s_page * page_stride;
    __half v0[3], v1[3];
    roi_warp_px(src, src_h, src_w, src_step, s_M, s_crop_w, x0, y, nm, v0);
    __half *o = dst + (long long)b * 3 * plane + (long long)y * dst_w + x0;
    if (pair) {
      roi_warp_px(src, src_h, src_w, src_step, s_M, s_crop_w, x0 + 1, y, nm, v1);
#pragma unroll
      for (int c = 0; c < 3; ++c)
        *reinterpret_cast<__half2 *>(o + c * plane) = __halves2half2(v0[c], v1[c]);
    } else {
#pragma unroll
      for (int c = 0; c < 3; ++c) o[c * plane] = v0[c];
      if (x0 + 1 < dst_w) {
        roi_warp_px(src, src_h, src_w, src_step, s_M, s_crop_w, x0 + 1, y, nm, v1);
#pragma unroll
        for (int c = 0; c < 3; ++c) o[c * plane + 1] = v1[c];
      }
    }
  }
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
  const float dm[3] = {0.485f, 0.456f, 0.406f};
  const float ds[3] = {1.0f / 0.229f, 1.0f / 0.224f, 1.0f / 0.225f};
  for (int co = 0; co < kStemCo; ++co) {
    for (int ci = 0; ci < 3; ++ci)
      for (int ky = 0; ky < 3; ++ky)
        for (int kx = 0; kx < 3; ++kx)
          p.w[co][(ky * 3 + kx) * 3 + ci] = w[((co * 3 + ci) * 3 + ky) * 3 + kx];
    p.b[co] = b[co];
  }
  for (int c = 0; c < 3; ++c) {
    p.mean[c] = mean3 ? mean3[c] : dm[c];
    p.inv_std[c] = inv_std3 ? inv_std3[c] : ds[c];
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
  const dim3 grid((Wo + kStemTW - 1) / kStemTW, (Ho + kStemTH - 1) / kStemTH, n);
  stem_kernel<<<grid, 256, 0, as_stream(stream)>>>(d_pages, h, w, page_stride, (__half *)d_out, sp);
  return check_launch("stem_kernel");
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
  TOCR_REQUIRE(max_crops >= 0 && dst_h > 0 && dst_w > 0 && src_h > 0 && src_w > 0,
               "tocr_roi_warp_f16: bad sizes");
  if (max_crops == 0) return TOCR_OK;
  RecNorm nm;
  for (int c = 0; c < 3; ++c) {
    nm.mean[c] = mean3 ? mean3[c] : 0.5f;
    nm.inv_std[c] = inv_std3 ? inv_std3[c] : 2.0f;
  }
  nm.inv_scale = inv_scale;
  const dim3 block(32, 8);
  const unsigned gx = (dst_w + 63) / 64, gy = (dst_h + 7) / 8;
  // about 16 CTAs per SM in flight; each z slice strides over the crops
  const unsigned zmax = (unsigned)std::max(1, sm_count() * 16 / (int)(gx * gy));
  const dim3 grid(gx, gy, std::min<unsigned>((unsigned)max_crops, std::min(zmax, 65535u)));
  roi_warp_kernel<<<grid, block, 0, as_stream(stream)>>>(d_pages, page_stride, src_h, src_w,
                                                         src_step, d_minv, d_crop_w, d_crop_page,
                                                         d_n_crops, max_crops, (__half *)d_dst,
                                                         dst_h, dst_w, nm);
  return check_launch("roi_warp_kernel");
}

}  // extern "C"
