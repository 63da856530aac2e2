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

// A CTA computes an 8 x 64 tile of output pixels (two per thread). The
// 17 x 129-pixel input window is staged once in shared memory, already
// normalised (zero outside the image: the conv pads the normalised tensor);
// the weights arrive by value in the kernel's parameter (constant) bank, so
// every FMA takes its weight straight from there. grid (tiles_x, tiles_y, n).
constexpr int kStemTH = 8, kStemTW = 64;
constexpr int kStemIH = 2 * kStemTH + 1, kStemIW = 2 * kStemTW + 1;

__global__ void __launch_bounds__(256, 2)
stem_kernel(const uint8_t *__restrict__ pages, int H, int W, long long page_stride,
            __half *__restrict__ out, const StemParams sp) {
  __shared__ float s_in[kStemIH][kStemIW][3];
  const int Ho = (H - 1) / 2 + 1, Wo = (W - 1) / 2 + 1;
  const int n = blockIdx.z;
  const int oy0 = blockIdx.y * kStemTH, ox0 = blockIdx.x * kStemTW;
  const int iy0 = 2 * oy0 - 1, ix0 = 2 * ox0 - 1;
  const uint8_t *pg = pages + (long long)n * page_stride;
  float *flat = &s_in[0][0][0];
  for (int i = threadIdx.x; i < kStemIH * kStemIW * 3; i += blockDim.x) flat[i] = 0.f;
  __syncthreads();
  // 16-byte loads of each input row's byte range [bs, be) (rows are 3W bytes)
  const long long row_bytes = 3ll * W;
  const int bs0 = 3 * ix0, be0 = 3 * (ix0 + kStemIW);
  const int bs = bs0 > 0 ? bs0 : 0;
  const int be = be0 < row_bytes ? be0 : (int)row_bytes;
  const int a0 = bs & ~15;
  const int chunks = (be - a0 + 15) >> 4;
  const bool vec_ok = (row_bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(pg) & 15) == 0;
  for (int i = threadIdx.x; i < kStemIH * chunks; i += blockDim.x) {
    const int row = i / chunks, k = i % chunks;
    const int y = iy0 + row;
    if (y < 0 || y >= H) continue;
    const uint8_t *rp = pg + (long long)y * row_bytes;
    const int b0 = a0 + 16 * k;
    uint8_t v[16];
    if (vec_ok && b0 + 16 <= row_bytes) {
      *reinterpret_cast<uint4 *>(v) = __ldg(reinterpret_cast<const uint4 *>(rp + b0));
    } else {
      for (int j = 0; j < 16; ++j) v[j] = (b0 + j < row_bytes) ? rp[b0 + j] : 0;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int b = b0 + j;
      if (b < bs || b >= be) continue;
      const int lb = b - bs0;
      const int col = lb / 3, c = lb - 3 * col;
      flat[(row * kStemIW + col) * 3 + c] =
          ((float)v[j] * (1.0f / 255.0f) - sp.mean[c]) * sp.inv_std[c];
    }
  }
  __syncthreads();
  for (int q = threadIdx.x; q < kStemTH * kStemTW; q += blockDim.x) {
    const int ty = q / kStemTW, tx = q % kStemTW;
    const int oy = oy0 + ty, ox = ox0 + tx;
    if (oy >= Ho || ox >= Wo) continue;
    float tap[27];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx)
#pragma unroll
        for (int c = 0; c < 3; ++c) tap[(ky * 3 + kx) * 3 + c] = s_in[2 * ty + ky][2 * tx + kx][c];
    uint4 packed[kStemCo / 8];
    uint32_t *pw = reinterpret_cast<uint32_t *>(packed);
#pragma unroll
    for (int co = 0; co < kStemCo; co += 2) {
      float a0 = sp.b[co], a1 = sp.b[co + 1];
#pragma unroll
      for (int k = 0; k < 27; ++k) {
        a0 = fmaf(sp.w[co][k], tap[k], a0);
        a1 = fmaf(sp.w[co + 1][k], tap[k], a1);
      }
      const __half2 h = __floats2half2_rn(hswish(a0), hswish(a1));
      pw[co / 2] = *reinterpret_cast<const uint32_t *>(&h);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out + (((long long)n * Ho + oy) * Wo + ox) * kStemCo);
#pragma unroll
    for (int k = 0; k < kStemCo / 8; ++k) dst[k] = packed[k];
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

// grid (ceil(dst_w/32), ceil(dst_h/8), max_crops), block (32, 8). Crops at or
// beyond *d_n_crops exit. Arithmetic as batch_roi_warp_kernel.
__global__ void __launch_bounds__(256)
roi_warp_kernel(const uint8_t *__restrict__ pages, long long page_stride, int src_h, int src_w,
                int src_step, const float *__restrict__ minv, const int *__restrict__ crop_w,
                const int *__restrict__ crop_page, const int *__restrict__ n_crops,
                __half *__restrict__ dst, int dst_h, int dst_w, RecNorm nm) {
  const int b = blockIdx.z;
  if (b >= *n_crops) return;
  __shared__ float s_M[9];
  __shared__ int s_crop_w, s_page;
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  if (tid < 9) s_M[tid] = minv[(long long)b * 9 + tid];
  if (tid == 0) { s_crop_w = crop_w[b]; s_page = crop_page[b]; }
  __syncthreads();
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  const int y = blockIdx.y * blockDim.y + threadIdx.y;
  if (x >= dst_w || y >= dst_h) return;
  const long long plane = (long long)dst_h * dst_w;
  __half *o = dst + (long long)b * 3 * plane + (long long)y * dst_w + x;
  if (x >= s_crop_w) {
    o[0] = __float2half_rn(0.f); o[plane] = __float2half_rn(0.f); o[2 * plane] = __float2half_rn(0.f);
    return;
  }
  float denom = s_M[6] * x + s_M[7] * y + s_M[8];
  denom = copysignf(fmaxf(fabsf(denom), 1e-7f), denom);
  const float inv_denom = 1.0f / denom;
  float sx = (s_M[0] * x + s_M[1] * y + s_M[2]) * inv_denom;
  float sy = (s_M[3] * x + s_M[4] * y + s_M[5]) * inv_denom;
  if (!isfinite(sx) || !isfinite(sy)) {
    o[0] = __float2half_rn(0.f); o[plane] = __float2half_rn(0.f); o[2 * plane] = __float2half_rn(0.f);
    return;
  }
  sx = fminf(fmaxf(sx, -1.0f), (float)(src_w + 1));
  sy = fminf(fmaxf(sy, -1.0f), (float)(src_h + 1));
  int xl = (int)floorf(sx), yl = (int)floorf(sy);
  int xh = xl + 1, yh = yl + 1;
  const float dx = sx - xl, dy = sy - yl;
  xl = min(max(xl, 0), src_w - 1); xh = min(max(xh, 0), src_w - 1);
  yl = min(max(yl, 0), src_h - 1); yh = min(max(yh, 0), src_h - 1);
  const uint8_t *src = pages + (long long)s_page * page_stride;
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
  o[plane] = __float2half_rn((g * nm.inv_scale - nm.mean[1]) * nm.inv_std[1]);
  o[2 * plane] = __float2half_rn((bl * nm.inv_scale - nm.mean[2]) * nm.inv_std[2]);
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
  const dim3 grid((w + kInkTile - 1) / kInkTile, h, n);
  ink_kernel<<<grid, kInkTile, 0, as_stream(stream)>>>(d_pages, h, w, page_stride, d_prob, gain);
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
  const dim3 grid((dst_w + 31) / 32, (dst_h + 7) / 8, max_crops);
  roi_warp_kernel<<<grid, block, 0, as_stream(stream)>>>(d_pages, page_stride, src_h, src_w,
                                                         src_step, d_minv, d_crop_w, d_crop_page,
                                                         d_n_crops, (__half *)d_dst, dst_h, dst_w, nm);
  return check_launch("roi_warp_kernel");
}

}  // extern "C"
