// Subsystem 1 — batched det preprocessing (resize + letterbox + normalise).
//
// Reference arithmetic (TurboOCR):
//   bilinear_sample_bgr .............. src/kernels/preprocess_kernels.cu:19-54
//   batch kernel + letterbox pad ..... src/kernels/preprocess_kernels.cu:128-178
//   host wrapper / det mean & std .... src/kernels/preprocess_kernels.cu:180-201
// The per-pixel formula is kept operation for operation (same tap formula,
// same weight products, same accumulation order, same normalisation), so the
// fp32 value is the reference's and the fp16 output is its round-to-nearest.
//
// B200 design: each thread owns 2 neighbouring canvas columns, so the lanes
// of a warp cover 64 consecutive columns: their bilinear taps fall in one
// short, contiguous span of each source row (a few L1 wavefronts per byte
// load, not one cache line per lane), and each plane is written as one
// 4-byte pair per lane (128 contiguous bytes per warp for fp16). The x-taps
// of a thread's 2 columns are computed once and reused for every row of the
// CTA's band (8 rows), which takes the float->int conversions off the
// per-pixel path. Source bytes become floats with the exact 2^23
// magic-number trick instead of the quarter-rate I2F conversion.
#include "tocr_common.cuh"

namespace tocr {
namespace {

constexpr int kPrepThreads = 160;  // pairs of columns per CTA (320 columns)
constexpr int kPrepCols = 2;       // columns per thread
constexpr int kPrepRows = 8;       // canvas rows per CTA

__device__ __forceinline__ float u8f(uint32_t b) {
  // 0x4B000000 is 2^23: (2^23 + b) - 2^23 == b exactly for 0 <= b < 2^23.
  return __int_as_float(0x4B000000 | b) - 8388608.f;
}

template <typename OutT>
struct Store2;
template <>
struct Store2<__half> {
  static __device__ __forceinline__ void put(__half *p, const float v[2]) {
    *reinterpret_cast<__half2 *>(p) = __floats2half2_rn(v[0], v[1]);
  }
};
template <>
struct Store2<float> {
  static __device__ __forceinline__ void put(float *p, const float v[2]) {
    *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
  }
};
struct Norm {
  float mean[3];
  float inv_std[3];
};

// One image's source and letterbox content size.
struct SrcDesc {
  const void *ptr;
  int step, h, w, dh, dw;
};

template <typename OutT>
__device__ __forceinline__ void preprocess_image_rows(const SrcDesc d, int b, OutT *__restrict__ dst,
                                                      int W, int H, const Norm &nm);

template <typename OutT>
__global__ void __launch_bounds__(kPrepThreads)
preprocess_batch_kernel(const void *const *__restrict__ src_ptrs,
                        const int *__restrict__ src_steps, const int *__restrict__ src_hs,
                        const int *__restrict__ src_ws, const int *__restrict__ dst_hs,
                        const int *__restrict__ dst_ws, OutT *__restrict__ dst, int W, int H,
                        Norm nm) {
  const int b = blockIdx.z;
  if ((blockIdx.x * kPrepThreads + threadIdx.x) * kPrepCols >= W) return;
  const SrcDesc d{src_ptrs[b], src_steps[b], src_hs[b], src_ws[b], dst_hs[b], dst_ws[b]};
  preprocess_image_rows<OutT>(d, b, dst, W, H, nm);
}

// The single-image form (cuda_fused_resize_normalize_det): the descriptor is
// a kernel parameter, so nothing is staged in device memory.
template <typename OutT>
__global__ void __launch_bounds__(kPrepThreads)
preprocess_one_kernel(SrcDesc d, OutT *__restrict__ dst, int W, int H, Norm nm) {
  if ((blockIdx.x * kPrepThreads + threadIdx.x) * kPrepCols >= W) return;
  preprocess_image_rows<OutT>(d, 0, dst, W, H, nm);
}

template <typename OutT>
__device__ __forceinline__ void preprocess_image_rows(const SrcDesc d, int b, OutT *__restrict__ dst,
                                                      int W, int H, const Norm &nm) {
  const int gx = blockIdx.x * kPrepThreads + threadIdx.x;
  const int x_base = gx * kPrepCols;
  const unsigned char *src = static_cast<const unsigned char *>(d.ptr);
  const int src_step = d.step;
  const int src_h = d.h;
  const int src_w = d.w;
  const int content_h = d.dh;
  const int content_w = d.dw;

  const float inv_255 = 1.0f / 255.0f;
  const float pad0 = (0.0f - nm.mean[0]) * nm.inv_std[0];
  const float pad1 = (0.0f - nm.mean[1]) * nm.inv_std[1];
  const float pad2 = (0.0f - nm.mean[2]) * nm.inv_std[2];

  const bool has_content = content_w > 0 && content_h > 0 && src_w > 0 && src_h > 0;
  const float scale_x = has_content ? (float)src_w / content_w : 0.f;
  const float scale_y = has_content ? (float)src_h / content_h : 0.f;

  // x-taps of this thread's columns (byte offsets of the two taps).
  int xo0[kPrepCols], xo1[kPrepCols];
  float fxs[kPrepCols];
#pragma unroll
  for (int j = 0; j < kPrepCols; ++j) {
    const int dx = x_base + j;
    float sx = (dx + 0.5f) * scale_x - 0.5f;
    int x0 = (int)floorf(sx);
    fxs[j] = sx - x0;
    int x1 = x0 + 1;
    x0 = max(0, min(x0, src_w - 1));
    x1 = max(0, min(x1, src_w - 1));
    xo0[j] = x0 * 3;
    xo1[j] = x1 * 3;
  }

  const size_t plane = (size_t)H * W;
  OutT *out0 = dst + (size_t)b * 3 * plane + x_base;
  const int y_begin = blockIdx.y * kPrepRows;
  const int y_end = min(H, y_begin + kPrepRows);

  for (int dy = y_begin; dy < y_end; ++dy) {
    float c0[kPrepCols], c1[kPrepCols], c2[kPrepCols];
    if (!has_content || dy >= content_h || x_base >= content_w) {
#pragma unroll
      for (int j = 0; j < kPrepCols; ++j) { c0[j] = pad0; c1[j] = pad1; c2[j] = pad2; }
    } else {
      float sy = (dy + 0.5f) * scale_y - 0.5f;
      int y0 = (int)floorf(sy);
      const float fy = sy - y0;
      int y1 = y0 + 1;
      y0 = max(0, min(y0, src_h - 1));
      y1 = max(0, min(y1, src_h - 1));
      const unsigned char *row0 = src + (size_t)y0 * src_step;
      const unsigned char *row1 = src + (size_t)y1 * src_step;
#pragma unroll
      for (int j = 0; j < kPrepCols; ++j) {
        if (x_base + j >= content_w) { c0[j] = pad0; c1[j] = pad1; c2[j] = pad2; continue; }
        const float fx = fxs[j];
        const unsigned char *p00 = row0 + xo0[j], *p10 = row0 + xo1[j];
        const unsigned char *p01 = row1 + xo0[j], *p11 = row1 + xo1[j];
        const float w00 = (1.0f - fx) * (1.0f - fy);
        const float w10 = fx * (1.0f - fy);
        const float w01 = (1.0f - fx) * fy;
        const float w11 = fx * fy;
        float v[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          v[c] = w00 * u8f(__ldg(p00 + c)) + w10 * u8f(__ldg(p10 + c)) +
                 w01 * u8f(__ldg(p01 + c)) + w11 * u8f(__ldg(p11 + c));
        }
        c0[j] = (v[0] * inv_255 - nm.mean[0]) * nm.inv_std[0];
        c1[j] = (v[1] * inv_255 - nm.mean[1]) * nm.inv_std[1];
        c2[j] = (v[2] * inv_255 - nm.mean[2]) * nm.inv_std[2];
      }
    }
    OutT *o = out0 + (size_t)dy * W;
    Store2<OutT>::put(o, c0);
    Store2<OutT>::put(o + plane, c1);
    Store2<OutT>::put(o + 2 * plane, c2);
  }
}

Norm make_norm(const float *mean3, const float *inv_std3) {
  Norm n;
  const float dm[3] = {0.485f, 0.456f, 0.406f};
  const float ds[3] = {1.0f / 0.229f, 1.0f / 0.224f, 1.0f / 0.225f};
  for (int c = 0; c < 3; ++c) {
    n.mean[c] = mean3 ? mean3[c] : dm[c];
    n.inv_std[c] = inv_std3 ? inv_std3[c] : ds[c];
  }
  return n;
}

template <typename OutT>
int launch_preprocess(const void *const *d_src_ptrs, const int *d_src_steps,
                      const int *d_src_heights, const int *d_src_widths,
                      const int *d_dst_heights, const int *d_dst_widths, OutT *dst,
                      int dst_w, int dst_h, int batch_size, const float *mean3,
                      const float *inv_std3, void *stream, const char *name) {
  TOCR_REQUIRE(batch_size >= 0 && dst_w >= 0 && dst_h >= 0, "%s: negative size", name);
  if (batch_size == 0 || dst_w == 0 || dst_h == 0) return TOCR_OK;
  TOCR_REQUIRE(batch_size <= 65535, "%s: batch_size %d > 65535", name, batch_size);
  TOCR_REQUIRE(dst_w % 8 == 0, "%s: dst_w %d must be a multiple of 8", name, dst_w);
  TOCR_REQUIRE(d_src_ptrs && d_src_steps && d_src_heights && d_src_widths &&
                   d_dst_heights && d_dst_widths && dst,
               "%s: null pointer", name);
  TOCR_REQUIRE(aligned(dst, 16), "%s: dst must be 16-byte aligned", name);
  if ((size_t)dst_w * dst_h > (size_t)INT_MAX)
    return set_error(TOCR_ERR_OVERFLOW, "%s: canvas %dx%d too large", name, dst_w, dst_h);
  dim3 grid((dst_w / kPrepCols + kPrepThreads - 1) / kPrepThreads, (dst_h + kPrepRows - 1) / kPrepRows,
            batch_size);
  TOCR_REQUIRE(grid.y <= 65535, "%s: dst_h %d too large", name, dst_h);
  preprocess_batch_kernel<OutT><<<grid, kPrepThreads, 0, as_stream(stream)>>>(
      d_src_ptrs, d_src_steps, d_src_heights, d_src_widths, d_dst_heights, d_dst_widths, dst,
      dst_w, dst_h, make_norm(mean3, inv_std3));
  return check_launch(name);
}

template <typename OutT>
int launch_preprocess_one(const void *src, int step, int h, int w, OutT *dst, int dst_w,
                          int dst_h, const float *mean3, const float *inv_std3, void *stream,
                          const char *name) {
  TOCR_REQUIRE(dst_w >= 0 && dst_h >= 0 && h >= 0 && w >= 0 && step >= 0, "%s: negative size",
               name);
  if (dst_w == 0 || dst_h == 0) return TOCR_OK;
  TOCR_REQUIRE(dst_w % 8 == 0, "%s: dst_w %d must be a multiple of 8", name, dst_w);
  TOCR_REQUIRE(dst && (src || h == 0 || w == 0), "%s: null pointer", name);
  TOCR_REQUIRE(aligned(dst, 16), "%s: dst must be 16-byte aligned", name);
  if ((size_t)dst_w * dst_h > (size_t)INT_MAX)
    return set_error(TOCR_ERR_OVERFLOW, "%s: canvas %dx%d too large", name, dst_w, dst_h);
  dim3 grid((dst_w / kPrepCols + kPrepThreads - 1) / kPrepThreads, (dst_h + kPrepRows - 1) / kPrepRows,
            1);
  TOCR_REQUIRE(grid.y <= 65535, "%s: dst_h %d too large", name, dst_h);
  const SrcDesc d{src, step, h, w, dst_h, dst_w};
  preprocess_one_kernel<OutT><<<grid, kPrepThreads, 0, as_stream(stream)>>>(
      d, dst, dst_w, dst_h, make_norm(mean3, inv_std3));
  return check_launch(name);
}

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API int tocr_preprocess_batch_f16(const void *const *d_src_ptrs, const int *d_src_steps,
                                       const int *d_src_heights, const int *d_src_widths,
                                       const int *d_dst_heights, const int *d_dst_widths,
                                       void *dst_f16, int dst_w, int dst_h, int batch_size,
                                       const float *mean3, const float *inv_std3,
                                       void *stream) {
  TOCR_ENTRY();
  return launch_preprocess<__half>(d_src_ptrs, d_src_steps, d_src_heights, d_src_widths,
                                   d_dst_heights, d_dst_widths, static_cast<__half *>(dst_f16),
                                   dst_w, dst_h, batch_size, mean3, inv_std3, stream,
                                   "tocr_preprocess_batch_f16");
}

TOCR_API int tocr_preprocess_batch_f32(const void *const *d_src_ptrs, const int *d_src_steps,
                                       const int *d_src_heights, const int *d_src_widths,
                                       const int *d_dst_heights, const int *d_dst_widths,
                                       float *dst_f32, int dst_w, int dst_h, int batch_size,
                                       const float *mean3, const float *inv_std3,
                                       void *stream) {
  TOCR_ENTRY();
  return launch_preprocess<float>(d_src_ptrs, d_src_steps, d_src_heights, d_src_widths,
                                  d_dst_heights, d_dst_widths, dst_f32, dst_w, dst_h,
                                  batch_size, mean3, inv_std3, stream,
                                  "tocr_preprocess_batch_f32");
}

TOCR_API int tocr_preprocess_one_f32(const void *d_src, int src_step, int src_h, int src_w,
                                     float *dst_f32, int dst_w, int dst_h, const float *mean3,
                                     const float *inv_std3, void *stream) {
  TOCR_ENTRY();
  return launch_preprocess_one<float>(d_src, src_step, src_h, src_w, dst_f32, dst_w, dst_h, mean3,
                                      inv_std3, stream, "tocr_preprocess_one_f32");
}

TOCR_API int tocr_preprocess_one_f16(const void *d_src, int src_step, int src_h, int src_w,
                                     void *dst_f16, int dst_w, int dst_h, const float *mean3,
                                     const float *inv_std3, void *stream) {
  TOCR_ENTRY();
  return launch_preprocess_one<__half>(d_src, src_step, src_h, src_w,
                                       static_cast<__half *>(dst_f16), dst_w, dst_h, mean3,
                                       inv_std3, stream, "tocr_preprocess_one_f16");
}

}  // extern "C"
