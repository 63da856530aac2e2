/*
 * ORACLE — test infrastructure only. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg may load it; the product path never does.
 *
 * CPU restatement of the reference's det preprocessing arithmetic:
 *   bilinear_sample_bgr ............ src/kernels/preprocess_kernels.cu:19-54
 *   batch kernel + letterbox ........ src/kernels/preprocess_kernels.cu:128-178
 *   det mean / inv_std constants .... src/kernels/preprocess_kernels.cu:196-200
 * Compiled with -ffp-contract=off; the multiply-adds that nvcc contracts into
 * FMAs in the reference kernel are written as explicit fmaf() calls, so the
 * fp32 result is the reference kernel's value.
 *
 * Parity status: pinned only by restatement (the reference has no test for
 * this kernel); the GPU kernel is checked against it within 1 fp16 ulp.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* One image: src u8 HWC (pitch step), content ch x cw inside a canvas
 * dst_h x dst_w, planar fp32 output dst[3][dst_h][dst_w]. */
void oracle_preprocess_image(const uint8_t *src, int src_h, int src_w, int step, int ch,
                             int cw, float *dst, int dst_h, int dst_w, const float mean[3],
                             const float inv_std[3]) {
  const float inv_255 = 1.0f / 255.0f;
  const size_t plane = (size_t)dst_h * dst_w;
  float scale_x = 0.f, scale_y = 0.f;
  if (cw > 0 && ch > 0) {
    scale_x = (float)src_w / cw;
    scale_y = (float)src_h / ch;
  }
  for (int dy = 0; dy < dst_h; ++dy) {
    for (int dx = 0; dx < dst_w; ++dx) {
      const size_t idx = (size_t)dy * dst_w + dx;
      if (dx >= cw || dy >= ch) {
        for (int c = 0; c < 3; ++c) dst[c * plane + idx] = (0.0f - mean[c]) * inv_std[c];
        continue;
      }
      const float sx = fmaf((float)dx + 0.5f, scale_x, -0.5f);
      const float sy = fmaf((float)dy + 0.5f, scale_y, -0.5f);
      int x0 = (int)floorf(sx);
      int y0 = (int)floorf(sy);
      const float fx = sx - (float)x0;
      const float fy = sy - (float)y0;
      int x1 = x0 + 1, y1 = y0 + 1;
      x0 = clampi(x0, 0, src_w - 1);
      x1 = clampi(x1, 0, src_w - 1);
      y0 = clampi(y0, 0, src_h - 1);
      y1 = clampi(y1, 0, src_h - 1);
      const uint8_t *r0 = src + (size_t)y0 * step;
      const uint8_t *r1 = src + (size_t)y1 * step;
      const float w00 = (1.0f - fx) * (1.0f - fy);
      const float w10 = fx * (1.0f - fy);
      const float w01 = (1.0f - fx) * fy;
      const float w11 = fx * fy;
      for (int c = 0; c < 3; ++c) {
        const float p00 = r0[x0 * 3 + c], p10 = r0[x1 * 3 + c];
        const float p01 = r1[x0 * 3 + c], p11 = r1[x1 * 3 + c];
        /* nvcc (LLVM) contracts fadd(fmul(a,b), fmul(c,d)) into
         * fma(a, b, c*d), then folds each further product term. */
        float v = fmaf(w00, p00, w10 * p10);
        v = fmaf(w01, p01, v);
        v = fmaf(w11, p11, v);
        dst[c * plane + idx] = fmaf(v, inv_255, -mean[c]) * inv_std[c];
      }
    }
  }
}

/* compute_det_resize (include/turbo_ocr/detection/det_config.h:58-81):
 * limit_type 1 = "max", 0 = "min"; writes (resize_h, resize_w). */
static int round32_floor(double v) {
  const int r = (int)(round(v / 32.0) * 32);
  return r > 32 ? r : 32;
}
void oracle_det_resize(int h, int w, int limit_max, int limit_side_len, int max_side_limit,
                       int *out_h, int *out_w) {
  float ratio = 1.0f;
  if (limit_max) {
    const int longest = h > w ? h : w;
    if (longest > limit_side_len) ratio = (float)limit_side_len / longest;
  } else {
    const int shortest = h < w ? h : w;
    if (shortest < limit_side_len) ratio = (float)limit_side_len / shortest;
  }
  int rh = round32_floor((double)(h * ratio));
  int rw = round32_floor((double)(w * ratio));
  const int longest_out = rh > rw ? rh : rw;
  if (longest_out > max_side_limit) {
    const double rescale = (double)max_side_limit / longest_out;
    rh = round32_floor(rh * rescale);
    rw = round32_floor(rw * rescale);
  }
  *out_h = rh;
  *out_w = rw;
}
