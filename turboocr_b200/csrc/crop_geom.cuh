// Crop geometry of the recognition stage, written once for the device
// (crop.cu) and for a host build used by the CPU tests:
//   compute_crop_transform ... include/turbo_ocr/common/geometry/perspective.h:25-67
//   compute_perspective_inv .. include/turbo_ocr/common/geometry/perspective_math.h:16-47
// The reference compiles these host functions with GCC -O3 -march=x86-64-v3,
// which fuses a*b+c into FMAs; the restatement writes those FMAs as fma() and
// is compiled without any other contraction (-fmad=false / -ffp-contract=off).
#pragma once

#include <cmath>

#if defined(__CUDACC__)
#define TGC __host__ __device__ __forceinline__
#else
#define TGC inline
#endif

namespace tocr {
namespace crop {

constexpr float kVerticalAspectRatio = 1.5f;  // box.h:30

// 8x8 Gauss-Jordan with partial pivoting in double: maps the dst quad to the
// src quad. M[9] row-major, M[8] = 1.
TGC void perspective_inv(const float *dst_pts, const float *src_pts, float *M) {
  const double x0 = dst_pts[0], y0 = dst_pts[1], x1 = dst_pts[2], y1 = dst_pts[3];
  const double x2 = dst_pts[4], y2 = dst_pts[5], x3 = dst_pts[6], y3 = dst_pts[7];
  const double u0 = src_pts[0], v0 = src_pts[1], u1 = src_pts[2], v1 = src_pts[3];
  const double u2 = src_pts[4], v2 = src_pts[5], u3 = src_pts[6], v3 = src_pts[7];
  double A[8][8] = {{x0, y0, 1, 0, 0, 0, -x0 * u0, -y0 * u0}, {x1, y1, 1, 0, 0, 0, -x1 * u1, -y1 * u1},
                    {x2, y2, 1, 0, 0, 0, -x2 * u2, -y2 * u2}, {x3, y3, 1, 0, 0, 0, -x3 * u3, -y3 * u3},
                    {0, 0, 0, x0, y0, 1, -x0 * v0, -y0 * v0}, {0, 0, 0, x1, y1, 1, -x1 * v1, -y1 * v1},
                    {0, 0, 0, x2, y2, 1, -x2 * v2, -y2 * v2}, {0, 0, 0, x3, y3, 1, -x3 * v3, -y3 * v3}};
  double b[8] = {u0, u1, u2, u3, v0, v1, v2, v3};
  for (int col = 0; col < 8; ++col) {
    int piv = col;
    double mx = fabs(A[col][col]);
    for (int r = col + 1; r < 8; ++r)
      if (fabs(A[r][col]) > mx) { mx = fabs(A[r][col]); piv = r; }
    if (piv != col) {
      const double tb = b[col]; b[col] = b[piv]; b[piv] = tb;
      for (int k = 0; k < 8; ++k) { const double t = A[col][k]; A[col][k] = A[piv][k]; A[piv][k] = t; }
    }
    double d = A[col][col];
    if (fabs(d) < 1e-12) d = (d < 0) ? -1e-12 : 1e-12;
    for (int k = col; k < 8; ++k) A[col][k] /= d;
    b[col] /= d;
    for (int r = 0; r < 8; ++r) {
      if (r == col) continue;
      const double f = A[r][col];
      for (int k = col; k < 8; ++k) A[r][k] = fma(-f, A[col][k], A[r][k]);
      b[r] = fma(-f, b[col], b[r]);
    }
  }
  for (int i = 0; i < 8; ++i) M[i] = (float)b[i];
  M[8] = 1.0f;
}

// compute_crop_transform: box int [4][2] (tl tr br bl) -> M_inv, crop width,
// vertical flag.
TGC void crop_transform(const int *box, int target_h, int max_width, float *M, int *crop_w,
                        int *vertical) {
  const float bx0 = (float)box[0], by0 = (float)box[1], bx1 = (float)box[2], by1 = (float)box[3];
  const float bx2 = (float)box[4], by2 = (float)box[5], bx3 = (float)box[6], by3 = (float)box[7];
  float cw = sqrtf(fmaf(bx0 - bx1, bx0 - bx1, (by0 - by1) * (by0 - by1)));
  float ch = sqrtf(fmaf(bx0 - bx3, bx0 - bx3, (by0 - by3) * (by0 - by3)));
  const bool vert = ch >= cw * kVerticalAspectRatio;
  float src[8];
  if (vert) {
    const float s[8] = {bx3, by3, bx0, by0, bx1, by1, bx2, by2};
    for (int i = 0; i < 8; ++i) src[i] = s[i];
    const float t = cw; cw = ch; ch = t;
  } else {
    const float s[8] = {bx0, by0, bx1, by1, bx2, by2, bx3, by3};
    for (int i = 0; i < 8; ++i) src[i] = s[i];
  }
  const float ar = (ch > 0) ? (cw / ch) : 0.f;
  int rw = (int)ceilf((float)target_h * ar);
  rw = rw < max_width ? rw : max_width;
  rw = rw > 1 ? rw : 1;
  const float fw = (float)rw, fh = (float)target_h;
  const float dst[8] = {0.f, 0.f, fw, 0.f, fw, fh, 0.f, fh};
  perspective_inv(dst, src, M);
  *crop_w = rw;
  *vertical = vert ? 1 : 0;
}

}  // namespace crop
}  // namespace tocr
