// Inverse perspective transform of the reference
// (include/turbo_ocr/common/geometry/perspective_math.h:16-47). Compiled in
// the library (8x8 Gauss-Jordan in double, the reference build's fused
// multiply-adds written out), so results do not depend on the caller's
// compiler flags.
#pragma once

namespace turbo_ocr {

// Maps the dst quad to the src quad: M_inv[9], row-major, M_inv[8] = 1.
void compute_perspective_inv(const float *dst_pts, const float *src_pts, float *M_inv);

}  // namespace turbo_ocr
