// Test-infrastructure wrapper (oracle only): the reference's own crop
// geometry, include/turbo_ocr/common/geometry/perspective.h:25-67 and
// perspective_math.h:16-47 (header-only), compiled with the reference's
// flags by oracle/Makefile, behind a C entry point.
#include "turbo_ocr/common/geometry/perspective.h"

extern "C" int crop_ref_transform(const int *box8, int target_h, int max_width, float *m9,
                                  int *crop_w, int *vertical) {
  turbo_ocr::Box b{};
  for (int k = 0; k < 4; ++k) {
    b[k][0] = box8[2 * k];
    b[k][1] = box8[2 * k + 1];
  }
  const turbo_ocr::CropTransform ct = turbo_ocr::compute_crop_transform(b, target_h, max_width);
  for (int i = 0; i < 9; ++i) m9[i] = ct.M_inv[i];
  *crop_w = ct.crop_width;
  *vertical = ct.vertical ? 1 : 0;
  return 0;
}
