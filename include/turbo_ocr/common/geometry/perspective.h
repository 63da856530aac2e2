// Crop transform of the reference (include/turbo_ocr/common/geometry/perspective.h:25-67).
#pragma once

#include "turbo_ocr/common/geometry/box.h"
#include "turbo_ocr/common/geometry/perspective_math.h"

namespace turbo_ocr {

struct CropTransform {
  float M_inv[9];  // dst rectangle -> source quad
  int crop_width;  // resized crop width, clamped to [1, max_width]
  bool vertical;   // the box was rotated (vertical text)
};

// Edge lengths of the quad, the vertical swap (h >= 1.5 w), resize width
// ceil(target_h * w / h) clamped to [1, max_width], and the inverse
// perspective transform from (0,0)-(width, target_h) to the quad.
[[nodiscard]] CropTransform compute_crop_transform(const Box &box, int target_h, int max_width);

}  // namespace turbo_ocr
