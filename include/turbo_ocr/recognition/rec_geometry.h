// Recognizer input widths of the reference
// (include/turbo_ocr/recognition/rec_geometry.h:23-67).
#pragma once

#include <algorithm>
#include <array>

#include "turbo_ocr/common/geometry/perspective.h"
#include "turbo_ocr/common/types.h"

namespace turbo_ocr::recognition {

inline constexpr int kMaxRecWidth = 4000;  // every crop width is clamped here
inline constexpr int kMinRecWidth = 32;    // narrower crops are right-padded
inline constexpr std::array kRecWidthBuckets = {320, 480, 800, 1200, 1600, 2000, 2500, 3200, 4000};
static_assert(kRecWidthBuckets.back() == kMaxRecWidth, "the buckets cover every width");

// The crop's natural width (after the vertical swap) from the same transform
// the warp uses, at least kMinRecWidth.
[[nodiscard]] inline int rec_input_width(const turbo_ocr::Box &box, int rec_image_h) {
  return std::max(turbo_ocr::compute_crop_transform(box, rec_image_h, kMaxRecWidth).crop_width,
                  kMinRecWidth);
}

// The smallest bucket >= w (w clamped to kMaxRecWidth).
[[nodiscard]] inline int snap_width_bucket(int w) {
  return *std::lower_bound(kRecWidthBuckets.begin(), kRecWidthBuckets.end(),
                           std::min(w, kMaxRecWidth));
}

// w rounded up to a multiple of step, at most kMaxRecWidth, never below w.
[[nodiscard]] inline int snap_width_step(int target_w, int step) {
  int b = target_w;
  if (step > 1) b = (target_w + step - 1) / step * step;
  b = std::min(b, kMaxRecWidth);
  return std::max(b, target_w);
}

}  // namespace turbo_ocr::recognition
