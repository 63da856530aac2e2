// Result item and drop score of the reference (include/turbo_ocr/common/types.h:8-26).
#pragma once

#include <string>

#include "turbo_ocr/common/geometry/box.h"

namespace turbo_ocr {

struct OCRResultItem {
  std::string text;
  float confidence = 0.0f;
  Box box{};
  std::string source;  // "" (OCR) or "pdf"
  int id = -1;
  int layout_id = -1;
};

// Recognition results below this confidence are dropped.
inline constexpr float kDropScore = 0.5f;

}  // namespace turbo_ocr
