// Text-line orientation classifier options of the reference
// (include/turbo_ocr/classification/cls_options.h:13-34 in TurboOCR).
#pragma once

#include <cctype>
#include <cstdlib>
#include <string>

namespace turbo_ocr::classification {

// 1 / true / yes / on (any case) are true; everything else, unset included,
// is false.
[[nodiscard]] inline bool truthy_env_value(const char *v) {
  if (!v || !*v) return false;
  std::string s(v);
  for (char &ch : s) ch = static_cast<char>(std::tolower(static_cast<unsigned char>(ch)));
  return s == "1" || s == "true" || s == "yes" || s == "on";
}

// CLS_ALL_BOXES: classify every crop, not only the vertical-looking ones
// (read once per process, as the reference does).
[[nodiscard]] inline bool cls_all_boxes_enabled() {
  static const bool on = truthy_env_value(std::getenv("CLS_ALL_BOXES"));
  return on;
}

}  // namespace turbo_ocr::classification
