// The part of the reference's pipeline result (include/turbo_ocr/pipeline/
// pipeline_result.h) that the det+rec path fills: recognised items and the
// text-degraded flag with its warning.
#pragma once

#include <string>
#include <vector>

#include "turbo_ocr/common/types.h"

namespace turbo_ocr::pipeline {

struct OcrPipelineResult {
  std::vector<OCRResultItem> results;
  bool text_degraded = false;
  std::string text_warning;
};

}  // namespace turbo_ocr::pipeline
