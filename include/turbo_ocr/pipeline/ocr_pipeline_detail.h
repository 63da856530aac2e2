// The combine step of the reference's pipelines
// (src/pipeline/ocr/ocr_pipeline_detail.h:19-60): pair recognition output
// with its boxes, drop empty or low-confidence results, flag degraded pages.
#pragma once

#include <algorithm>
#include <cstddef>
#include <string>
#include <utility>
#include <vector>

#include "turbo_ocr/common/types.h"
#include "turbo_ocr/pipeline/pipeline_result.h"

namespace turbo_ocr::pipeline::detail {

// Boxes were found but nothing readable came back: never a clean empty page.
inline void flag_text_degraded(OcrPipelineResult &out, std::size_t num_boxes) {
  if (num_boxes > 0 && out.results.empty()) {
    out.text_degraded = true;
    out.text_warning = "text stage degraded: detection found " + std::to_string(num_boxes) +
                       " text region(s) but recognition produced no usable text "
                       "(all crops decoded empty/blank; not a genuinely blank page)";
  }
}

// Crops the recognizer had to skip also mark the page degraded.
inline void flag_dropped_crops(OcrPipelineResult &out, int dropped) {
  if (dropped <= 0) return;
  out.text_degraded = true;
  const std::string w = "text stage degraded: recognition dropped " + std::to_string(dropped) +
                        " crop(s) (engine output exceeded decode buffers)";
  out.text_warning = out.text_warning.empty() ? w : out.text_warning + "; " + w;
}

// Keeps result i when its confidence is >= kDropScore and its text is not
// empty; then applies flag_text_degraded.
inline void combine_recognition(OcrPipelineResult &out, const std::vector<Box> &boxes,
                                std::vector<std::pair<std::string, float>> &rec_results) {
  out.results.reserve(out.results.size() + boxes.size());
  const std::size_t n = std::min(boxes.size(), rec_results.size());
  for (std::size_t i = 0; i < n; ++i) {
    if (rec_results[i].second < turbo_ocr::kDropScore) continue;
    if (rec_results[i].first.empty()) continue;
    OCRResultItem item;
    item.text = std::move(rec_results[i].first);
    item.confidence = rec_results[i].second;
    item.box = boxes[i];
    out.results.push_back(std::move(item));
  }
  flag_text_degraded(out, boxes.size());
}

}  // namespace turbo_ocr::pipeline::detail
