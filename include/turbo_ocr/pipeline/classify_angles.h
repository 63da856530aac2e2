// The angle-classification step of the reference's GPU pipeline
// (OcrPipeline::classify_angles_, src/pipeline/ocr/ocr_pipeline_runtime.cpp:87-118):
// with CLS_ALL_BOXES every box is classified; otherwise only the boxes that
// look vertical (is_vertical_box) are, and the results go back to their
// positions.
#pragma once

#include <cstddef>
#include <vector>

#include <cuda_runtime.h>

#include "turbo_ocr/classification/cls_options.h"
#include "turbo_ocr/classification/paddle_cls.h"
#include "turbo_ocr/common/geometry/box.h"
#include "turbo_ocr/decode/gpu_image.h"

namespace turbo_ocr::pipeline {

inline void classify_angles(classification::PaddleCls &cls, const GpuImage &img,
                            std::vector<Box> &boxes, cudaStream_t stream) {
  if (boxes.empty()) return;
  if (classification::cls_all_boxes_enabled()) {
    cls.run(img, boxes, stream);
    return;
  }
  std::vector<int> idx;
  std::vector<Box> vert;
  for (int i = 0; i < static_cast<int>(boxes.size()); ++i)
    if (is_vertical_box(boxes[i])) {
      idx.push_back(i);
      vert.push_back(boxes[i]);
    }
  if (idx.empty()) return;
  cls.run(img, vert, stream);
  for (std::size_t j = 0; j < idx.size(); ++j) boxes[idx[j]] = vert[j];
}

}  // namespace turbo_ocr::pipeline
