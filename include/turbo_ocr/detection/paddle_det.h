// The detection module of the reference (include/turbo_ocr/detection/
// paddle_det.h:20-44) on this library's kernels: the same public methods and
// semantics (resize policy with environment overrides, letterboxed batches
// of at most 8 images, one more image per call through the single-image
// path, DB post-processing with the reference's box geometry), with every
// device and pinned buffer allocated once by load_model.
//
// The network stage: the reference runs a TensorRT DB network; its trained
// weights are not available here, so the only model this build loads is
// "synthetic", the stand-in DB head of the benchmark's synthetic pages
// (tocr_det_standin_prob_f32). Every other stage is the product path.
// One instance per thread (not thread-safe), as in the reference.
#pragma once

#include <memory>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "turbo_ocr/common/geometry/box.h"
#include "turbo_ocr/decode/gpu_image.h"
#include "turbo_ocr/detection/det_config.h"

namespace turbo_ocr::detection {

class PaddleDet {
 public:
  PaddleDet();
  ~PaddleDet() noexcept;
  PaddleDet(const PaddleDet &) = delete;
  PaddleDet &operator=(const PaddleDet &) = delete;

  // resize / db are the model's base config; DET_* environment variables
  // override them (read_det_resize, read_db_params). Returns false when the
  // model cannot be loaded (only "synthetic" exists in this build).
  [[nodiscard]] bool load_model(const std::string &model_path,
                                const DetResizeParams &resize = kDetResizeDefault,
                                const DbParams &db = kDbDefaults);

  // One image: resized to compute_det_resize(orig_h, orig_w) (no letterbox),
  // boxes in original image coordinates, in the reference's contour order.
  [[nodiscard]] std::vector<Box> run(const GpuImage &gpu_img, int orig_h, int orig_w,
                                     cudaStream_t stream = 0);

  // Up to 8 images letterboxed into one canvas (max of their /32 sizes); the
  // rest go through run(). One result vector per image, in input order.
  [[nodiscard]] std::vector<std::vector<Box>> run_batch(
      const std::vector<GpuImage> &gpu_imgs, const std::vector<std::pair<int, int>> &orig_dims,
      cudaStream_t stream = 0);

  // box_score_fast of every box of the last run / run_batch (per image).
  [[nodiscard]] const std::vector<std::vector<float>> &last_scores() const;
  [[nodiscard]] const DetResizeParams &resize_params() const;
  [[nodiscard]] const DbParams &db_params() const;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

}  // namespace turbo_ocr::detection
