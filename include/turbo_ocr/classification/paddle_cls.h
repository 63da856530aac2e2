// The 0/180-degree text-line classifier module of the reference
// (include/turbo_ocr/classification/paddle_cls.h:15-55,
// src/classification/paddle_cls.cpp:43-103) on this library's kernels: the
// same public methods and semantics. Boxes go in batches of at most 128;
// each is cropped to 80 x 160 with its crop transform and the recognizer's
// normalisation ((p/255 - 0.5) / 0.5, as the reference's classifier uses),
// the network gives (score_0, score_180), and a box whose score_180 is above
// score_0 and above 0.9 gets its corners rotated by two ([tl, tr, br, bl] ->
// [br, bl, tl, tr]). run() synchronises the stream once per batch.
//
// The network: the reference runs PP-LCNet textline orientation in TensorRT;
// its weights are not available here, so the one model this build loads is
// "synthetic": a 3x3 stride-2 conv stem (3 -> 32, hardswish), five
// DW3x3+PW1x1 INT8 blocks (32->64, 64->64 s2, 64->128, 128->128 s2,
// 128->256; tocr_dwpw_block) and global average pool + FC 256 -> 2 +
// softmax, with seeded weights (tocr_synth_weights; the seeds and scales are
// listed in tocr_capi.h beside tocr_cls_stem_f16).
// One instance per thread (not thread-safe), as in the reference.
#pragma once

#include <array>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "turbo_ocr/common/geometry/box.h"
#include "turbo_ocr/decode/gpu_image.h"

namespace turbo_ocr::classification {

class PaddleCls {
 public:
  PaddleCls();
  ~PaddleCls() noexcept;
  PaddleCls(const PaddleCls &) = delete;
  PaddleCls &operator=(const PaddleCls &) = delete;

  // Only "synthetic" loads in this build; false otherwise.
  [[nodiscard]] bool load_model(const std::string &model_path);

  // Classify the crops of `boxes` in `img` and rotate the 180-degree ones in
  // place.
  void run(const GpuImage &img, std::vector<Box> &boxes, cudaStream_t stream = 0);

  // Allocates every device and pinned buffer (the reference's warm-up call).
  void allocate_buffers();

  // (score_0, score_180) of every box of the last run(), in box order.
  [[nodiscard]] const std::vector<std::array<float, 2>> &last_scores() const;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

}  // namespace turbo_ocr::classification
