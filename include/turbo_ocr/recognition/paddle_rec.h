// The recognition module of the reference (include/turbo_ocr/recognition/
// paddle_rec.h:19-63) on this library's kernels: crops bucketed by width
// (rec_input_width + snap_width_bucket), at most set_batch_num() crops per
// batch of one width, every batch queued without a host round trip into its
// own output slot (20 slots, then one sync and decode), one final
// synchronisation, results in box order. The ROI warp is the reference's
// arithmetic; CTC argmax, max-softmax and collapse run on the device
// (tocr_ctc_greedy_f16) and the host maps tokens to text.
//
// The network stage: the reference runs a TensorRT CRNN whose trained weights
// are not available here; the only model this build loads is "synthetic",
// whose logits (seq_len = width / 4 steps, one class per dictionary entry)
// come from tocr_rec_standin_logits_f16 keyed by the crop's index in the call.
// One instance per thread (not thread-safe), as in the reference.
#pragma once

#include <memory>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "turbo_ocr/common/geometry/box.h"
#include "turbo_ocr/decode/gpu_image.h"
#include "turbo_ocr/recognition/rec_geometry.h"

namespace turbo_ocr::recognition {

class PaddleRec {
 public:
  PaddleRec();
  ~PaddleRec() noexcept;
  PaddleRec(const PaddleRec &) = delete;
  PaddleRec &operator=(const PaddleRec &) = delete;

  // Maximum crops per batch; call before load_model (default 32).
  void set_batch_num(int n);
  [[nodiscard]] bool load_model(const std::string &model_path);
  // ["blank"] + one label per line + [" "] (load_label_dict).
  [[nodiscard]] bool load_dict(const std::string &dict_path);

  [[nodiscard]] std::vector<std::pair<std::string, float>> run(const GpuImage &img,
                                                              const std::vector<Box> &boxes,
                                                              cudaStream_t stream = 0);

  struct ImageCrops {
    GpuImage img;
    std::vector<Box> boxes;
  };
  // All images' crops batched together (by width, then image); one result
  // vector per image in input order.
  [[nodiscard]] std::vector<std::vector<std::pair<std::string, float>>> run_multi(
      const std::vector<ImageCrops> &image_crops, cudaStream_t stream = 0);

  // Allocates every device and pinned buffer (also done by the first run).
  void allocate_buffers();
  // The reference records CUDA graphs of its TensorRT profiles here; the
  // stand-in network has none, so this only allocates.
  void bake_graphs(cudaStream_t stream);

  [[nodiscard]] int last_dropped_crops() const;
  [[nodiscard]] const std::vector<int> &last_dropped_per_image() const;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

}  // namespace turbo_ocr::recognition
