// Non-owning device image descriptor with the reference layout
// (include/turbo_ocr/decode/gpu_image.h:9-16 in TurboOCR): u8 HWC pixels,
// `step` bytes between rows.
#pragma once
#include <cstddef>

namespace turbo_ocr::decode {
struct GpuImage {
  void *data = nullptr;
  std::size_t step = 0;
  int rows = 0;
  int cols = 0;
  [[nodiscard]] constexpr bool empty() const noexcept {
    return data == nullptr || rows == 0 || cols == 0;
  }
};
}  // namespace turbo_ocr::decode

namespace turbo_ocr {
using decode::GpuImage;
}
