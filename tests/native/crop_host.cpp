// Test-only host build of turboocr_b200/csrc/crop_geom.cuh (the device crop
// transform), compared by the CPU tests with the reference's own header.
#include "crop_geom.cuh"

extern "C" int crop_host_transform(const int *box8, int target_h, int max_width, float *m9,
                                   int *crop_w, int *vertical) {
  tocr::crop::crop_transform(box8, target_h, max_width, m9, crop_w, vertical);
  return 0;
}
