// Crop transforms of the recognition stage on the device: one thread per
// detected quad computes compute_crop_transform
// (include/turbo_ocr/common/geometry/perspective.h:25-67) so the crops never
// go through the host. Built with -fmad=false (see crop_geom.cuh).
#include "tocr_common.cuh"

#include "crop_geom.cuh"

namespace tocr {
namespace {

// exclusive scan of per-page box counts -> crop offsets (+ total at [n]).
__global__ void crop_offsets_kernel(const int *__restrict__ counts, int n_pages,
                                    int *__restrict__ crop_off) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int s = 0;
  for (int i = 0; i < n_pages; ++i) {
    crop_off[i] = s;
    s += counts[i];
  }
  crop_off[n_pages] = s;
}

// One thread per (page, box slot); crops are numbered page-major.
__global__ void __launch_bounds__(128)
crop_kernel(const int *__restrict__ boxes, const int *__restrict__ counts,
            const int *__restrict__ crop_off, int n_pages, int max_boxes, int target_h,
            int max_width, float *__restrict__ minv, int *__restrict__ crop_w,
            int *__restrict__ crop_page, int *__restrict__ vertical) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long long)n_pages * max_boxes) return;
  const int pg = (int)(t / max_boxes), k = (int)(t % max_boxes);
  if (k >= counts[pg]) return;
  const int c = crop_off[pg] + k;
  crop::crop_transform(boxes + t * 8, target_h, max_width, minv + (long long)c * 9, crop_w + c,
                       vertical + c);
  crop_page[c] = pg;
}

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API int tocr_crop_transforms(const int *d_boxes, const int *d_counts, int n_pages,
                                  int max_boxes, int target_h, int max_width, int *d_crop_off,
                                  float *d_minv, int *d_crop_w, int *d_crop_page,
                                  int *d_vertical, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n_pages >= 0 && max_boxes > 0 && target_h > 0 && max_width > 0,
               "tocr_crop_transforms: bad sizes");
  if (n_pages == 0) return TOCR_OK;
  cudaStream_t st = as_stream(stream);
  crop_offsets_kernel<<<1, 32, 0, st>>>(d_counts, n_pages, d_crop_off);
  const long long slots = (long long)n_pages * max_boxes;
  crop_kernel<<<(unsigned)((slots + 127) / 128), 128, 0, st>>>(
      d_boxes, d_counts, d_crop_off, n_pages, max_boxes, target_h, max_width, d_minv, d_crop_w,
      d_crop_page, d_vertical);
  return check_launch("crop_kernel");
}

}  // extern "C"
