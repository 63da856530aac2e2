// C-ABI over the detection resize policy (include/turbo_ocr/detection/det_config.h),
// so ctypes callers and the benchmark use the same arithmetic as the C++ modules.
#include <climits>

#include "tocr_capi.h"
#include "turbo_ocr/detection/det_config.h"

namespace {
namespace det = turbo_ocr::detection;
det::DetResizeParams make(int limit_max, int len, int cap) {
  return {limit_max ? "max" : "min", len, cap};
}
}  // namespace

extern "C" {

TOCR_API int tocr_compute_det_resize(int h, int w, int limit_max, int limit_side_len,
                                     int max_side_limit, int *out_h, int *out_w) {
  if (h <= 0 || w <= 0 || limit_side_len <= 0 || max_side_limit <= 0 || !out_h || !out_w)
    return TOCR_ERR_INVALID;
  const auto [rh, rw] = det::compute_det_resize(h, w, make(limit_max, limit_side_len,
                                                           max_side_limit));
  *out_h = rh;
  *out_w = rw;
  return TOCR_OK;
}

TOCR_API int tocr_read_det_resize(int *limit_max, int *limit_side_len, int *max_side_limit) {
  if (!limit_max || !limit_side_len || !max_side_limit) return TOCR_ERR_INVALID;
  const det::DetResizeParams p =
      det::read_det_resize(make(*limit_max, *limit_side_len, *max_side_limit));
  *limit_max = p.limit_type[1] == 'a' ? 1 : 0;
  *limit_side_len = p.limit_side_len;
  *max_side_limit = p.max_side_limit;
  return TOCR_OK;
}

TOCR_API int tocr_effective_det_max_side(int max_side_limit) {
  return det::effective_det_max_side(make(0, 64, max_side_limit));
}

TOCR_API int tocr_read_db_params(float *thresh, float *box_thresh, float *unclip_ratio) {
  if (!thresh || !box_thresh || !unclip_ratio) return TOCR_ERR_INVALID;
  const det::DbParams p = det::read_db_params({*thresh, *box_thresh, *unclip_ratio});
  *thresh = p.thresh;
  *box_thresh = p.box_thresh;
  *unclip_ratio = p.unclip_ratio;
  return TOCR_OK;
}

}  // extern "C"
