// Detection post-processing entry points of the reference
// (include/turbo_ocr/detection/det_postprocess.h:14-41) that carry no OpenCV
// types. extract_boxes_from_bitmap, box_score_fast, unclip and
// get_mini_boxes take cv::Mat / cv::Point there; this library runs that whole
// step on the device instead (tocr_db_postprocess in tocr_capi.h, bit-exact
// with it), which PaddleDet calls, so no OpenCV type appears here.
#pragma once

#include "turbo_ocr/common/geometry/box.h"

namespace turbo_ocr::detection {

// Orders 4 corners in place as [tl, tr, br, bl]: stable sort by x, the left
// pair split into tl/bl by y, the right pair into tr/br.
void order_quad_tl_tr_br_bl(float xs[4], float ys[4]) noexcept;

}  // namespace turbo_ocr::detection
