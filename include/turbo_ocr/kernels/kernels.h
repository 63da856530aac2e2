// Reference-signature C++ entry points of the B200 kernels
// (include/turbo_ocr/kernels/kernels.h in TurboOCR). Each function forwards to
// the C-ABI in tocr_capi.h and throws turbo_ocr::CudaError on failure, the
// CUDA_CHECK convention of the reference (common/cuda/cuda_check.h:8-17).
// All work is enqueued asynchronously on `stream`.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "turbo_ocr/common/geometry/perspective_math.h"
#include "turbo_ocr/decode/gpu_image.h"

namespace turbo_ocr::kernels {

using decode::GpuImage;

// kernels.h:19-25 — ROI warp of batch_size crops of one source image into
// [batch][3][dst_h][dst_w] fp32: inverse-perspective bilinear sample, BGR->RGB,
// (p * inv_scale - mean_c) * inv_std_c, zero beyond each crop's width. The
// defaults are the recognizer's (p / 255 - 0.5) / 0.5.
void cuda_batch_roi_warp(const GpuImage &src, const float *d_M_invs, const int *d_crop_widths,
                         float *d_dst_batch, int batch_size, int dst_h, int dst_w,
                         cudaStream_t stream = 0, float mean0 = 0.5f, float mean1 = 0.5f,
                         float mean2 = 0.5f, float inv_std0 = 2.0f, float inv_std1 = 2.0f,
                         float inv_std2 = 2.0f, float inv_scale = 1.0f / 255.0f);

// kernels.h:27-30 — per-row max value + lowest index of the max.
void cuda_argmax(const float *input_probs, int *output_indices, float *output_scores,
                 int batch_size, int seq_len, int num_classes, cudaStream_t stream = 0);

// kernels.h:33-35 — single image, canvas == content, fp32 CHW output.
void cuda_fused_resize_normalize_det(const GpuImage &src, float *dst_chw, int dst_w,
                                     int dst_h, cudaStream_t stream = 0);

// kernels.h:97-102 — batched, letterboxed, fp32 CHW output.
void cuda_batch_fused_resize_normalize_det(const void *const *d_src_ptrs,
                                           const int *d_src_steps, const int *d_src_heights,
                                           const int *d_src_widths, const int *d_dst_heights,
                                           const int *d_dst_widths, float *dst_chw,
                                           int dst_w, int dst_h, int batch_size,
                                           cudaStream_t stream = 0);

// kernels.h:105-107 — batched threshold to a 255/0 bitmap.
void cuda_batch_threshold_to_u8(const float *src, uint8_t *dst, int w, int h, int batch_size,
                                float thresh, cudaStream_t stream = 0);

// kernels.h:110-111
void cuda_threshold_to_u8(const float *src, uint8_t *dst, int w, int h, float thresh,
                          cudaStream_t stream = 0);

// kernels.h:114-118 — forwards to turbo_ocr::compute_perspective_inv.
inline void compute_perspective_inv(const float *dst_pts, const float *src_pts, float *M_inv) {
  turbo_ocr::compute_perspective_inv(dst_pts, src_pts, M_inv);
}

// kernels.h:118-130 — one connected component (resize coordinates).
struct GpuDetBox {
  int xmin, ymin, xmax, ymax;
  float score;      // mean prediction over the component's pixels
  int pixel_count;
  float ox[4], oy[4];  // oriented corners; not filled by cuda_gpu_ccl_detect
};
static constexpr int kMaxGpuComponents = 3000;

// kernels.h:131-145 — 8-connected labelling of the 255/0 bitmap, per-component
// box, pixel count and mean prediction, kept when pixel_count >= 3, both box
// sides >= 3 and mean >= box_thresh. Synchronises `stream` once; returns the
// kept count (also in *h_num_boxes), boxes in h_boxes (at least
// kMaxGpuComponents entries, pinned). Components are numbered in raster order
// of their first pixel, at most kMaxGpuComponents (the reference numbers them
// in an unspecified order, so its output order is unspecified too).
// Buffers: d_labels / d_compact_ids int[w*h], d_id_counter int[1],
// d_bboxes GpuDetBox[2 * kMaxGpuComponents], d_num_boxes int[1]; all
// allocated by the caller. *h_num_total (optional) receives the number of
// components before the cap and the filter.
int cuda_gpu_ccl_detect(const uint8_t *d_bitmap, const float *d_pred_map, int w, int h,
                        float box_thresh, int *d_labels, int *d_compact_ids, int *d_id_counter,
                        GpuDetBox *d_bboxes, int *d_num_boxes, GpuDetBox *h_boxes,
                        int *h_num_boxes, cudaStream_t stream, int *h_num_total = nullptr);

// kernels.h:172-179 — mode-2 growth of every component by its own distance
// (d_expand_per_comp, indexed by compact id): d_expanded_labels = 1 + the
// winning component (0 = none). d_seeds (uint32[w*h]) holds the per-pixel
// winner keys; d_seeds_alt (uint32[w*h], may be null) receives the compacted
// boundary pixels. max_expand is not needed (each disc has its own radius).
void cuda_jfa_expand_labels(const uint8_t *d_bitmap, const int32_t *d_compact_ids,
                            const float *d_expand_per_comp, uint32_t *d_expanded_labels, int w,
                            int h, float max_expand, uint32_t *d_seeds, uint32_t *d_seeds_alt,
                            cudaStream_t stream);

// kernels.h:181-189 — exposed 4-connected crack edges per compact id
// (d_perim_per_comp zeroed here).
void cuda_accumulate_crack_perimeter(const int32_t *d_compact_ids, const uint8_t *d_bitmap,
                                     int w, int h, int num_slots, int *d_perim_per_comp,
                                     cudaStream_t stream);

// kernels.h:191-200 — per-slot growth distance from the PRE-filter boxes of
// cuda_gpu_ccl_detect and the crack perimeters.
void cuda_compute_expand_per_comp(const GpuDetBox *d_bboxes, const int *d_perim_per_comp,
                                  int num_slots, float unclip_ratio, float min_expand,
                                  float max_expand, float box_thresh, float *d_expand_per_comp,
                                  cudaStream_t stream);

// kernels.h:202-209 — box and pixel count of every grown region.
void cuda_jfa_extract_bboxes(const uint32_t *d_expanded_labels, int w, int h,
                             GpuDetBox *d_bboxes, int num_slots, cudaStream_t stream);

// kernels.h:210-229 — box, pixel count and principal-axis rectangle corners
// (ox/oy) of every grown region; d_moments uint64[num_slots*6] and d_orient
// float[num_slots*6] scratch.
void cuda_jfa_extract_oriented(const uint32_t *d_expanded_labels, int w, int h,
                               GpuDetBox *d_bboxes, int num_slots,
                               unsigned long long *d_moments, float *d_orient,
                               cudaStream_t stream);

}  // namespace turbo_ocr::kernels
