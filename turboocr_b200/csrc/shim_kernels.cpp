// Reference-signature C++ wrappers (turbo_ocr::kernels::cuda_*) over the C-ABI.
// A failing status becomes turbo_ocr::CudaError / TimeoutError / InferenceError.
#include "turbo_ocr/kernels/kernels.h"

#include <climits>
#include <cuda_runtime.h>
#include <string>

#include "tocr_capi.h"
#include "turbo_ocr/common/errors.h"

#define TOCR_SHIM_API __attribute__((visibility("default")))

namespace turbo_ocr {

TOCR_SHIM_API void throw_on_status(int status, const char *where) {
  if (status == TOCR_OK) return;
  std::string msg = std::string(where) + ": " + tocr_last_error_string();
  switch (status) {
    case TOCR_ERR_TIMEOUT:
      throw TimeoutError(msg);
    case TOCR_ERR_INJECTED:
      throw InferenceError(msg);
    default:
      throw CudaError(msg);
  }
}

namespace kernels {

TOCR_SHIM_API void cuda_argmax(const float *input_probs, int *output_indices,
                               float *output_scores, int batch_size, int seq_len,
                               int num_classes, cudaStream_t stream) {
  throw_on_status(tocr_argmax_f32(input_probs, output_indices, output_scores, batch_size,
                                  seq_len, num_classes, stream),
                  "cuda_argmax");
}

TOCR_SHIM_API void cuda_batch_fused_resize_normalize_det(
    const void *const *d_src_ptrs, const int *d_src_steps, const int *d_src_heights,
    const int *d_src_widths, const int *d_dst_heights, const int *d_dst_widths,
    float *dst_chw, int dst_w, int dst_h, int batch_size, cudaStream_t stream) {
  throw_on_status(tocr_preprocess_batch_f32(d_src_ptrs, d_src_steps, d_src_heights,
                                            d_src_widths, d_dst_heights, d_dst_widths,
                                            dst_chw, dst_w, dst_h, batch_size, nullptr,
                                            nullptr, stream),
                  "cuda_batch_fused_resize_normalize_det");
}

TOCR_SHIM_API void cuda_fused_resize_normalize_det(const GpuImage &src, float *dst_chw,
                                                   int dst_w, int dst_h,
                                                   cudaStream_t stream) {
  // The descriptor travels as a kernel parameter: no device staging, no
  // allocation, nothing shared between calls or streams.
  if (src.step > (size_t)INT_MAX) throw CudaError("cuda_fused_resize_normalize_det: step too large");
  throw_on_status(tocr_preprocess_one_f32(src.data, (int)src.step, src.rows, src.cols, dst_chw,
                                          dst_w, dst_h, nullptr, nullptr, stream),
                  "cuda_fused_resize_normalize_det");
}

TOCR_SHIM_API void cuda_batch_roi_warp(const GpuImage &src, const float *d_M_invs,
                                       const int *d_crop_widths, float *d_dst_batch,
                                       int batch_size, int dst_h, int dst_w,
                                       cudaStream_t stream, float mean0, float mean1,
                                       float mean2, float inv_std0, float inv_std1,
                                       float inv_std2, float inv_scale) {
  if (src.step > (size_t)INT_MAX) throw CudaError("cuda_batch_roi_warp: step too large");
  const float mean[3] = {mean0, mean1, mean2}, inv_std[3] = {inv_std0, inv_std1, inv_std2};
  throw_on_status(tocr_roi_warp_f32(static_cast<const uint8_t *>(src.data), src.rows, src.cols,
                                    (int)src.step, d_M_invs, d_crop_widths, batch_size, dst_h,
                                    dst_w, mean, inv_std, inv_scale, d_dst_batch, stream),
                  "cuda_batch_roi_warp");
}

TOCR_SHIM_API int cuda_gpu_ccl_detect(const uint8_t *d_bitmap, const float *d_pred_map, int w,
                                      int h, float box_thresh, int *d_labels,
                                      int *d_compact_ids, int *d_id_counter,
                                      GpuDetBox *d_bboxes, int *d_num_boxes,
                                      GpuDetBox *h_boxes, int *h_num_boxes,
                                      cudaStream_t stream, int *h_num_total) {
  throw_on_status(tocr_gpu_ccl_detect(d_bitmap, d_pred_map, w, h, box_thresh, d_labels,
                                      d_compact_ids, d_id_counter, d_bboxes, d_num_boxes,
                                      h_boxes, h_num_boxes, h_num_total, stream),
                  "cuda_gpu_ccl_detect");
  return *h_num_boxes;
}

TOCR_SHIM_API void cuda_jfa_expand_labels(const uint8_t *d_bitmap, const int32_t *d_compact_ids,
                                          const float *d_expand_per_comp,
                                          uint32_t *d_expanded_labels, int w, int h,
                                          float /*max_expand*/, uint32_t *d_seeds,
                                          uint32_t *d_seeds_alt, cudaStream_t stream) {
  throw_on_status(tocr_jfa_expand_labels(d_bitmap, d_compact_ids, d_expand_per_comp,
                                         d_expanded_labels, w, h, d_seeds, d_seeds_alt, stream),
                  "cuda_jfa_expand_labels");
}

TOCR_SHIM_API void cuda_accumulate_crack_perimeter(const int32_t *d_compact_ids,
                                                   const uint8_t *d_bitmap, int w, int h,
                                                   int num_slots, int *d_perim_per_comp,
                                                   cudaStream_t stream) {
  throw_on_status(tocr_jfa_crack_perimeter(d_compact_ids, d_bitmap, w, h, num_slots,
                                           d_perim_per_comp, stream),
                  "cuda_accumulate_crack_perimeter");
}

TOCR_SHIM_API void cuda_compute_expand_per_comp(const GpuDetBox *d_bboxes,
                                                const int *d_perim_per_comp, int num_slots,
                                                float unclip_ratio, float min_expand,
                                                float max_expand, float box_thresh,
                                                float *d_expand_per_comp, cudaStream_t stream) {
  throw_on_status(tocr_jfa_expand_per_comp(d_bboxes, d_perim_per_comp, num_slots, unclip_ratio,
                                           min_expand, max_expand, box_thresh,
                                           d_expand_per_comp, stream),
                  "cuda_compute_expand_per_comp");
}

TOCR_SHIM_API void cuda_jfa_extract_bboxes(const uint32_t *d_expanded_labels, int w, int h,
                                           GpuDetBox *d_bboxes, int num_slots,
                                           cudaStream_t stream) {
  throw_on_status(tocr_jfa_extract_bboxes(d_expanded_labels, w, h, d_bboxes, num_slots, stream),
                  "cuda_jfa_extract_bboxes");
}

TOCR_SHIM_API void cuda_jfa_extract_oriented(const uint32_t *d_expanded_labels, int w, int h,
                                             GpuDetBox *d_bboxes, int num_slots,
                                             unsigned long long *d_moments, float *d_orient,
                                             cudaStream_t stream) {
  throw_on_status(tocr_jfa_extract_oriented(d_expanded_labels, w, h, d_bboxes, num_slots,
                                            d_moments, d_orient, stream),
                  "cuda_jfa_extract_oriented");
}

TOCR_SHIM_API void cuda_batch_threshold_to_u8(const float *src, uint8_t *dst, int w, int h,
                                              int batch_size, float thresh,
                                              cudaStream_t stream) {
  throw_on_status(tocr_threshold_u8(src, dst, w, h, batch_size, thresh, stream),
                  "cuda_batch_threshold_to_u8");
}

TOCR_SHIM_API void cuda_threshold_to_u8(const float *src, uint8_t *dst, int w, int h,
                                        float thresh, cudaStream_t stream) {
  throw_on_status(tocr_threshold_u8(src, dst, w, h, 1, thresh, stream),
                  "cuda_threshold_to_u8");
}

}  // namespace kernels
}  // namespace turbo_ocr
