// Reference-signature C++ entry points of the B200 kernels
// (include/turbo_ocr/kernels/kernels.h in TurboOCR). Each function forwards to
// the C-ABI in tocr_capi.h and throws turbo_ocr::CudaError on failure, the
// CUDA_CHECK convention of the reference (common/cuda/cuda_check.h:8-17).
// All work is enqueued asynchronously on `stream`.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "turbo_ocr/decode/gpu_image.h"

namespace turbo_ocr::kernels {

using decode::GpuImage;

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

}  // namespace turbo_ocr::kernels
