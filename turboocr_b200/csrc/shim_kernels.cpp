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
  // One-image batch: the descriptor arrays live in a small device block that
  // is written with a stream-ordered copy from this call's stack frame, so the
  // call stays asynchronous without any allocation per call.
  struct Meta {
    const void *ptr;
    int step, h, w, dh, dw;
  };
  thread_local void *d_meta = nullptr;
  thread_local int meta_dev = -1;
  int dev = 0;
  throw_on_status(cudaGetDevice(&dev) == cudaSuccess ? TOCR_OK : TOCR_ERR_CUDA,
                  "cuda_fused_resize_normalize_det");
  if (d_meta == nullptr || meta_dev != dev) {
    // One-time per thread and device; freed at process exit.
    if (cudaMalloc(&d_meta, 64) != cudaSuccess)
      throw CudaError("cuda_fused_resize_normalize_det: metadata allocation failed");
    meta_dev = dev;
  }
  if (src.step > (size_t)INT_MAX) throw CudaError("cuda_fused_resize_normalize_det: step too large");
  const void *ptrs[1] = {src.data};
  const int ints[5] = {(int)src.step, src.rows, src.cols, dst_h, dst_w};
  char host[64];
  __builtin_memcpy(host, ptrs, sizeof(ptrs));
  __builtin_memcpy(host + 8, ints, sizeof(ints));
  // cudaMemcpyAsync from pageable memory is staged synchronously w.r.t. the
  // host buffer, so `host` may go out of scope after the call returns.
  if (cudaMemcpyAsync(d_meta, host, 28, cudaMemcpyHostToDevice, stream) != cudaSuccess)
    throw CudaError("cuda_fused_resize_normalize_det: metadata copy failed");
  char *m = static_cast<char *>(d_meta);
  const int *di = reinterpret_cast<const int *>(m + 8);
  throw_on_status(tocr_preprocess_batch_f32(reinterpret_cast<const void *const *>(m), di,
                                            di + 1, di + 2, di + 3, di + 4, dst_chw, dst_w,
                                            dst_h, 1, nullptr, nullptr, stream),
                  "cuda_fused_resize_normalize_det");
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
