// Test-infrastructure wrapper (oracle only): C entry points over the
// REFERENCE's own CUDA kernels (src/kernels/preprocess_kernels.cu,
// src/kernels/reduce_kernels.cu and src/kernels/jfa.cu, compiled unchanged
// from the reference tree by oracle/Makefile). Used on the GPU box by tests/ to pin the fp32
// arithmetic of the B200 kernels to the reference kernel's bits.
#include <exception>

#include "turbo_ocr/decode/gpu_image.h"
#include "turbo_ocr/kernels/kernels.h"

extern "C" {

int refk_batch_preprocess(const void *const *ptrs, const int *steps, const int *sh,
                          const int *sw, const int *dh, const int *dw, float *dst, int dst_w,
                          int dst_h, int batch, void *stream) {
  try {
    turbo_ocr::kernels::cuda_batch_fused_resize_normalize_det(
        ptrs, steps, sh, sw, dh, dw, dst, dst_w, dst_h, batch, (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_argmax(const float *probs, int *idx, float *scores, int batch, int seq_len,
                int classes, void *stream) {
  try {
    turbo_ocr::kernels::cuda_argmax(probs, idx, scores, batch, seq_len, classes,
                                    (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_threshold(const float *src, unsigned char *dst, int w, int h, int batch, float t,
                   void *stream) {
  try {
    turbo_ocr::kernels::cuda_batch_threshold_to_u8(src, dst, w, h, batch, t,
                                                   (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_roi_warp(const void *src, int rows, int cols, long long step, const float *minv,
                  const int *crop_w, float *dst, int batch, int dst_h, int dst_w, void *stream) {
  try {
    turbo_ocr::GpuImage img;
    img.data = const_cast<void *>(src);
    img.step = (std::size_t)step;
    img.rows = rows;
    img.cols = cols;
    turbo_ocr::kernels::cuda_batch_roi_warp(img, minv, crop_w, dst, batch, dst_h, dst_w,
                                            (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_fused_single(const void *src, int rows, int cols, long long step, float *dst, int dst_w,
                      int dst_h, void *stream) {
  try {
    turbo_ocr::GpuImage img;
    img.data = const_cast<void *>(src);
    img.step = (std::size_t)step;
    img.rows = rows;
    img.cols = cols;
    turbo_ocr::kernels::cuda_fused_resize_normalize_det(img, dst, dst_w, dst_h,
                                                        (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

// src/kernels/jfa.cu: the mode-2 unclip stages, one call each.
int refk_jfa_crack(const int *cid, const unsigned char *bm, int w, int h, int slots, int *perim,
                   void *stream) {
  try {
    turbo_ocr::kernels::cuda_accumulate_crack_perimeter(cid, bm, w, h, slots, perim,
                                                        (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_jfa_expand_per_comp(const void *boxes, const int *perim, int slots, float ratio,
                             float emin, float emax, float box_thresh, float *expand,
                             void *stream) {
  try {
    turbo_ocr::kernels::cuda_compute_expand_per_comp(
        static_cast<const turbo_ocr::kernels::GpuDetBox *>(boxes), perim, slots, ratio, emin,
        emax, box_thresh, expand, (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_jfa_expand_labels(const unsigned char *bm, const int *cid, const float *expand,
                           unsigned *labels, int w, int h, float max_expand, unsigned *seeds,
                           unsigned *seeds_alt, void *stream) {
  try {
    turbo_ocr::kernels::cuda_jfa_expand_labels(bm, cid, expand, labels, w, h, max_expand, seeds,
                                               seeds_alt, (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_jfa_extract_bboxes(const unsigned *labels, int w, int h, void *boxes, int slots,
                            void *stream) {
  try {
    turbo_ocr::kernels::cuda_jfa_extract_bboxes(
        labels, w, h, static_cast<turbo_ocr::kernels::GpuDetBox *>(boxes), slots,
        (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}

int refk_jfa_extract_oriented(const unsigned *labels, int w, int h, void *boxes, int slots,
                              unsigned long long *mom, float *orient, void *stream) {
  try {
    turbo_ocr::kernels::cuda_jfa_extract_oriented(
        labels, w, h, static_cast<turbo_ocr::kernels::GpuDetBox *>(boxes), slots, mom, orient,
        (cudaStream_t)stream);
  } catch (const std::exception &) {
    return 2;
  }
  return 0;
}
}
