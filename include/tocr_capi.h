/*
 * tocr_capi.h — C-ABI of the B200-native TurboOCR det+rec hot path.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a cudaStream_t (passed as void*),
 *   - enqueues its work asynchronously on that stream (unless documented to
 *     synchronise, exactly like the reference function it replaces),
 *   - allocates nothing: all device/pinned buffers are owned by the caller,
 *   - returns TOCR_OK (0) or a TOCR_ERR_* status; no C++ exception crosses
 *     this boundary. tocr_last_error_string() gives the message of the most
 *     recent failure on the calling thread.
 *
 * The reference signature each entry replaces is cited as
 * <file>:<line> inside the TurboOCR source tree (include/, src/).
 */
#ifndef TOCR_CAPI_H
#define TOCR_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TOCR_API __attribute__((visibility("default")))
#else
#define TOCR_API
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
  TOCR_OK = 0,
  TOCR_ERR_INVALID = 1,  /* bad argument (null pointer, size, alignment)   */
  TOCR_ERR_CUDA = 2,     /* a CUDA runtime/launch error                     */
  TOCR_ERR_OVERFLOW = 3, /* a size product exceeds the kernel's index range */
  TOCR_ERR_TIMEOUT = 4,  /* a bounded device-side wait gave up              */
  TOCR_ERR_INJECTED = 5  /* forced by tocr_debug_inject_error (tests only)   */
};

/* Message of the last failing call on this thread ("" if none). */
TOCR_API const char *tocr_last_error_string(void);
/* Library version as 0xMMmmpp. */
TOCR_API int tocr_version(void);

/* Host-side fault injection for failure-path tests: the next `count` calls of
 * any tocr_* compute entry return `status` without touching the GPU.
 * count <= 0 clears the injection. Never faults a device. */
TOCR_API void tocr_debug_inject_error(int status, int count);

/* ---- subsystem 4: CTC greedy decode ------------------------------------ */

/* Replaces turbo_ocr::kernels::cuda_argmax
 *   (include/turbo_ocr/kernels/kernels.h:27-30, src/kernels/reduce_kernels.cu:85-93).
 * Per (line, timestep) row of `num_classes` fp32 values: the maximum value and
 * its index, ties broken toward the LOWEST index (reduce_kernels.cu:45-51). */
TOCR_API int tocr_argmax_f32(const float *d_probs, int *d_indices,
                             float *d_scores, int batch_size, int seq_len,
                             int num_classes, void *stream);

/* Fused replacement of cuda_argmax + the host-side ctc_greedy_decode
 *   (src/recognition/ctc_decode.cpp:25-92, include/turbo_ocr/recognition/ctc_decode.h:10-18)
 * on fp16 logits [batch, seq_len, num_classes] (index 0 = blank).
 * Per row: argmax (lowest index on ties) and the max softmax probability
 * p = 1 / sum_j exp(x_j - x_max). Per line: collapse — emit idx when
 * idx != previous idx, idx != 0 and idx < num_labels; the line score is the
 * sequential fp32 mean of the emitted p (0 when nothing is emitted).
 * Outputs: d_tokens [batch*seq_len] (first d_lengths[b] entries of row b are
 * valid), d_lengths [batch], d_line_scores [batch].
 * d_step_idx / d_step_prob [batch*seq_len] receive the per-step argmax and
 * probability; they double as the kernel's scratch and must not be NULL.
 * d_logits must be 2-byte aligned; rows need not be 16-byte aligned. */
TOCR_API int tocr_ctc_greedy_f16(const void *d_logits, int batch_size,
                                 int seq_len, int num_classes, int num_labels,
                                 int *d_tokens, int *d_lengths,
                                 float *d_line_scores, int *d_step_idx,
                                 float *d_step_prob, void *stream);

/* ---- subsystem 1: batched det preprocessing ----------------------------- */

/* Replaces turbo_ocr::kernels::cuda_batch_fused_resize_normalize_det
 *   (include/turbo_ocr/kernels/kernels.h:97-102, src/kernels/preprocess_kernels.cu:128-201)
 * with an fp16 NCHW output. Per image b: half-pixel bilinear resize of the
 * u8 HWC source (pitch d_src_steps[b] bytes, d_src_heights[b] x
 * d_src_widths[b]) to d_dst_heights[b] x d_dst_widths[b], letterboxed at the
 * top-left of a dst_h x dst_w canvas; channel c (positional, bytes 0/1/2) is
 * normalised as (v/255 - mean[c]) / std[c]; pixels outside the content are
 * the normalised black value (0 - mean[c]) / std[c]. mean/inv_std may be
 * NULL for the det defaults (0.485, 0.456, 0.406) and 1/(0.229, 0.224, 0.225).
 * dst_f16 must be 16-byte aligned and dst_w a multiple of 8. */
TOCR_API int tocr_preprocess_batch_f16(
    const void *const *d_src_ptrs, const int *d_src_steps,
    const int *d_src_heights, const int *d_src_widths,
    const int *d_dst_heights, const int *d_dst_widths, void *dst_f16,
    int dst_w, int dst_h, int batch_size, const float *mean3,
    const float *inv_std3, void *stream);

/* fp32-output variant with the exact reference signature semantics
 * (cuda_batch_fused_resize_normalize_det, preprocess_kernels.cu:180-201). */
TOCR_API int tocr_preprocess_batch_f32(
    const void *const *d_src_ptrs, const int *d_src_steps,
    const int *d_src_heights, const int *d_src_widths,
    const int *d_dst_heights, const int *d_dst_widths, float *dst_f32,
    int dst_w, int dst_h, int batch_size, const float *mean3,
    const float *inv_std3, void *stream);

/* ---- DB threshold (replaces cuda_batch_threshold_to_u8) ----------------- */

/* src/kernels/reduce_kernels.cu:97-151: dst = src > thresh ? 255 : 0 over
 * batch_size * w * h elements. */
TOCR_API int tocr_threshold_u8(const float *d_src, uint8_t *d_dst, int w,
                               int h, int batch_size, float thresh,
                               void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TOCR_CAPI_H */
