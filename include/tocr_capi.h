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

/* Test hook: the widest point set (x columns) tocr_db_postprocess's
 * shared-memory geometry takes (0: every set above 96 points uses the global
 * scratch pool; < 0: the compiled capacity, 6144). Process-wide; results do
 * not depend on it. */
TOCR_API void tocr_debug_db_shared_columns(int columns);

/* ---- detection resize policy (host) ------------------------------------ */

/* Replaces turbo_ocr::detection::compute_det_resize
 *   (include/turbo_ocr/detection/det_config.h:58-81): the /32-rounded det
 * input size of an h x w image under limit type "max" (limit_max = 1: shrink
 * the longer side to limit_side_len) or "min" (0: grow the shorter side),
 * with the longer output side capped at max_side_limit. Host only. */
TOCR_API int tocr_compute_det_resize(int h, int w, int limit_max, int limit_side_len,
                                     int max_side_limit, int *out_h, int *out_w);
/* read_det_resize (det_config.h:89-127): applies DET_LIMIT_TYPE,
 * DET_LIMIT_SIDE_LEN, DET_MAX_SIDE_LIMIT and DET_MAX_SIDE to the base passed
 * in the three in/out arguments. */
TOCR_API int tocr_read_det_resize(int *limit_max, int *limit_side_len, int *max_side_limit);
/* effective_det_max_side (det_config.h:158-163): the buffer side for a
 * max_side_limit (DET_MAX_SIDE wins), clamped to [32, 4096], rounded up to /32. */
TOCR_API int tocr_effective_det_max_side(int max_side_limit);
/* read_db_params (det_config.h:132-141): DET_DB_THRESH, DET_BOX_THRESH and
 * DET_UNCLIP over the in/out base values. */
TOCR_API int tocr_read_db_params(float *thresh, float *box_thresh, float *unclip_ratio);

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

/* The recognizer's CTC head fused with the greedy decode, on the tensor
 * cores: logits l = feat · W^T + bias are formed tile by tile in TMEM and
 * reduced on the SM (never written), then collapsed as tocr_ctc_greedy_f16
 * does. The reference writes the logits [N, T, V] from its TensorRT
 * recognizer (src/recognition/paddle_rec.cpp:48-90) and decodes them with
 * cuda_argmax + ctc_greedy_decode (reduce_kernels.cu:15-93,
 * ctc_decode.cpp:25-88); per step the results are the same argmax (lowest
 * index on ties) and p = 1 / sum_j exp(l_j - l_max).
 * d_feat fp16 [batch_size * seq_len][K], d_w fp16 [num_classes][K] (both
 * row-major, 16-byte aligned), d_bias fp32 [num_classes]; K = 64 or 128.
 * Outputs and step buffers as tocr_ctc_greedy_f16. d_err (device int,
 * caller-zeroed) receives a non-zero code if a bounded device-side wait gave
 * up (the call itself still returns TOCR_OK). */
TOCR_API int tocr_rec_head_ctc_f16(const void *d_feat, int batch_size, int seq_len, int K,
                                   const void *d_w, const float *d_bias, int num_classes,
                                   int num_labels, int *d_tokens, int *d_lengths,
                                   float *d_line_scores, int *d_step_idx, float *d_step_prob,
                                   int *d_err, void *stream);

/* Allocation-free variant of tocr_ctc_greedy_f16 (no counterpart in the
 * reference). It is for callers that may not call cudaMalloc at all: plugins
 * hosted by an engine that owns every device allocation, or serving
 * processes whose allocator reserved the GPU's memory at start-up and gives
 * none to third-party code. Same kernels and results, but the per-step
 * scratch lives in a static device array of 2^20 steps (8 MiB, held by every
 * GPU that loads the library until exit), so batch_size * seq_len must not
 * exceed 1048576 (TOCR_ERR_INVALID otherwise). Nothing is allocated. Every
 * call looks up the array's address in the current context
 * (cudaGetSymbolAddress); the first call on a device may load the module, so
 * make it before any stream capture. Calls that overlap on one device share
 * the scratch and race: serialise them (one stream, or events). */
TOCR_API int tocr_ctc_greedy_f16_noalloc(const void *d_logits, int batch_size,
                                         int seq_len, int num_classes, int num_labels,
                                         int *d_tokens, int *d_lengths,
                                         float *d_line_scores, void *stream);

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

/* Replaces cuda_fused_resize_normalize_det (include/turbo_ocr/kernels/
 * kernels.h:33-35, src/kernels/preprocess_kernels.cu:58-97): one u8 HWC image
 * (pitch src_step) resized to the whole dst_h x dst_w canvas (no letterbox),
 * normalised, CHW. The image descriptor is passed by value to the kernel, so
 * nothing is staged in device memory. dst_w must be a multiple of 8. */
TOCR_API int tocr_preprocess_one_f32(const void *d_src, int src_step, int src_h, int src_w,
                                     float *dst_f32, int dst_w, int dst_h, const float *mean3,
                                     const float *inv_std3, void *stream);
TOCR_API int tocr_preprocess_one_f16(const void *d_src, int src_step, int src_h, int src_w,
                                     void *dst_f16, int dst_w, int dst_h, const float *mean3,
                                     const float *inv_std3, void *stream);

/* ---- DB threshold (replaces cuda_batch_threshold_to_u8) ----------------- */

/* src/kernels/reduce_kernels.cu:97-151: dst = src > thresh ? 255 : 0 over
 * batch_size * w * h elements. */
TOCR_API int tocr_threshold_u8(const float *d_src, uint8_t *d_dst, int w,
                               int h, int batch_size, float thresh,
                               void *stream);

/* ---- subsystem 3: DB post-processing -------------------------------------- */

/* Device replacement of the CPU path extract_boxes_from_bitmap
 * (src/detection/det_postprocess.cpp:145-222, include/turbo_ocr/detection/
 * det_postprocess.h:33-41) fused with its threshold (cv::compare GT,
 * src/detection/cpu_paddle_det.cpp:115), for n_maps fp32 probability maps
 * [n_maps][h][w]. Per map: contours in cv::findContours(RETR_LIST,
 * CHAIN_APPROX_SIMPLE) order capped at 3000; filters and geometry as the
 * reference (min_box_side / min_unclipped_side are kMinBoxSide = 3 and
 * kMinUnclippedSide = 5 there, paddle_det.h:62-63). Writes the kept quads
 * (int [n_maps][max_boxes][4][2], tl tr br bl), their box_score_fast values
 * ([n_maps][max_boxes]) and counts ([n_maps]) in contour order.
 * d_geometry: NULL (identity) or int [n_maps][4] = orig_h, orig_w, resize_h,
 * resize_w for the scaling of det_postprocess.cpp:205-210.
 * unclip is the reference's: Clipper's round-join offset and then Clipper's
 * union of that path (positive fill), largest ring kept, so the boxes are
 * bit-exact with the reference's CPU path.
 * point_cap bounds the traced contour points of a call; offset_cap sizes a
 * scratch pool (256 bytes per point) that holds every unclip's offset ring,
 * union sweep and hull work space, and the rare point sets wider than the
 * shared-memory geometry takes (6144 columns); <= 0: defaults (h*w/4 + 4096
 * points per map for both). The workspace (256-byte aligned) must hold
 * tocr_db_workspace_bytes(n_maps, h, w, point_cap, offset_cap) bytes.
 * d_status (device int) receives 0 or a bit set: 1 point pool full, 2 a
 * border walk exceeded its bound, 4 scratch pool full, 8 more than max_boxes
 * kept (truncated), 16 a union sweep exceeded its bounds (that box was built
 * from the raw offset ring). Enqueued on `stream`; no synchronisation, no
 * allocation. */
TOCR_API size_t tocr_db_workspace_bytes(int n_maps, int h, int w, long long point_cap,
                                        long long offset_cap);
TOCR_API int tocr_db_postprocess(const float *d_pred, int n_maps, int h, int w,
                                 const int *d_geometry, float thresh, float box_thresh,
                                 float unclip_ratio, float min_box_side,
                                 float min_unclipped_side, long long point_cap,
                                 long long offset_cap, void *d_workspace,
                                 size_t workspace_bytes, int *d_boxes, float *d_scores,
                                 int *d_counts, int max_boxes, int *d_status, void *stream);

/* Connected components of the thresholded maps (the labelling stage of
 * tocr_db_postprocess; the reference's GPU labelling is cuda_gpu_ccl_detect,
 * src/kernels/ccl_kernels.cu:387-493). labels [n_maps][h][w]: 0 for
 * background joined to the image frame, otherwise 1 + the raster index of the
 * smallest pixel of the component (foreground 8-connected, background
 * 4-connected). d_bitmap [n_maps][h][w] receives the 0/255 bitmap.
 * d_scratch: NULL, or tocr_db_components_scratch_bytes(n_maps, h, w) bytes
 * that enable the background-tile shortcuts of tocr_db_postprocess. */
TOCR_API size_t tocr_db_components_scratch_bytes(int n_maps, int h, int w);
TOCR_API int tocr_db_components(const float *d_pred, int n_maps, int h, int w, float thresh,
                                int *d_labels, uint8_t *d_bitmap, void *d_scratch, void *stream);

/* Replaces cuda_gpu_ccl_detect (include/turbo_ocr/kernels/kernels.h:131-145,
 * src/kernels/ccl_kernels.cu:387-493): 8-connected components of the 255/0
 * bitmap [h][w], per component the box, pixel count and mean of d_pred, kept
 * when pixel_count >= 3, both sides >= 3 and mean >= box_thresh. Components
 * are numbered in raster order of their first pixel (at most 3000); kept
 * boxes (56-byte GpuDetBox records) in that order. Caller buffers as the
 * reference: d_labels / d_compact_ids int[w*h], d_id_counter int[1],
 * d_bboxes 2*3000 records, d_num_boxes int[1]; h_boxes >= 3000 records
 * (pinned). Synchronises `stream` once (the reference's contract);
 * *h_num_boxes = kept count, *h_num_total (optional) = components found. */
TOCR_API int tocr_gpu_ccl_detect(const uint8_t *d_bitmap, const float *d_pred, int w, int h,
                                 float box_thresh, int *d_labels, int *d_compact_ids,
                                 int *d_id_counter, void *d_bboxes, int *d_num_boxes,
                                 void *h_boxes, int *h_num_boxes, int *h_num_total,
                                 void *stream);

/* ---- mode-2 unclip: per-component disc growth (src/kernels/jfa.cu) -------- */

/* Replaces cuda_accumulate_crack_perimeter (kernels.h:181-189,
 * src/kernels/jfa.cu:165-185, 458-469): d_perim[id] (num_slots ints, zeroed
 * here) = number of 4-connected pixel edges of component id (compact-id map
 * int[h][w], -1 = background) that face background or the image border. */
TOCR_API int tocr_jfa_crack_perimeter(const int32_t *d_compact_ids, const uint8_t *d_bitmap,
                                      int w, int h, int num_slots, int *d_perim, void *stream);

/* Replaces cuda_compute_expand_per_comp (kernels.h:191-200, jfa.cu:191-212,
 * 471-482): per slot of the PRE-filter records of tocr_gpu_ccl_detect (sum
 * of prediction in `score`), 0 when pixel_count < 3, a box side < 3 or the
 * mean < box_thresh, else pixel_count * unclip_ratio / perimeter clamped to
 * [min_expand, max_expand]. */
TOCR_API int tocr_jfa_expand_per_comp(const void *d_bboxes, const int *d_perim, int num_slots,
                                      float unclip_ratio, float min_expand, float max_expand,
                                      float box_thresh, float *d_expand, void *stream);

/* Replaces cuda_jfa_expand_labels (kernels.h:172-179, jfa.cu:75-146,
 * 436-456): d_labels uint32[h][w] = 1 + the component id a pixel belongs to
 * after growth (0 = none): foreground keeps its component (when its distance
 * is positive); background goes to the nearest boundary pixel (foreground
 * with a background 8-neighbour) whose component's distance e reaches it
 * (d2 <= e*e), ties to the smaller id. d_keys uint32[h][w] scratch.
 * d_seed_list: NULL, or uint32[h*w] scratch that receives the compacted
 * boundary pixels (faster; the reference's unused d_seeds_alt). */
TOCR_API int tocr_jfa_expand_labels(const uint8_t *d_bitmap, const int32_t *d_compact_ids,
                                    const float *d_expand, uint32_t *d_labels, int w, int h,
                                    uint32_t *d_keys, uint32_t *d_seed_list, void *stream);

/* Replaces cuda_jfa_extract_bboxes (kernels.h:202-209, jfa.cu:214-250,
 * 484-498): per slot (label - 1) the box and pixel count of the grown
 * region (slots without pixels: pixel_count 0). */
TOCR_API int tocr_jfa_extract_bboxes(const uint32_t *d_labels, int w, int h, void *d_bboxes,
                                     int num_slots, void *stream);

/* Replaces cuda_jfa_extract_oriented (kernels.h:210-229, jfa.cu:252-434):
 * the box, pixel count and the corners of the rectangle aligned with the
 * principal axis of the grown region (PCA of its pixel coordinates, angle 0
 * when nearly isotropic) in ox/oy. d_moments uint64[num_slots*6] and
 * d_orient float[num_slots*6] scratch. */
TOCR_API int tocr_jfa_extract_oriented(const uint32_t *d_labels, int w, int h, void *d_bboxes,
                                       int num_slots, unsigned long long *d_moments,
                                       float *d_orient, void *stream);

/* ---- recognition crops (replace the host-side crop loop of PaddleRec) ----- */

/* compute_crop_transform (include/turbo_ocr/common/geometry/perspective.h:25-67,
 * perspective_math.h:16-47) for every detected quad of n_pages pages, on the
 * device. d_boxes int [n_pages][max_boxes][4][2] and d_counts [n_pages] as
 * written by tocr_db_postprocess. Crops are numbered page-major; d_crop_off
 * [n_pages + 1] receives their offsets (total at [n_pages]); per crop:
 * d_minv [9] (M_inv), d_crop_w (resize width, clamped to [1, max_width]),
 * d_crop_page (page index), d_vertical (rotated vertical text). */
TOCR_API int tocr_crop_transforms(const int *d_boxes, const int *d_counts, int n_pages,
                                  int max_boxes, int target_h, int max_width, int *d_crop_off,
                                  float *d_minv, int *d_crop_w, int *d_crop_page,
                                  int *d_vertical, void *stream);

/* batch_roi_warp_kernel / cuda_batch_roi_warp (src/kernels/preprocess_kernels.cu:211-344)
 * over crops of several same-size pages (u8 HWC, page i at d_pages + i *
 * page_stride, row pitch src_step), fp16 NCHW out [max_crops][3][dst_h][dst_w].
 * The crop count is read from *d_n_crops (at most max_crops). mean3 /
 * inv_std3 NULL = the rec defaults (0.5, 2.0); inv_scale = 1/255. */
TOCR_API int tocr_roi_warp_f16(const uint8_t *d_pages, long long page_stride, int src_h,
                               int src_w, int src_step, const float *d_minv, const int *d_crop_w,
                               const int *d_crop_page, const int *d_n_crops, int max_crops,
                               int dst_h, int dst_w, const float *mean3, const float *inv_std3,
                               float inv_scale, void *d_dst, void *stream);

/* Replaces cuda_batch_roi_warp (include/turbo_ocr/kernels/kernels.h:19-25,
 * src/kernels/preprocess_kernels.cu:211-344) with its signature's meaning:
 * batch_size crops of ONE u8 HWC image (pitch src_step), transforms d_minv
 * [batch][9] and widths d_crop_w [batch], fp32 output [batch][3][dst_h]
 * [dst_w] = (p * inv_scale - mean_c) * inv_std_c in RGB order, zero beyond
 * each crop's width. mean3 / inv_std3 NULL: 0.5 / 2.0 (recognition). */
TOCR_API int tocr_roi_warp_f32(const uint8_t *d_src, int src_h, int src_w, int src_step,
                               const float *d_minv, const int *d_crop_w, int batch_size,
                               int dst_h, int dst_w, const float *mean3, const float *inv_std3,
                               float inv_scale, float *d_dst, void *stream);

/* ---- DB head of the detection network (FPN neck + binarisation head) ----- */
/* The reference runs PP-OCR's DBFPN + DBHead inside TensorRT
 * (include/turbo_ocr/engine/trt/trt_engine.h:37). The pieces:
 *
 * Convolution on the tensor cores (implicit GEMM, tcgen05): y fp16 NHWC
 * [n][h][w][cout] = conv_k(x)(+ d_bias)(+ up2(d_up))(ReLU if relu), stride
 * 1, pad k/2, x fp16 NHWC [n][h][w][cin]; d_up (optional) is the coarser
 * level [n][h/2][w/2][cout] added after nearest upsampling. Shapes built:
 * k=1 cin 256 or 128 -> cout 96 (with or without d_up), k=3 cin 96 -> 24,
 * k=3 cin 72 -> 24 with ReLU. d_packed from tocr_conv_tc_pack (weights
 * [cout][cin][k][k] fp32). Buffers 16-byte aligned. d_err (device int,
 * caller-zeroed) receives a code if a bounded device-side wait gave up. */
TOCR_API size_t tocr_conv_tc_packed_bytes(int cin, int cout, int ksize);
TOCR_API int tocr_conv_tc_pack(int cin, int cout, int ksize, const float *w, void *out,
                               size_t out_bytes);
TOCR_API int tocr_conv_tc_f16(const void *d_x, int n, int h, int w, int cin, int cout, int ksize,
                              const void *d_packed, const float *d_bias, int relu,
                              const void *d_up, void *d_y, int *d_err, void *stream);
/* fuse fp16 NHWC [n][h][w][72] = (p4 [n][h/4][w/4][24] up 4, p3 [n][h/2][w/2][24]
 * up 2, p2 [n][h][w][24]) along channels (nearest upsampling). */
TOCR_API int tocr_fpn_concat_f16(const void *d_p4, const void *d_p3, const void *d_p2, int n,
                                 int h, int w, void *d_fuse, void *stream);
/* The head's two stride-2 2x2 transposed convolutions and the sigmoid:
 * h1 fp16 NHWC [n][h][w][24] -> h2 = ReLU(convT(h1; w2 [24][24][2][2], b2))
 * -> prob fp32 [n][4h][4w] = sigmoid(convT(h2; w3 [24][1][2][2], b3)). */
TOCR_API int tocr_db_head_up_f32(const void *d_h1, int n, int h, int w, const float *d_w2,
                                 const float *d_b2, const float *d_w3, float b3, float *d_prob,
                                 void *stream);

/* ---- text-line angle classifier (PaddleCls, src/classification/paddle_cls.cpp) */

/* The classifier network's stem: y = hardswish(conv3x3 stride 2 pad 1 (x) +
 * b), x fp16 NCHW [n][3][h][w] (crops of tocr_roi_warp_f16), weights d_w
 * fp32 [32][3][3][3], d_b [32]; y fp16 NHWC [n][(h-1)/2+1][(w-1)/2+1][32]
 * (16-byte aligned). The module's synthetic model ("synthetic", no trained
 * weights in this build) draws every tensor with tocr_synth_weights from
 * seed 0x7EC0C150 + k: stem w (k=0, scale 0.53), b (k=1, 0.1); block j of
 * (32,64,s1) (64,64,s2) (64,128,s1) (128,128,s2) (128,256,s1): wdw [C][9]
 * (k=16+4j, 0.9), bdw (k=17+4j, 0.1), wpw [C_out][C] (k=18+4j, 0.48 / 0.34
 * / 0.34 / 0.24 / 0.24), bpw (k=19+4j, 0.1), INT8; head w [2][256] (k=64,
 * 1.0), b (k=65, 0.1). The scales keep the activation variance near one
 * through the hardswish layers. */
TOCR_API int tocr_cls_stem_f16(const void *d_x, int n, int h, int w, const float *d_w,
                               const float *d_b, void *d_y, void *stream);

/* The classifier network's head: per sample the mean of every channel over
 * the hw pixels of x fp16 NHWC [n][hw][c], logits l_k = b_k + sum_c w[k][c]
 * mean_c (k = 0, 1), scores fp32 [n][2] = softmax(l) = (score_0, score_180). */
TOCR_API int tocr_cls_head_f32(const void *d_x, int n, int hw, int c, const float *d_w,
                               const float *d_b, float *d_scores, void *stream);

/* Host: n seeded weights in [-scale, scale): out[i] = scale * (2u - 1), u =
 * (splitmix64(seed + (i + 1) * 0x9E3779B97F4A7C15) >> 40) / 2^24. */
TOCR_API int tocr_synth_weights(uint64_t seed, float scale, float *out, long long n);

/* ---- stand-in network heads (no trained weights in this build) ------------- */

/* The detection module's stand-in for the trained DB network (the synthetic
 * pages' probability map): from the normalised fp32 canvas [n][3][h][w],
 * ink = 1 - mean of the de-normalised channels (0 outside each image's
 * letterbox content d_content_hw [n][2], NULL = whole canvas), 15-pixel
 * horizontal max, prob = sigmoid(gain * (max - 0.5)) into d_prob [n][h][w].
 * mean3 / inv_std3 NULL: the det normalisation. */
TOCR_API int tocr_det_standin_prob_f32(const float *d_chw, int n, int h, int w,
                                       const int *d_content_hw, const float *mean3,
                                       const float *inv_std3, float gain, float *d_prob,
                                       void *stream);
/* The recognition module's stand-in for the trained CRNN: fp16 logits
 * [n][seq_len][num_classes], 0 except 16.0 at one class per step; crop c's
 * class at step t is drawn from (seed, id = d_ids[c] or c when NULL, t / 3):
 * blank with probability 1/2, else uniform over 1..num_classes-1. */
TOCR_API int tocr_rec_standin_logits_f16(void *d_logits, const int *d_ids, int n, int seq_len,
                                         int num_classes, uint64_t seed, void *stream);

/* tocr_ctc_greedy_f16 for a line count that lives on the device: lines
 * [0, min(*d_batch, max_batch)) of d_logits [max_batch][seq_len][num_classes]
 * are decoded (no counterpart in the reference, whose batch is a host int). */
TOCR_API int tocr_ctc_greedy_f16_dev(const void *d_logits, const int *d_batch, int max_batch,
                                     int seq_len, int num_classes, int num_labels,
                                     int *d_tokens, int *d_lengths, float *d_line_scores,
                                     int *d_step_idx, float *d_step_prob, void *stream);

/* ---- end-to-end page path (config 5) --------------------------------------- */

/* Det preprocessing of same-size u8 HWC pages at scale 1 (the reference's
 * resize is then the identity; normalisation as preprocess_kernels.cu:169-177)
 * fused with the backbone stem: 3x3 stride-2 pad-1 conv 3->32 + folded BN +
 * hardswish, fp16 NHWC out [n][(h-1)/2+1][(w-1)/2+1][32], as an implicit
 * GEMM on tcgen05 (fp32-accurate: split fp16 weights). h_params is a HOST
 * tocr_stem_pack blob (normalisation folded into the weights), passed to the
 * kernel by value; no counterpart in the reference, whose backbone runs in
 * TensorRT. */
TOCR_API size_t tocr_stem_params_bytes(void);
TOCR_API int tocr_stem_pack(const float *w, const float *b, const float *mean3,
                            const float *inv_std3, void *out, size_t out_bytes);
TOCR_API int tocr_stem_f16(const uint8_t *d_pages, int n, int h, int w, long long page_stride,
                           const void *h_params, void *d_out, void *stream);
/* The stem runs on the tensor cores with bounded waits; a wait that gives up
 * (no completion within about a second) ends the kernel and records a
 * non-zero code. This writes that code to *out_code (0: none) and clears it;
 * it synchronises the current device. */
TOCR_API int tocr_stem_take_error(int *out_code);

/* Synthetic DB probability map of config 5 (no trained det head exists):
 * sigmoid(gain * (max_{|dx|<=7} ink(x+dx, y) - 0.5)), ink = 1 - mean(RGB)/255,
 * fp32 [n][h][w]. */
TOCR_API int tocr_ink_map(const uint8_t *d_pages, int n, int h, int w, long long page_stride,
                          float gain, float *d_prob, void *stream);

/* 1x1 conv c->1 + bias + sigmoid over fp16 NHWC pixels (the det head). */
TOCR_API int tocr_head_sigmoid(const void *d_x, long long npix, int c, const float *d_w,
                               float bias, float *d_out, void *stream);

/* ---- subsystem 2: fused depthwise-3x3 + pointwise-1x1 block ------------- */

/* Replaces one DW-separable block of the det backbone that the reference runs
 * inside TensorRT (include/turbo_ocr/engine/trt/trt_engine.h:37; INT8/FP8 QDQ
 * from scripts/quantize_onnx_int8.py:1-80, scripts/quantize_onnx_fp8.py:2-8;
 * WMMA precedent tools/fused_dwpw_bench.cu:98-152).
 *   y = hardswish(PW(hardswish(DW3x3_stride(x) + b_dw)) * s + b_pw)
 * x: fp16 NHWC [N][H][W][C]; y: fp16 NHWC [N][Ho][Wo][C_out] with
 * Ho = (H-1)/stride + 1 (pad 1). kind 0 = INT8, 1 = FP8-E4M3 PW weights,
 * per output channel. d_packed is the device copy of a tocr_dwpw_pack blob.
 * d_err (device int, caller-zeroed) receives a non-zero code if a bounded
 * device-side wait gave up (the launch itself still returns TOCR_OK).
 * Supported (C, C_out, stride): (128,256,1) (128,128,1) (64,128,1)
 * (64,64,1) (32,64,1) and stride 2 for (64,64) (128,128) (64,128) (32,64). */
TOCR_API int tocr_dwpw_block(const void *d_x, void *d_y, int N, int H, int W,
                             int C, int C_out, int stride, int kind,
                             const void *d_packed, int *d_err, void *stream);

/* Host-side size of a packed parameter blob for (C, C_out). */
TOCR_API size_t tocr_dwpw_packed_bytes(int C, int C_out);

/* Host-side packing of BN-folded block parameters into the kernel's blob:
 * wdw [C][3][3], bdw [C], wpw [C_out][C], bpw [C_out] (all fp32). PW weights
 * are quantised symmetrically per output channel (INT8: max|w|/127, FP8:
 * max|w|/448) and laid out as the 128B-swizzled K-major tcgen05 B operand. */
TOCR_API int tocr_dwpw_pack(int C, int C_out, int kind, const float *wdw,
                            const float *bdw, const float *wpw,
                            const float *bpw, void *out, size_t out_bytes);

/* Dequantised PW weights [C_out][C] of a packed blob (host). */
TOCR_API int tocr_dwpw_dequant_pw(const void *blob, int C, int C_out, int kind,
                                  float *w_out);


/* ---- PNG decode to device BGR ---------------------------------------- */
/* Replaces the reference's CPU decode + upload of one page image:
 * turbo_ocr::decode::FastPngDecoder::decode (src/decode/fast_png_decoder.cpp:48-128,
 * include/turbo_ocr/decode/fast_png_decoder.h:12-15; Wuffs v0.4 to a BGR
 * cv::Mat, 16-bit files through cv::imdecode) followed by
 * OcrPipeline::upload_image (src/pipeline/ocr/ocr_pipeline_runtime.cpp:120-147),
 * whose result is a GpuImage (include/turbo_ocr/decode/gpu_image.h:9-16):
 * here the files go to HBM compressed and the pixels are made there.
 * Output pixels match the reference decode byte for byte: Wuffs' BGR for
 * 1-8 bit files (grey scaled up, alpha premultiplied, tRNS keys and palette
 * alphas applied, palette indices past the PLTE black), OpenCV's for
 * 16-bit files (high byte, alpha dropped). */
typedef struct tocr_png_info {
  int32_t width, height;
  int32_t bit_depth, color_type, interlace;
  int32_t reserved;
  uint64_t raw_bytes;     /* inflated scanline bytes (all passes, filter bytes included) */
  uint64_t scratch_bytes; /* device scratch this file needs (tocr_png_job.scratch_off) */
} tocr_png_info;

typedef struct tocr_png_job {
  uint64_t src_off, src_len; /* the file at d_src + src_off */
  uint64_t dst_off;          /* BGR u8 rows at d_dst + dst_off, dst_pitch bytes apart */
  uint64_t dst_pitch;        /* >= 3 * width */
  uint64_t scratch_off;      /* 16-byte aligned; scratch_bytes from tocr_png_peek */
  int32_t width, height;     /* from tocr_png_peek; the device re-reads the IHDR */
} tocr_png_job;

/* Per-image status written by tocr_png_decode_batch. */
enum {
  TOCR_PNG_OK = 0,
  TOCR_PNG_BAD_HEADER = 1,      /* signature or IHDR                                */
  TOCR_PNG_BAD_CHUNK = 2,       /* chunk layout, truncation, PLTE / tRNS rules       */
  TOCR_PNG_BAD_CHECKSUM = 3,    /* CRC-32 of a critical chunk, or the zlib Adler-32  */
  TOCR_PNG_MISSING_PALETTE = 4, /* colour type 3 without PLTE                        */
  TOCR_PNG_BAD_ZLIB = 5,        /* zlib header                                       */
  TOCR_PNG_BAD_DEFLATE = 6,     /* DEFLATE block, Huffman code or distance           */
  TOCR_PNG_TOO_MUCH_DATA = 7,   /* more scanline bytes than the IHDR implies         */
  TOCR_PNG_NOT_ENOUGH_DATA = 8, /* fewer scanline bytes than the IHDR implies        */
  TOCR_PNG_BAD_FILTER = 9,      /* a scanline filter type above 4                    */
  TOCR_PNG_SIZE_MISMATCH = 10,  /* IHDR differs from the job's width / height        */
  TOCR_PNG_UNSUPPORTED = 11,    /* a side above 16777215                             */
  TOCR_PNG_TIMEOUT = 12         /* a bounded wait between row groups gave up         */
};

/* Host only, no GPU: the signature and IHDR of one file (the first 33 bytes),
 * as image_dims.h:31-48 peeks them, then the reference's caps
 * (fast_png_decoder.cpp:84-93): TOCR_ERR_INVALID when the bytes are not a
 * PNG, the IHDR is malformed, a side is 0 or above max_dim, or
 * width * height > max_pixels (info->width / height are filled whenever the
 * IHDR could be read). On TOCR_OK, info->scratch_bytes is the device scratch
 * the file needs for a file of src_len bytes. */
TOCR_API int tocr_png_peek(const uint8_t *data, size_t len, int max_dim, long long max_pixels,
                           tocr_png_info *info);

/* Decodes n files: d_src holds the files, d_jobs (device, n entries) says
 * where each one is, where its pixels go and which scratch it uses; d_status
 * (device, n int32) receives TOCR_PNG_* per file. The pixels of a file whose
 * status is not TOCR_PNG_OK are unspecified. Three kernels, no allocation,
 * no synchronisation. */
TOCR_API int tocr_png_decode_batch(const uint8_t *d_src, const tocr_png_job *d_jobs, int n,
                                   uint8_t *d_dst, uint8_t *d_scratch, int32_t *d_status,
                                   void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TOCR_CAPI_H */
