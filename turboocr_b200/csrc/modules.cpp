// The reference's detection and recognition modules (PaddleDet, PaddleRec)
// over this library's C-ABI, plus the host geometry they share. Buffers are
// allocated once (load_model / allocate_buffers) and reused; every call
// enqueues on the caller's stream and synchronises it once before returning
// host results, as the reference modules do (paddle_det.cpp:136-311,
// paddle_rec.cpp:215-448).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include <climits>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "crop_geom.cuh"
#include "tocr_capi.h"
#include "turbo_ocr/classification/paddle_cls.h"
#include "turbo_ocr/common/errors.h"
#include "turbo_ocr/common/geometry/perspective.h"
#include "turbo_ocr/detection/det_postprocess.h"
#include "turbo_ocr/detection/paddle_det.h"
#include "turbo_ocr/recognition/ctc_decode.h"
#include "turbo_ocr/recognition/paddle_rec.h"

#define TOCR_MOD_API __attribute__((visibility("default")))

namespace turbo_ocr {

namespace {

void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
struct DevBuf {
  T *p = nullptr;
  size_t n = 0;
  void alloc(size_t count) {
    if (count <= n) return;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    cuda_check(cudaMalloc(&p, count * sizeof(T)), "cudaMalloc");
    n = count;
  }
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

template <class T>
struct PinBuf {
  T *p = nullptr;
  size_t n = 0;
  void alloc(size_t count) {
    if (count <= n) return;
    if (p) cudaFreeHost(p);
    p = nullptr;
    n = 0;
    cuda_check(cudaMallocHost(&p, count * sizeof(T)), "cudaMallocHost");
    n = count;
  }
  ~PinBuf() {
    if (p) cudaFreeHost(p);
  }
};

constexpr uint64_t kStandinSeed = 0x7EC00005ull;
constexpr float kStandinGain = 12.0f;

}  // namespace

// ---------------------------------------------------------------- geometry --
TOCR_MOD_API void compute_perspective_inv(const float *dst_pts, const float *src_pts,
                                          float *M_inv) {
  tocr::crop::perspective_inv(dst_pts, src_pts, M_inv);
}

TOCR_MOD_API CropTransform compute_crop_transform(const Box &box, int target_h, int max_width) {
  int b[8];
  for (int k = 0; k < 4; ++k) {
    b[2 * k] = box[k][0];
    b[2 * k + 1] = box[k][1];
  }
  CropTransform ct{};
  int cw = 0, vert = 0;
  tocr::crop::crop_transform(b, target_h, max_width, ct.M_inv, &cw, &vert);
  ct.crop_width = cw;
  ct.vertical = vert != 0;
  return ct;
}

namespace detection {

TOCR_MOD_API void order_quad_tl_tr_br_bl(float xs[4], float ys[4]) noexcept {
  for (int i = 1; i < 4; ++i) {  // insertion sort by x; equal x keep their order
    const float kx = xs[i], ky = ys[i];
    int j = i - 1;
    for (; j >= 0 && xs[j] > kx; --j) {
      xs[j + 1] = xs[j];
      ys[j + 1] = ys[j];
    }
    xs[j + 1] = kx;
    ys[j + 1] = ky;
  }
  const int tl = ys[0] < ys[1] ? 0 : 1, bl = 1 - tl;
  const int tr = ys[2] < ys[3] ? 2 : 3, br = 5 - tr;
  const float ox[4] = {xs[tl], xs[tr], xs[br], xs[bl]};
  const float oy[4] = {ys[tl], ys[tr], ys[br], ys[bl]};
  for (int k = 0; k < 4; ++k) {
    xs[k] = ox[k];
    ys[k] = oy[k];
  }
}

// ----------------------------------------------------------------- PaddleDet --
struct PaddleDet::Impl {
  static constexpr int kMaxBatch = 8;        // paddle_det.h:81
  static constexpr int kMaxBoxes = 3000;     // the reference's candidate cap
  static constexpr float kMinBoxSide = 3.0f;       // paddle_det.h:62
  static constexpr float kMinUnclippedSide = 5.0f; // paddle_det.h:63

  static constexpr int kMaxComp = 3000;     // kMaxGpuComponents
  static constexpr int kRec = 14;           // ints per GpuDetBox record (56 bytes)
  static constexpr float kMaxExpand = 24.0f;  // paddle_det_ccl.cpp:190

  bool loaded = false;
  DetResizeParams resize = kDetResizeDefault;
  DbParams db = kDbDefaults;
  // GPU_CCL mode (paddle_det.cpp:74-97): 0 contours, 1 CCL + per-ROI contours
  // (the reference default), 2 per-component disc growth. Modes 0 and 1 both
  // run the full-map contour path here (tocr_db_postprocess).
  int mode = 1;
  float box_thresh = kDbDefaults.box_thresh;
  float unclip_scale = 1.0f;
  int max_side = 0;
  size_t ws_bytes = 0;

  // mode 2 buffers (allocated by load_model when mode == 2)
  DevBuf<uint8_t> bitmap;
  DevBuf<int> ccl_labels, ccl_cid, ccl_counter, ccl_nbox, ccl_boxes, perim;
  DevBuf<uint32_t> jfa_labels, jfa_keys, jfa_seeds;
  DevBuf<float> expand, orient;
  DevBuf<unsigned long long> moments;
  PinBuf<int> h_ccl_boxes, h_exp_boxes;

  DevBuf<float> canvas, prob;
  DevBuf<char> ws;
  DevBuf<int> boxes, counts, geo, content, status, src_steps, src_h, src_w, dst_h, dst_w;
  DevBuf<const void *> src_ptrs;
  DevBuf<float> scores;
  PinBuf<int> h_boxes, h_counts, h_geo, h_content, h_status, h_steps, h_sh, h_sw, h_dh, h_dw;
  PinBuf<const void *> h_ptrs;
  PinBuf<float> h_scores;
  std::vector<std::vector<float>> last_scores;

  void allocate() {
    const size_t px = (size_t)max_side * max_side;
    canvas.alloc((size_t)kMaxBatch * 3 * px);
    prob.alloc((size_t)kMaxBatch * px);
    ws_bytes = tocr_db_workspace_bytes(kMaxBatch, max_side, max_side, 0, 0);
    ws.alloc(ws_bytes + 256);
    boxes.alloc((size_t)kMaxBatch * kMaxBoxes * 8);
    scores.alloc((size_t)kMaxBatch * kMaxBoxes);
    counts.alloc(kMaxBatch);
    geo.alloc(4 * kMaxBatch);
    content.alloc(2 * kMaxBatch);
    status.alloc(1);
    src_ptrs.alloc(kMaxBatch);
    src_steps.alloc(kMaxBatch);
    src_h.alloc(kMaxBatch);
    src_w.alloc(kMaxBatch);
    dst_h.alloc(kMaxBatch);
    dst_w.alloc(kMaxBatch);
    h_boxes.alloc((size_t)kMaxBatch * kMaxBoxes * 8);
    h_scores.alloc((size_t)kMaxBatch * kMaxBoxes);
    h_counts.alloc(kMaxBatch);
    h_geo.alloc(4 * kMaxBatch);
    h_content.alloc(2 * kMaxBatch);
    h_status.alloc(1);
    h_ptrs.alloc(kMaxBatch);
    h_steps.alloc(kMaxBatch);
    h_sh.alloc(kMaxBatch);
    h_sw.alloc(kMaxBatch);
    h_dh.alloc(kMaxBatch);
    h_dw.alloc(kMaxBatch);
    if (mode == 2) {
      bitmap.alloc(px);
      ccl_labels.alloc(px);
      ccl_cid.alloc(px);
      ccl_counter.alloc(1);
      ccl_nbox.alloc(1);
      ccl_boxes.alloc((size_t)2 * kMaxComp * kRec);
      perim.alloc(kMaxComp);
      jfa_labels.alloc(px);
      jfa_keys.alloc(px);
      jfa_seeds.alloc(px);
      expand.alloc(kMaxComp);
      moments.alloc((size_t)kMaxComp * 6);
      orient.alloc((size_t)kMaxComp * 6);
      h_ccl_boxes.alloc((size_t)kMaxComp * kRec);
      h_exp_boxes.alloc((size_t)kMaxComp * kRec);
    }
  }

  // run_gpu_ccl_fast (paddle_det_ccl.cpp:142-258) on map m of `prob` (h x w
  // canvas, content ch x cw of an oh x ow image): CCL, crack perimeters,
  // growth distances (min 2, max 24), disc growth, principal-axis rectangles,
  // then the reference's host filter and scaling. The score kept per box is
  // the component's mean prediction. Synchronises the stream.
  std::vector<Box> post_mode2(int m, int h, int w, int oh, int ow, int ch, int cw,
                              std::vector<float> &scores, cudaStream_t st) {
    const float *pm = prob.p + (size_t)m * h * w;
    throw_on_status(tocr_threshold_u8(pm, bitmap.p, w, h, 1, db.thresh, st), "PaddleDet threshold");
    int h_nb = 0, h_total = 0;
    throw_on_status(tocr_gpu_ccl_detect(bitmap.p, pm, w, h, box_thresh, ccl_labels.p, ccl_cid.p,
                                        ccl_counter.p, ccl_boxes.p, ccl_nbox.p, h_ccl_boxes.p,
                                        &h_nb, &h_total, st),
                    "PaddleDet CCL");
    std::vector<Box> out;
    scores.clear();
    if (h_nb == 0) return out;
    const int slots = std::min(h_total, kMaxComp);
    if (slots == 0) return out;
    int *exp_boxes = ccl_boxes.p + (size_t)kMaxComp * kRec;
    throw_on_status(tocr_jfa_crack_perimeter(ccl_cid.p, bitmap.p, w, h, slots, perim.p, st),
                    "PaddleDet crack perimeter");
    throw_on_status(tocr_jfa_expand_per_comp(ccl_boxes.p, perim.p, slots,
                                             db.unclip_ratio * unclip_scale, 2.0f, kMaxExpand,
                                             box_thresh, expand.p, st),
                    "PaddleDet expand distances");
    throw_on_status(tocr_jfa_expand_labels(bitmap.p, ccl_cid.p, expand.p, jfa_labels.p, w, h,
                                           jfa_keys.p, jfa_seeds.p, st),
                    "PaddleDet label growth");
    // component means come from the pre-filter records, read before the
    // oriented pass overwrites the filtered half of the box buffer
    cuda_check(cudaMemcpyAsync(h_ccl_boxes.p, ccl_boxes.p, (size_t)slots * kRec * sizeof(int),
                               cudaMemcpyDeviceToHost, st),
               "PaddleDet D2H");
    throw_on_status(tocr_jfa_extract_oriented(jfa_labels.p, w, h, exp_boxes, slots, moments.p,
                                              orient.p, st),
                    "PaddleDet oriented boxes");
    cuda_check(cudaMemcpyAsync(h_exp_boxes.p, exp_boxes, (size_t)slots * kRec * sizeof(int),
                               cudaMemcpyDeviceToHost, st),
               "PaddleDet D2H");
    cuda_check(cudaStreamSynchronize(st), "PaddleDet sync");
    const float ratio_h = static_cast<float>(ch) / oh;
    const float ratio_w = static_cast<float>(cw) / ow;
    for (int i = 0; i < slots; ++i) {
      const int *r = h_exp_boxes.p + (size_t)i * kRec;
      const int xmin = r[0], ymin = r[1], xmax = r[2], ymax = r[3], pc = r[5];
      if (pc < 9) continue;
      const int bw = xmax - xmin + 1, bh = ymax - ymin + 1;
      if (bw < kMinUnclippedSide || bh < kMinUnclippedSide) continue;
      float px[4], py[4];
      std::memcpy(px, r + 6, sizeof px);
      std::memcpy(py, r + 10, sizeof py);
      order_quad_tl_tr_br_bl(px, py);
      Box box;
      for (int k = 0; k < 4; ++k)
        box[k] = {std::clamp(static_cast<int>(std::round(px[k] / ratio_w)), 0, ow - 1),
                  std::clamp(static_cast<int>(std::round(py[k] / ratio_h)), 0, oh - 1)};
      const int rw = static_cast<int>(std::sqrt(double((box[0][0] - box[1][0]) * (box[0][0] - box[1][0]) +
                                                       (box[0][1] - box[1][1]) * (box[0][1] - box[1][1]))));
      const int rh = static_cast<int>(std::sqrt(double((box[0][0] - box[3][0]) * (box[0][0] - box[3][0]) +
                                                       (box[0][1] - box[3][1]) * (box[0][1] - box[3][1]))));
      if (rw <= 3 || rh <= 3) continue;
      out.push_back(box);
      const int *pre = h_ccl_boxes.p + (size_t)i * kRec;
      float sum;
      std::memcpy(&sum, pre + 4, sizeof sum);
      scores.push_back(pre[5] > 0 ? sum / (float)pre[5] : 0.0f);
    }
    return out;
  }

  char *ws_aligned() const {
    return reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(ws.p) + 255) & ~uintptr_t(255));
  }

  // Stand-in network + DB over n maps of h x w already in `prob`'s input
  // canvas; geometry and content already staged on the device. Synchronises.
  std::vector<std::vector<Box>> post(int n, int h, int w, cudaStream_t st) {
    throw_on_status(tocr_det_standin_prob_f32(canvas.p, n, h, w, content.p, nullptr, nullptr,
                                              kStandinGain, prob.p, st),
                    "PaddleDet stand-in head");
    if (mode == 2) {
      std::vector<std::vector<Box>> out(n);
      last_scores.assign(n, {});
      for (int m = 0; m < n; ++m)
        out[m] = post_mode2(m, h, w, h_geo.p[4 * m], h_geo.p[4 * m + 1], h_content.p[2 * m],
                            h_content.p[2 * m + 1], last_scores[m], st);
      return out;
    }
    const size_t need = tocr_db_workspace_bytes(n, h, w, 0, 0);
    if (need > ws_bytes) throw InferenceError("PaddleDet: DB workspace too small");
    throw_on_status(tocr_db_postprocess(prob.p, n, h, w, geo.p, db.thresh, box_thresh,
                                        db.unclip_ratio * unclip_scale, kMinBoxSide, kMinUnclippedSide, 0, 0,
                                        ws_aligned(), need, boxes.p, scores.p, counts.p,
                                        kMaxBoxes, status.p, st),
                    "PaddleDet DB post-process");
    cuda_check(cudaMemcpyAsync(h_counts.p, counts.p, n * sizeof(int), cudaMemcpyDeviceToHost, st),
               "PaddleDet D2H");
    cuda_check(cudaMemcpyAsync(h_status.p, status.p, sizeof(int), cudaMemcpyDeviceToHost, st),
               "PaddleDet D2H");
    cuda_check(cudaMemcpyAsync(h_boxes.p, boxes.p, (size_t)n * kMaxBoxes * 8 * sizeof(int),
                               cudaMemcpyDeviceToHost, st),
               "PaddleDet D2H");
    cuda_check(cudaMemcpyAsync(h_scores.p, scores.p, (size_t)n * kMaxBoxes * sizeof(float),
                               cudaMemcpyDeviceToHost, st),
               "PaddleDet D2H");
    cuda_check(cudaStreamSynchronize(st), "PaddleDet sync");
    if (h_status.p[0] & (1 | 2 | 4 | 16))
      throw InferenceError("PaddleDet: DB post-process status " + std::to_string(h_status.p[0]));
    std::vector<std::vector<Box>> out(n);
    last_scores.assign(n, {});
    for (int m = 0; m < n; ++m) {
      const int c = h_counts.p[m];
      out[m].resize(c);
      last_scores[m].resize(c);
      for (int k = 0; k < c; ++k) {
        const int *q = h_boxes.p + ((size_t)m * kMaxBoxes + k) * 8;
        for (int v = 0; v < 4; ++v) out[m][k][v] = {q[2 * v], q[2 * v + 1]};
        last_scores[m][k] = h_scores.p[(size_t)m * kMaxBoxes + k];
      }
    }
    return out;
  }
};

TOCR_MOD_API PaddleDet::PaddleDet() : impl_(std::make_unique<Impl>()) {}
TOCR_MOD_API PaddleDet::~PaddleDet() noexcept = default;

TOCR_MOD_API bool PaddleDet::load_model(const std::string &model_path,
                                        const DetResizeParams &resize, const DbParams &db) {
  if (model_path != "synthetic") return false;
  Impl &I = *impl_;
  I.resize = read_det_resize(resize);
  I.db = read_db_params(db);
  // GPU_CCL / GPU_BOX_THRESH / GPU_UNCLIP_SCALE (paddle_det.cpp:74-103):
  // empty or malformed values keep the default, parsed values are clamped.
  auto env_num = [](const char *name, float cur) {
    const char *v = std::getenv(name);
    if (!v || !*v) return cur;
    char *end = nullptr;
    const float x = std::strtof(v, &end);
    if (end == v || *end != '\0' || std::isnan(x)) {
      std::fprintf(stderr, "[PaddleDet] ignoring malformed %s=\"%s\"\n", name, v);
      return cur;
    }
    return x;
  };
  {
    const char *v = std::getenv("GPU_CCL");
    int mode = 1;
    if (v && *v) {
      char *end = nullptr;
      const long x = std::strtol(v, &end, 10);
      if (end == v || *end != '\0')
        std::fprintf(stderr, "[PaddleDet] ignoring malformed GPU_CCL=\"%s\"\n", v);
      else
        mode = (int)std::clamp<long>(x, 0, 2);
    }
    I.mode = mode;
  }
  I.box_thresh = std::clamp(env_num("GPU_BOX_THRESH", I.db.box_thresh), 0.001f, 1.0f);
  I.unclip_scale = std::clamp(env_num("GPU_UNCLIP_SCALE", 1.0f), 0.1f, 10.0f);
  I.max_side = effective_det_max_side(I.resize);
  I.allocate();
  I.loaded = true;
  return true;
}

TOCR_MOD_API std::vector<Box> PaddleDet::run(const GpuImage &img, int orig_h, int orig_w,
                                             cudaStream_t stream) {
  Impl &I = *impl_;
  if (!I.loaded) throw InferenceError("PaddleDet::run: no model loaded");
  const auto [rh, rw] = compute_det_resize(orig_h, orig_w, I.resize);
  if (rh > I.max_side || rw > I.max_side) throw InferenceError("PaddleDet::run: size beyond max side");
  throw_on_status(tocr_preprocess_one_f32(img.data, (int)img.step, img.rows, img.cols, I.canvas.p,
                                          rw, rh, nullptr, nullptr, stream),
                  "PaddleDet preprocess");
  I.h_geo.p[0] = orig_h;
  I.h_geo.p[1] = orig_w;
  I.h_geo.p[2] = rh;
  I.h_geo.p[3] = rw;
  I.h_content.p[0] = rh;
  I.h_content.p[1] = rw;
  cuda_check(cudaMemcpyAsync(I.geo.p, I.h_geo.p, 4 * sizeof(int), cudaMemcpyHostToDevice, stream),
             "PaddleDet H2D");
  cuda_check(cudaMemcpyAsync(I.content.p, I.h_content.p, 2 * sizeof(int), cudaMemcpyHostToDevice,
                             stream),
             "PaddleDet H2D");
  return std::move(I.post(1, rh, rw, stream)[0]);
}

TOCR_MOD_API std::vector<std::vector<Box>> PaddleDet::run_batch(
    const std::vector<GpuImage> &imgs, const std::vector<std::pair<int, int>> &dims,
    cudaStream_t stream) {
  Impl &I = *impl_;
  const int n = (int)imgs.size();
  if (n == 0) return {};
  if ((int)dims.size() != n) throw InferenceError("PaddleDet::run_batch: dims size mismatch");
  if (n == 1) {
    std::vector<std::vector<Box>> one;
    one.push_back(run(imgs[0], dims[0].first, dims[0].second, stream));
    I.last_scores.resize(1);
    return one;
  }
  if (!I.loaded) throw InferenceError("PaddleDet::run_batch: no model loaded");
  const int b = std::min(n, Impl::kMaxBatch);
  int H = 0, W = 0;
  for (int i = 0; i < b; ++i) {
    const auto [rh, rw] = compute_det_resize(dims[i].first, dims[i].second, I.resize);
    I.h_ptrs.p[i] = imgs[i].data;
    I.h_steps.p[i] = (int)imgs[i].step;
    I.h_sh.p[i] = imgs[i].rows;
    I.h_sw.p[i] = imgs[i].cols;
    I.h_dh.p[i] = rh;
    I.h_dw.p[i] = rw;
    I.h_geo.p[4 * i] = dims[i].first;
    I.h_geo.p[4 * i + 1] = dims[i].second;
    I.h_geo.p[4 * i + 2] = rh;
    I.h_geo.p[4 * i + 3] = rw;
    I.h_content.p[2 * i] = rh;
    I.h_content.p[2 * i + 1] = rw;
    H = std::max(H, rh);
    W = std::max(W, rw);
  }
  if (H > I.max_side || W > I.max_side) throw InferenceError("PaddleDet::run_batch: size beyond max side");
  auto up = [&](void *d, const void *h, size_t bytes) {
    cuda_check(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, stream), "PaddleDet H2D");
  };
  up(I.src_ptrs.p, I.h_ptrs.p, b * sizeof(void *));
  up(I.src_steps.p, I.h_steps.p, b * sizeof(int));
  up(I.src_h.p, I.h_sh.p, b * sizeof(int));
  up(I.src_w.p, I.h_sw.p, b * sizeof(int));
  up(I.dst_h.p, I.h_dh.p, b * sizeof(int));
  up(I.dst_w.p, I.h_dw.p, b * sizeof(int));
  up(I.geo.p, I.h_geo.p, 4 * b * sizeof(int));
  up(I.content.p, I.h_content.p, 2 * b * sizeof(int));
  throw_on_status(tocr_preprocess_batch_f32(I.src_ptrs.p, I.src_steps.p, I.src_h.p, I.src_w.p,
                                            I.dst_h.p, I.dst_w.p, I.canvas.p, W, H, b, nullptr,
                                            nullptr, stream),
                  "PaddleDet batch preprocess");
  std::vector<std::vector<Box>> out = I.post(b, H, W, stream);
  if (n > b) {  // the overflow goes through the single-image path
    std::vector<std::vector<float>> scores = std::move(I.last_scores);
    out.resize(n);
    scores.resize(n);
    for (int i = b; i < n; ++i) {
      out[i] = run(imgs[i], dims[i].first, dims[i].second, stream);
      scores[i] = std::move(I.last_scores[0]);
    }
    I.last_scores = std::move(scores);
  }
  return out;
}

TOCR_MOD_API const std::vector<std::vector<float>> &PaddleDet::last_scores() const {
  return impl_->last_scores;
}
TOCR_MOD_API const DetResizeParams &PaddleDet::resize_params() const { return impl_->resize; }
TOCR_MOD_API const DbParams &PaddleDet::db_params() const { return impl_->db; }

}  // namespace detection

// ----------------------------------------------------------------- PaddleCls --
namespace classification {

struct PaddleCls::Impl {
  static constexpr int kBatch = 128;         // kClsBatchNum
  static constexpr int kH = 80, kW = 160;    // kClsImageH / kClsImageW
  static constexpr float kThresh = 0.9f;     // kClsThresh
  static constexpr uint64_t kSeed = 0x7EC0C150ull;
  struct BlockCfg {
    int c, co, stride;
    float pw_scale;
  };
  static constexpr BlockCfg kBlocks[5] = {
      {32, 64, 1, 0.48f}, {64, 64, 2, 0.34f}, {64, 128, 1, 0.34f},
      {128, 128, 2, 0.24f}, {128, 256, 1, 0.24f}};

  bool loaded = false, allocated = false;
  DevBuf<__half_raw> crops, act0, act1;
  DevBuf<float> stem_w, stem_b, head_w, head_b, scores, minv;
  DevBuf<char> blobs[5];
  DevBuf<int> crop_w, crop_page, n_crops, err;
  PinBuf<float> h_scores, h_minv;
  PinBuf<int> h_crop_w, h_n;
  std::vector<std::array<float, 2>> last;

  static std::vector<float> synth(int k, float scale, size_t n) {
    std::vector<float> v(n);
    throw_on_status(tocr_synth_weights(kSeed + (uint64_t)k, scale, v.data(), (long long)n),
                    "PaddleCls weights");
    return v;
  }
  template <class T>
  static void upload(DevBuf<T> &d, const std::vector<T> &h) {
    d.alloc(h.size());
    cuda_check(cudaMemcpy(d.p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice),
               "PaddleCls weights H2D");
  }

  void load_weights() {
    upload(stem_w, synth(0, 0.53f, 32 * 27));
    upload(stem_b, synth(1, 0.1f, 32));
    for (int j = 0; j < 5; ++j) {
      const BlockCfg &b = kBlocks[j];
      const auto wdw = synth(16 + 4 * j, 0.9f, (size_t)b.c * 9);
      const auto bdw = synth(17 + 4 * j, 0.1f, (size_t)b.c);
      const auto wpw = synth(18 + 4 * j, b.pw_scale, (size_t)b.co * b.c);
      const auto bpw = synth(19 + 4 * j, 0.1f, (size_t)b.co);
      const size_t bytes = tocr_dwpw_packed_bytes(b.c, b.co);
      std::vector<char> blob(bytes);
      throw_on_status(tocr_dwpw_pack(b.c, b.co, 0, wdw.data(), bdw.data(), wpw.data(),
                                     bpw.data(), blob.data(), bytes),
                      "PaddleCls block pack");
      upload(blobs[j], blob);
    }
    upload(head_w, synth(64, 1.0f, 2 * 256));
    upload(head_b, synth(65, 0.1f, 2));
  }

  void allocate() {
    if (allocated) return;
    crops.alloc((size_t)kBatch * 3 * kH * kW);
    act0.alloc((size_t)kBatch * (kH / 2) * (kW / 2) * 64);
    act1.alloc((size_t)kBatch * (kH / 2) * (kW / 2) * 64);
    scores.alloc((size_t)kBatch * 2);
    minv.alloc((size_t)kBatch * 9);
    crop_w.alloc(kBatch);
    n_crops.alloc(1);
    err.alloc(1);
    crop_page.alloc(kBatch);
    cuda_check(cudaMemset(crop_page.p, 0, kBatch * sizeof(int)), "PaddleCls memset");
    cuda_check(cudaMemset(err.p, 0, sizeof(int)), "PaddleCls memset");
    h_scores.alloc((size_t)kBatch * 2);
    h_minv.alloc((size_t)kBatch * 9);
    h_crop_w.alloc(kBatch);
    h_n.alloc(1);
    allocated = true;
  }
};

TOCR_MOD_API PaddleCls::PaddleCls() : impl_(std::make_unique<Impl>()) {}
TOCR_MOD_API PaddleCls::~PaddleCls() noexcept = default;

TOCR_MOD_API bool PaddleCls::load_model(const std::string &model_path) {
  if (model_path != "synthetic") return false;
  impl_->load_weights();
  impl_->loaded = true;
  return true;
}

TOCR_MOD_API void PaddleCls::allocate_buffers() { impl_->allocate(); }

TOCR_MOD_API const std::vector<std::array<float, 2>> &PaddleCls::last_scores() const {
  return impl_->last;
}

TOCR_MOD_API void PaddleCls::run(const GpuImage &img, std::vector<Box> &boxes,
                                 cudaStream_t stream) {
  Impl &I = *impl_;
  I.last.clear();
  if (boxes.empty()) return;
  if (!I.loaded) throw InferenceError("PaddleCls::run: no model loaded");
  if (img.step > (size_t)INT_MAX) throw InferenceError("PaddleCls::run: image step too large");
  I.allocate();
  const int total = (int)boxes.size();
  I.last.resize(total);
  for (int beg = 0; beg < total; beg += Impl::kBatch) {
    const int nb = std::min(Impl::kBatch, total - beg);
    for (int j = 0; j < nb; ++j) {
      const CropTransform ct = compute_crop_transform(boxes[beg + j], Impl::kH, Impl::kW);
      I.h_crop_w.p[j] = ct.crop_width;
      std::memcpy(I.h_minv.p + 9 * j, ct.M_inv, 9 * sizeof(float));
    }
    I.h_n.p[0] = nb;
    cuda_check(cudaMemcpyAsync(I.minv.p, I.h_minv.p, (size_t)nb * 9 * sizeof(float),
                               cudaMemcpyHostToDevice, stream), "PaddleCls H2D");
    cuda_check(cudaMemcpyAsync(I.crop_w.p, I.h_crop_w.p, (size_t)nb * sizeof(int),
                               cudaMemcpyHostToDevice, stream), "PaddleCls H2D");
    cuda_check(cudaMemcpyAsync(I.n_crops.p, I.h_n.p, sizeof(int), cudaMemcpyHostToDevice, stream),
               "PaddleCls H2D");
    throw_on_status(tocr_roi_warp_f16(static_cast<const uint8_t *>(img.data), 0, img.rows,
                                      img.cols, (int)img.step, I.minv.p, I.crop_w.p,
                                      I.crop_page.p, I.n_crops.p, nb, Impl::kH, Impl::kW,
                                      nullptr, nullptr, 1.0f / 255.0f, I.crops.p, stream),
                    "PaddleCls crops");
    throw_on_status(tocr_cls_stem_f16(I.crops.p, nb, Impl::kH, Impl::kW, I.stem_w.p, I.stem_b.p,
                                      I.act0.p, stream),
                    "PaddleCls stem");
    int h = Impl::kH / 2, w = Impl::kW / 2;
    DevBuf<__half_raw> *src = &I.act0, *dst = &I.act1;
    for (int j = 0; j < 5; ++j) {
      const Impl::BlockCfg &b = Impl::kBlocks[j];
      throw_on_status(tocr_dwpw_block(src->p, dst->p, nb, h, w, b.c, b.co, b.stride, 0,
                                      I.blobs[j].p, I.err.p, stream),
                      "PaddleCls block");
      h = (h - 1) / b.stride + 1;
      w = (w - 1) / b.stride + 1;
      std::swap(src, dst);
    }
    throw_on_status(tocr_cls_head_f32(src->p, nb, h * w, 256, I.head_w.p, I.head_b.p, I.scores.p,
                                      stream),
                    "PaddleCls head");
    cuda_check(cudaMemcpyAsync(I.h_scores.p, I.scores.p, (size_t)nb * 2 * sizeof(float),
                               cudaMemcpyDeviceToHost, stream), "PaddleCls D2H");
    cuda_check(cudaStreamSynchronize(stream), "PaddleCls sync");
    for (int j = 0; j < nb; ++j) {
      const float s0 = I.h_scores.p[2 * j], s180 = I.h_scores.p[2 * j + 1];
      I.last[beg + j] = {s0, s180};
      if (s180 > s0 && s180 > Impl::kThresh) {
        Box &box = boxes[beg + j];
        std::swap(box[0], box[2]);
        std::swap(box[1], box[3]);
      }
    }
  }
}

}  // namespace classification

// ----------------------------------------------------------------- PaddleRec --
namespace recognition {

struct PaddleRec::Impl {
  static constexpr int kMaxSlots = 20;  // paddle_rec.h:120
  int batch_num = 32;
  int rec_h = 48;
  bool loaded = false;
  bool allocated = false;
  int num_classes = 0;  // = labels.size() for the stand-in network
  std::vector<std::string> labels{"blank"};
  int dropped = 0;
  std::vector<int> dropped_per_image;

  DevBuf<float> input;     // [batch][3][48][kMaxRecWidth] fp32 crops
  DevBuf<uint16_t> logits; // [batch][T][V] fp16
  DevBuf<float> minv;
  DevBuf<int> crop_w, step_idx;
  DevBuf<float> step_prob;
  struct Slot {
    DevBuf<int> tokens, lengths, ids;
    DevBuf<float> scores;
    PinBuf<int> h_tokens, h_lengths, h_ids, h_crop_w;
    PinBuf<float> h_scores, h_minv;
  };
  Slot slots[kMaxSlots];

  static int max_steps() { return kMaxRecWidth / 4; }

  void allocate() {
    if (allocated) return;
    if (num_classes < 2) throw ModelLoadError("PaddleRec: load_model and load_dict first");
    const int T = max_steps();
    input.alloc((size_t)batch_num * 3 * rec_h * kMaxRecWidth);
    logits.alloc((size_t)batch_num * T * num_classes);
    minv.alloc((size_t)batch_num * 9);
    crop_w.alloc(batch_num);
    step_idx.alloc((size_t)batch_num * T);
    step_prob.alloc((size_t)batch_num * T);
    for (Slot &s : slots) {
      s.tokens.alloc((size_t)batch_num * T);
      s.lengths.alloc(batch_num);
      s.scores.alloc(batch_num);
      s.ids.alloc(batch_num);
      s.h_tokens.alloc((size_t)batch_num * T);
      s.h_lengths.alloc(batch_num);
      s.h_scores.alloc(batch_num);
      s.h_ids.alloc(batch_num);
      s.h_crop_w.alloc(batch_num);
      s.h_minv.alloc((size_t)batch_num * 9);
    }
    allocated = true;
  }

  struct Record {
    int beg, end, seq_len, slot;
  };

  // The deferred-sync queue loop (paddle_rec.cpp:215-314). Crop i of the
  // caller's width-sorted order: bucket(i), box(i), id(i) (the stand-in's
  // key), warp(beg, count, width) queues the crops' ROI warps, emit(i, r)
  // receives the result.
  template <class Bucket, class BoxAt, class Id, class Warp, class Emit>
  void queue_loop(int total, const Bucket &bucket, const BoxAt &box_at, const Id &id,
                  const Warp &warp, const Emit &emit, cudaStream_t st) {
    std::vector<Record> recs;
    auto decode = [&]() {
      for (const Record &r : recs) {
        Slot &s = slots[r.slot];
        for (int j = 0; j < r.end - r.beg; ++j) {
          const int *toks = s.h_tokens.p + (size_t)j * r.seq_len;
          emit(r.beg + j, std::make_pair(ctc_tokens_to_text(toks, s.h_lengths.p[j], labels),
                                         s.h_scores.p[j]));
        }
      }
      recs.clear();
    };
    int beg = 0, slot = 0;
    while (beg < total) {
      const int w = bucket(beg);
      int end = beg;
      while (end < total && end - beg < batch_num && bucket(end) == w) ++end;
      const int n = end - beg;
      if (slot >= kMaxSlots) {
        cuda_check(cudaStreamSynchronize(st), "PaddleRec sync");
        decode();
        slot = 0;
      }
      Slot &s = slots[slot];
      for (int j = 0; j < n; ++j) {
        const CropTransform ct = compute_crop_transform(box_at(beg + j), rec_h, w);
        s.h_crop_w.p[j] = ct.crop_width;
        std::memcpy(s.h_minv.p + 9 * j, ct.M_inv, 9 * sizeof(float));
        s.h_ids.p[j] = id(beg + j);
      }
      cuda_check(cudaMemcpyAsync(minv.p, s.h_minv.p, 9 * n * sizeof(float),
                                 cudaMemcpyHostToDevice, st), "PaddleRec H2D");
      cuda_check(cudaMemcpyAsync(crop_w.p, s.h_crop_w.p, n * sizeof(int), cudaMemcpyHostToDevice,
                                 st), "PaddleRec H2D");
      cuda_check(cudaMemcpyAsync(s.ids.p, s.h_ids.p, n * sizeof(int), cudaMemcpyHostToDevice, st),
                 "PaddleRec H2D");
      warp(beg, n, w);
      const int T = w / 4;
      throw_on_status(tocr_rec_standin_logits_f16(logits.p, s.ids.p, n, T, num_classes,
                                                  kStandinSeed, st),
                      "PaddleRec stand-in network");
      throw_on_status(tocr_ctc_greedy_f16(logits.p, n, T, num_classes,
                                          (int)labels.size(), s.tokens.p, s.lengths.p, s.scores.p,
                                          step_idx.p, step_prob.p, st),
                      "PaddleRec CTC");
      cuda_check(cudaMemcpyAsync(s.h_tokens.p, s.tokens.p, (size_t)n * T * sizeof(int),
                                 cudaMemcpyDeviceToHost, st), "PaddleRec D2H");
      cuda_check(cudaMemcpyAsync(s.h_lengths.p, s.lengths.p, n * sizeof(int),
                                 cudaMemcpyDeviceToHost, st), "PaddleRec D2H");
      cuda_check(cudaMemcpyAsync(s.h_scores.p, s.scores.p, n * sizeof(float),
                                 cudaMemcpyDeviceToHost, st), "PaddleRec D2H");
      recs.push_back({beg, end, T, slot});
      ++slot;
      beg = end;
    }
    cuda_check(cudaStreamSynchronize(st), "PaddleRec sync");
    decode();
  }
};

TOCR_MOD_API PaddleRec::PaddleRec() : impl_(std::make_unique<Impl>()) {}
TOCR_MOD_API PaddleRec::~PaddleRec() noexcept = default;

TOCR_MOD_API void PaddleRec::set_batch_num(int n) {
  if (!impl_->allocated && n > 0) impl_->batch_num = n;
}

TOCR_MOD_API bool PaddleRec::load_model(const std::string &model_path) {
  if (model_path != "synthetic") return false;
  impl_->loaded = true;
  if (impl_->labels.size() > 1) impl_->num_classes = (int)impl_->labels.size();
  return true;
}

TOCR_MOD_API bool PaddleRec::load_dict(const std::string &dict_path) {
  std::vector<std::string> labels{"blank"};
  if (!load_label_dict(dict_path, labels)) return false;
  if (impl_->allocated && (int)labels.size() != impl_->num_classes)
    throw ModelLoadError("PaddleRec: dictionary width differs from the allocated model width");
  impl_->labels = std::move(labels);
  impl_->num_classes = (int)impl_->labels.size();
  return true;
}

TOCR_MOD_API void PaddleRec::allocate_buffers() { impl_->allocate(); }
TOCR_MOD_API void PaddleRec::bake_graphs(cudaStream_t) { impl_->allocate(); }
TOCR_MOD_API int PaddleRec::last_dropped_crops() const { return impl_->dropped; }
TOCR_MOD_API const std::vector<int> &PaddleRec::last_dropped_per_image() const {
  return impl_->dropped_per_image;
}

TOCR_MOD_API std::vector<std::pair<std::string, float>> PaddleRec::run(
    const GpuImage &img, const std::vector<Box> &boxes, cudaStream_t stream) {
  Impl &I = *impl_;
  std::vector<std::pair<std::string, float>> results;
  if (boxes.empty()) return results;
  if (!I.loaded) throw InferenceError("PaddleRec::run: no model loaded");
  I.allocate();
  I.dropped = 0;
  I.dropped_per_image.clear();
  const int total = (int)boxes.size();
  results.resize(total);
  struct Crop {
    int idx, bucket;
  };
  std::vector<Crop> crops(total);
  for (int i = 0; i < total; ++i) crops[i] = {i, snap_width_bucket(rec_input_width(boxes[i], I.rec_h))};
  std::stable_sort(crops.begin(), crops.end(),
                   [](const Crop &a, const Crop &b) { return a.bucket < b.bucket; });
  I.queue_loop(
      total, [&](int i) { return crops[i].bucket; },
      [&](int i) -> const Box & { return boxes[crops[i].idx]; }, [&](int i) { return crops[i].idx; },
      [&](int, int n, int w) {
        throw_on_status(tocr_roi_warp_f32(static_cast<const uint8_t *>(img.data), img.rows,
                                          img.cols, (int)img.step, I.minv.p, I.crop_w.p, n,
                                          I.rec_h, w, nullptr, nullptr, 1.0f / 255.0f, I.input.p,
                                          stream),
                        "PaddleRec ROI warp");
      },
      [&](int ci, std::pair<std::string, float> &&r) { results[crops[ci].idx] = std::move(r); },
      stream);
  return results;
}

TOCR_MOD_API std::vector<std::vector<std::pair<std::string, float>>> PaddleRec::run_multi(
    const std::vector<ImageCrops> &image_crops, cudaStream_t stream) {
  Impl &I = *impl_;
  const int n_img = (int)image_crops.size();
  std::vector<std::vector<std::pair<std::string, float>>> all(n_img);
  int total = 0;
  for (int i = 0; i < n_img; ++i) {
    all[i].resize(image_crops[i].boxes.size());
    total += (int)image_crops[i].boxes.size();
  }
  if (total == 0) return all;
  if (!I.loaded) throw InferenceError("PaddleRec::run_multi: no model loaded");
  I.allocate();
  I.dropped = 0;
  I.dropped_per_image.assign(n_img, 0);
  struct Crop {
    int img, box, bucket, id;
  };
  std::vector<Crop> crops;
  crops.reserve(total);
  for (int i = 0, id = 0; i < n_img; ++i)
    for (int b = 0; b < (int)image_crops[i].boxes.size(); ++b, ++id)
      crops.push_back({i, b, snap_width_bucket(rec_input_width(image_crops[i].boxes[b], I.rec_h)),
                       id});
  std::stable_sort(crops.begin(), crops.end(), [](const Crop &a, const Crop &b) {
    if (a.bucket != b.bucket) return a.bucket < b.bucket;
    return a.img < b.img;
  });
  I.queue_loop(
      total, [&](int i) { return crops[i].bucket; },
      [&](int i) -> const Box & { return image_crops[crops[i].img].boxes[crops[i].box]; },
      [&](int i) { return crops[i].id; },
      [&](int beg, int n, int w) {  // one warp launch per run of crops of one image
        const size_t stride = (size_t)3 * I.rec_h * w;
        for (int j = 0; j < n;) {
          const int src = crops[beg + j].img, start = j;
          while (j < n && crops[beg + j].img == src) ++j;
          const GpuImage &img = image_crops[src].img;
          throw_on_status(tocr_roi_warp_f32(static_cast<const uint8_t *>(img.data), img.rows,
                                            img.cols, (int)img.step, I.minv.p + 9 * start,
                                            I.crop_w.p + start, j - start, I.rec_h, w, nullptr,
                                            nullptr, 1.0f / 255.0f, I.input.p + start * stride,
                                            stream),
                          "PaddleRec ROI warp");
        }
      },
      [&](int ci, std::pair<std::string, float> &&r) {
        all[crops[ci].img][crops[ci].box] = std::move(r);
      },
      stream);
  return all;
}

}  // namespace recognition
}  // namespace turbo_ocr
