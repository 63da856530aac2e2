// Test driver for the C++ interface of libtocr_b200.so, compiled by the tests
// with g++ against include/ exactly as a reference-side caller would be.
//
//   modules_test host <dict>            host-only API (no GPU): crop transform,
//                                       box utilities, CTC helpers, combine step
//   modules_test gpu <pages> <n> <dict> <outdir>
//                                       PaddleDet -> sorted_boxes -> PaddleRec ->
//                                       combine_recognition on n 960x960 pages, and
//                                       the reference-signature kernel shims; JSON on
//                                       stdout, raw kernel outputs in outdir
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "tocr_capi.h"
#include "turbo_ocr/classification/paddle_cls.h"
#include "turbo_ocr/common/errors.h"
#include "turbo_ocr/common/geometry/box.h"
#include "turbo_ocr/common/geometry/perspective.h"
#include "turbo_ocr/common/types.h"
#include "turbo_ocr/detection/det_config.h"
#include "turbo_ocr/detection/det_postprocess.h"
#include "turbo_ocr/detection/paddle_det.h"
#include "turbo_ocr/kernels/kernels.h"
#include "turbo_ocr/pipeline/classify_angles.h"
#include "turbo_ocr/pipeline/ocr_pipeline_detail.h"
#include "turbo_ocr/recognition/ctc_decode.h"
#include "turbo_ocr/recognition/paddle_rec.h"
#include "turbo_ocr/recognition/rec_geometry.h"

using namespace turbo_ocr;

namespace {

std::string jstr(const std::string &s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    if (c == '"' || c == '\\') { o += '\\'; o += (char)c; }
    else if (c < 0x20) { char b[8]; std::snprintf(b, sizeof b, "\\u%04x", c); o += b; }
    else o += (char)c;
  }
  return o + "\"";
}
std::string jbox(const Box &b) {
  std::string o = "[";
  for (int k = 0; k < 4; ++k) {
    o += "[" + std::to_string(b[k][0]) + "," + std::to_string(b[k][1]) + "]";
    if (k < 3) o += ",";
  }
  return o + "]";
}
void ck(cudaError_t e, const char *w) {
  if (e != cudaSuccess) { std::fprintf(stderr, "%s: %s\n", w, cudaGetErrorString(e)); std::exit(2); }
}
template <class T>
void dump(const std::string &path, const T *d, size_t n) {
  std::vector<T> h(n);
  ck(cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost), "dump");
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char *>(h.data()), (std::streamsize)(n * sizeof(T)));
}

int host_mode(const std::string &dict) {
  std::printf("{");
  // crop transforms and widths of a few quads
  const Box qs[] = {{{{{10, 20}, {210, 24}, {209, 60}, {9, 56}}}},
                    {{{{5, 5}, {25, 5}, {25, 200}, {5, 200}}}},
                    {{{{0, 0}, {3000, 0}, {3000, 20}, {0, 20}}}}};
  std::printf("\"crops\":[");
  for (int i = 0; i < 3; ++i) {
    const CropTransform ct = compute_crop_transform(qs[i], 48, 320);
    std::printf("%s{\"w\":%d,\"v\":%d,\"m\":[", i ? "," : "", ct.crop_width, (int)ct.vertical);
    for (int k = 0; k < 9; ++k) std::printf("%s%.9g", k ? "," : "", (double)ct.M_inv[k]);
    std::printf("],\"rw\":%d,\"bucket\":%d,\"vert\":%d}", recognition::rec_input_width(qs[i], 48),
                recognition::snap_width_bucket(recognition::rec_input_width(qs[i], 48)),
                (int)is_vertical_box(qs[i]));
  }
  std::printf("],");
  // reading order
  std::vector<Box> bs = {{{{{50, 31}, {90, 31}, {90, 40}, {50, 40}}}},
                         {{{{10, 35}, {40, 35}, {40, 45}, {10, 45}}}},
                         {{{{5, 2}, {9, 2}, {9, 8}, {5, 8}}}},
                         {{{{1, 39}, {4, 39}, {4, 49}, {1, 49}}}}};
  sorted_boxes(bs);
  std::printf("\"sorted\":[");
  for (size_t i = 0; i < bs.size(); ++i) std::printf("%s%s", i ? "," : "", jbox(bs[i]).c_str());
  std::printf("],");
  // quad order
  float xs[4] = {3.f, 1.f, 1.f, 3.f}, ys[4] = {5.f, 5.f, 1.f, 1.f};
  detection::order_quad_tl_tr_br_bl(xs, ys);
  std::printf("\"quad\":[%g,%g,%g,%g,%g,%g,%g,%g],", xs[0], ys[0], xs[1], ys[1], xs[2], ys[2],
              xs[3], ys[3]);
  // dictionary and CTC helpers
  std::vector<std::string> labels{"blank"};
  const bool ok = recognition::load_label_dict(dict, labels);
  std::printf("\"dict_ok\":%d,\"labels\":[", (int)ok);
  for (size_t i = 0; i < labels.size(); ++i) std::printf("%s%s", i ? "," : "", jstr(labels[i]).c_str());
  std::printf("],");
  const int idx[] = {0, 1, 1, 0, 2, 2, 3, 0, 3};
  const float sc[] = {0.9f, 0.8f, 0.7f, 0.9f, 0.6f, 0.5f, 0.4f, 0.9f, 0.2f};
  auto [t1, s1] = recognition::ctc_greedy_decode(idx, sc, 9, labels);
  std::vector<float> raw(9 * (int)labels.size(), 0.f);
  for (int t = 0; t < 9; ++t) raw[t * labels.size() + idx[t]] = sc[t];
  auto [t2, s2] = recognition::ctc_greedy_decode_raw(raw.data(), 9, (int)labels.size(), labels);
  std::printf("\"ctc\":[%s,%.9g,%s,%.9g],", jstr(t1).c_str(), (double)s1, jstr(t2).c_str(),
              (double)s2);
  // combine
  pipeline::OcrPipelineResult r;
  std::vector<Box> boxes = {qs[0], qs[1], qs[2]};
  std::vector<std::pair<std::string, float>> rec = {{"ab", 0.9f}, {"", 0.99f}, {"c", 0.49f}};
  pipeline::detail::combine_recognition(r, boxes, rec);
  pipeline::OcrPipelineResult r2;
  std::vector<std::pair<std::string, float>> rec2 = {{"", 0.9f}};
  pipeline::detail::combine_recognition(r2, boxes, rec2);
  pipeline::detail::flag_dropped_crops(r2, 2);
  std::printf("\"combine\":[%d,%s,%d,%d,%s],", (int)r.results.size(),
              r.results.empty() ? "\"\"" : jstr(r.results[0].text).c_str(), (int)r.text_degraded,
              (int)r2.text_degraded, jstr(r2.text_warning).c_str());
  // resize policy through the C++ header
  const auto [rh, rw] = detection::compute_det_resize(960, 1280, {"max", 960, 960});
  std::printf("\"resize\":[%d,%d]}\n", rh, rw);
  return 0;
}

int gpu_mode(const std::string &pages_path, int n, const std::string &dict, const std::string &out) {
  const int H = 960, W = 960;
  const size_t page_bytes = (size_t)H * W * 3;
  std::vector<unsigned char> host(page_bytes * n);
  {
    std::ifstream f(pages_path, std::ios::binary);
    f.read(reinterpret_cast<char *>(host.data()), (std::streamsize)host.size());
    if (!f) { std::fprintf(stderr, "cannot read pages\n"); return 2; }
  }
  unsigned char *d_pages = nullptr;
  ck(cudaMalloc(&d_pages, host.size()), "malloc");
  ck(cudaMemcpy(d_pages, host.data(), host.size(), cudaMemcpyHostToDevice), "H2D");
  cudaStream_t st;
  ck(cudaStreamCreate(&st), "stream");
  std::vector<GpuImage> imgs(n);
  std::vector<std::pair<int, int>> dims(n, {H, W});
  for (int i = 0; i < n; ++i) imgs[i] = GpuImage{d_pages + i * page_bytes, (size_t)W * 3, H, W};

  detection::PaddleDet det;
  if (!det.load_model("synthetic", {"max", 960, 960}, {0.3f, 0.6f, 1.5f})) return 3;
  if (det.load_model("/no/such/engine.trt")) return 4;
  auto boxes = det.run_batch(imgs, dims, st);
  auto scores = det.last_scores();
  auto single = det.run(imgs[0], H, W, st);
  const bool single_same = single == boxes[0];
  for (auto &b : boxes) sorted_boxes(b);

  recognition::PaddleRec rec;
  if (!rec.load_model("synthetic") || !rec.load_dict(dict)) return 5;
  std::vector<recognition::PaddleRec::ImageCrops> crops(n);
  for (int i = 0; i < n; ++i) crops[i] = {imgs[i], boxes[i]};
  auto multi = rec.run_multi(crops, st);
  auto one = rec.run(imgs[0], boxes[0], st);
  const bool run_same = one == multi[0];

  std::printf("{\"single_same\":%d,\"run_same\":%d,\"pages\":[", (int)single_same, (int)run_same);
  for (int i = 0; i < n; ++i) {
    pipeline::OcrPipelineResult res;
    auto r = multi[i];
    pipeline::detail::combine_recognition(res, boxes[i], r);
    std::printf("%s{\"boxes\":[", i ? "," : "");
    for (size_t k = 0; k < boxes[i].size(); ++k) std::printf("%s%s", k ? "," : "", jbox(boxes[i][k]).c_str());
    std::printf("],\"det_scores\":[");
    for (size_t k = 0; k < scores[i].size(); ++k) std::printf("%s%.7g", k ? "," : "", (double)scores[i][k]);
    std::printf("],\"texts\":[");
    for (size_t k = 0; k < multi[i].size(); ++k)
      std::printf("%s[%s,%.7g]", k ? "," : "", jstr(multi[i][k].first).c_str(), (double)multi[i][k].second);
    std::printf("],\"kept\":%d,\"degraded\":%d}", (int)res.results.size(), (int)res.text_degraded);
  }
  std::printf("],");

  // reference-signature kernel shims on page 0
  float *d_chw = nullptr;
  ck(cudaMalloc(&d_chw, sizeof(float) * 3 * 736 * 960), "malloc");
  kernels::cuda_fused_resize_normalize_det(imgs[0], d_chw, 960, 736, st);  // squash to 736 rows
  ck(cudaStreamSynchronize(st), "sync");
  dump(out + "/fused_det.f32", d_chw, (size_t)3 * 736 * 960);
  const int nb = std::min<int>(8, (int)boxes[0].size());
  std::vector<float> minv(9 * nb);
  std::vector<int> cw(nb);
  for (int k = 0; k < nb; ++k) {
    const CropTransform ct = compute_crop_transform(boxes[0][k], 48, 320);
    std::memcpy(&minv[9 * k], ct.M_inv, 9 * sizeof(float));
    cw[k] = ct.crop_width;
  }
  float *d_minv = nullptr, *d_crops = nullptr;
  int *d_cw = nullptr;
  ck(cudaMalloc(&d_minv, sizeof(float) * 9 * 8), "malloc");
  ck(cudaMalloc(&d_cw, sizeof(int) * 8), "malloc");
  ck(cudaMalloc(&d_crops, sizeof(float) * 8 * 3 * 48 * 320), "malloc");
  ck(cudaMemcpy(d_minv, minv.data(), sizeof(float) * 9 * nb, cudaMemcpyHostToDevice), "H2D");
  ck(cudaMemcpy(d_cw, cw.data(), sizeof(int) * nb, cudaMemcpyHostToDevice), "H2D");
  kernels::cuda_batch_roi_warp(imgs[0], d_minv, d_cw, d_crops, nb, 48, 320, st);
  ck(cudaStreamSynchronize(st), "sync");
  dump(out + "/roi_warp.f32", d_crops, (size_t)nb * 3 * 48 * 320);
  dump(out + "/roi_minv.f32", d_minv, (size_t)nb * 9);
  dump(out + "/roi_cw.i32", d_cw, (size_t)nb);
  // threshold + GPU CCL on the stand-in probability map of that canvas
  float *d_prob = nullptr;
  ck(cudaMalloc(&d_prob, sizeof(float) * 736 * 960), "malloc");
  throw_on_status(tocr_det_standin_prob_f32(d_chw, 1, 736, 960, nullptr, nullptr, nullptr, 12.f,
                                            d_prob, st), "stand-in prob");
  dump(out + "/prob.f32", d_prob, (size_t)736 * 960);
  unsigned char *d_bm = nullptr;
  ck(cudaMalloc(&d_bm, 736 * 960), "malloc");
  kernels::cuda_threshold_to_u8(d_prob, d_bm, 960, 736, 0.3f, st);
  int *d_labels = nullptr, *d_cid = nullptr, *d_cnt = nullptr, *d_nb = nullptr;
  kernels::GpuDetBox *d_boxes = nullptr, *h_boxes = nullptr;
  ck(cudaMalloc(&d_labels, sizeof(int) * 736 * 960), "malloc");
  ck(cudaMalloc(&d_cid, sizeof(int) * 736 * 960), "malloc");
  ck(cudaMalloc(&d_cnt, sizeof(int)), "malloc");
  ck(cudaMalloc(&d_nb, sizeof(int)), "malloc");
  ck(cudaMalloc(&d_boxes, sizeof(kernels::GpuDetBox) * 2 * kernels::kMaxGpuComponents), "malloc");
  ck(cudaMallocHost(&h_boxes, sizeof(kernels::GpuDetBox) * kernels::kMaxGpuComponents), "malloc");
  int h_nb = 0, h_total = 0;
  const int kept = kernels::cuda_gpu_ccl_detect(d_bm, d_prob, 960, 736, 0.6f, d_labels, d_cid, d_cnt,
                                                d_boxes, d_nb, h_boxes, &h_nb, st, &h_total);
  dump(out + "/threshold.u8", d_bm, (size_t)736 * 960);
  std::printf("\"ccl\":{\"kept\":%d,\"total\":%d,\"boxes\":[", kept, h_total);
  for (int k = 0; k < kept; ++k)
    std::printf("%s[%d,%d,%d,%d,%d,%.7g]", k ? "," : "", h_boxes[k].xmin, h_boxes[k].ymin,
                h_boxes[k].xmax, h_boxes[k].ymax, h_boxes[k].pixel_count, (double)h_boxes[k].score);
  std::printf("]},");
  // argmax shim on a few rows
  std::vector<float> rows(4 * 37);
  for (size_t i = 0; i < rows.size(); ++i) rows[i] = (float)((i * 7919) % 101) - 50.f;
  rows[37 + 5] = rows[37 + 9] = 1000.f;  // a tie: the lower index wins
  float *d_rows = nullptr, *d_sc = nullptr;
  int *d_idx = nullptr;
  ck(cudaMalloc(&d_rows, rows.size() * sizeof(float)), "malloc");
  ck(cudaMalloc(&d_sc, 4 * sizeof(float)), "malloc");
  ck(cudaMalloc(&d_idx, 4 * sizeof(int)), "malloc");
  ck(cudaMemcpy(d_rows, rows.data(), rows.size() * sizeof(float), cudaMemcpyHostToDevice), "H2D");
  kernels::cuda_argmax(d_rows, d_idx, d_sc, 2, 2, 37, st);
  int hi[4];
  float hs[4];
  ck(cudaMemcpy(hi, d_idx, sizeof hi, cudaMemcpyDeviceToHost), "D2H");
  ck(cudaMemcpy(hs, d_sc, sizeof hs, cudaMemcpyDeviceToHost), "D2H");
  std::printf("\"argmax\":[[%d,%d,%d,%d],[%g,%g,%g,%g]],", hi[0], hi[1], hi[2], hi[3], hs[0], hs[1],
              hs[2], hs[3]);
  // a failing call surfaces as the reference's exception type
  bool threw = false;
  try {
    kernels::cuda_batch_threshold_to_u8(d_chw, d_bm, -1, 10, 1, 0.5f, st);
  } catch (const CudaError &) {
    threw = true;
  }
  std::printf("\"throws\":%d}\n", (int)threw);
  ck(cudaStreamSynchronize(st), "sync");
  return 0;
}

// PaddleDet with GPU_CCL=2 (set by the caller): run_batch and run on the
// pages; the stand-in probability map of every page as PaddleDet computes it
// (the map the mode-2 chain starts from) goes to <outdir>/prob<i>.f32.
int det2_mode(const std::string &pages_path, int n, const std::string &out) {
  const int H = 960, W = 960;
  const size_t page_bytes = (size_t)H * W * 3;
  std::vector<unsigned char> host(page_bytes * n);
  {
    std::ifstream f(pages_path, std::ios::binary);
    f.read(reinterpret_cast<char *>(host.data()), (std::streamsize)host.size());
    if (!f) { std::fprintf(stderr, "cannot read pages\n"); return 2; }
  }
  unsigned char *d_pages = nullptr;
  ck(cudaMalloc(&d_pages, host.size()), "malloc");
  ck(cudaMemcpy(d_pages, host.data(), host.size(), cudaMemcpyHostToDevice), "H2D");
  cudaStream_t st;
  ck(cudaStreamCreate(&st), "stream");
  std::vector<GpuImage> imgs(n);
  std::vector<std::pair<int, int>> dims(n, {H, W});
  for (int i = 0; i < n; ++i) imgs[i] = GpuImage{d_pages + i * page_bytes, (size_t)W * 3, H, W};
  detection::PaddleDet det;
  if (!det.load_model("synthetic", {"max", 960, 960}, {0.3f, 0.6f, 1.5f})) return 3;
  auto boxes = det.run_batch(imgs, dims, st);
  auto scores = det.last_scores();
  auto single = det.run(imgs[0], H, W, st);
  float *d_chw = nullptr, *d_prob = nullptr;
  ck(cudaMalloc(&d_chw, sizeof(float) * 3 * H * W), "malloc");
  ck(cudaMalloc(&d_prob, sizeof(float) * H * W), "malloc");
  for (int i = 0; i < n; ++i) {
    throw_on_status(tocr_preprocess_one_f32(imgs[i].data, (int)imgs[i].step, H, W, d_chw, W, H,
                                            nullptr, nullptr, st), "preprocess");
    throw_on_status(tocr_det_standin_prob_f32(d_chw, 1, H, W, nullptr, nullptr, nullptr, 12.f,
                                              d_prob, st), "stand-in prob");
    ck(cudaStreamSynchronize(st), "sync");
    dump(out + "/prob" + std::to_string(i) + ".f32", d_prob, (size_t)H * W);
  }
  std::printf("{\"single_same\":%d,\"pages\":[", (int)(single == boxes[0]));
  for (int i = 0; i < n; ++i) {
    std::printf("%s{\"boxes\":[", i ? "," : "");
    for (size_t k = 0; k < boxes[i].size(); ++k) std::printf("%s%s", k ? "," : "", jbox(boxes[i][k]).c_str());
    std::printf("],\"scores\":[");
    for (size_t k = 0; k < scores[i].size(); ++k) std::printf("%s%.9g", k ? "," : "", (double)scores[i][k]);
    std::printf("]}");
  }
  std::printf("]}\n");
  return 0;
}

// PaddleCls on page 0: the boxes PaddleDet finds plus a few vertical ones;
// run() on all of them and the pipeline's gated classify_angles().
int cls_mode(const std::string &pages_path, const std::string &out) {
  (void)out;
  const int H = 960, W = 960;
  std::vector<unsigned char> host((size_t)H * W * 3);
  {
    std::ifstream f(pages_path, std::ios::binary);
    f.read(reinterpret_cast<char *>(host.data()), (std::streamsize)host.size());
    if (!f) { std::fprintf(stderr, "cannot read pages\n"); return 2; }
  }
  unsigned char *d_page = nullptr;
  ck(cudaMalloc(&d_page, host.size()), "malloc");
  ck(cudaMemcpy(d_page, host.data(), host.size(), cudaMemcpyHostToDevice), "H2D");
  cudaStream_t st;
  ck(cudaStreamCreate(&st), "stream");
  const GpuImage img{d_page, (size_t)W * 3, H, W};
  detection::PaddleDet det;
  if (!det.load_model("synthetic", {"max", 960, 960}, {0.3f, 0.6f, 1.5f})) return 3;
  std::vector<Box> all = det.run(img, H, W, st);
  for (int k = 0; k < 12; ++k) {  // vertical strips across the text lines
    const int x = 40 + 70 * k, y = 60 + 23 * k, w = 18 + 3 * (k % 4), h = 90 + 17 * k;
    all.push_back(Box{{{{x, y}, {x + w, y + 2}, {x + w - 1, y + h}, {x - 1, y + h - 2}}}});
  }
  classification::PaddleCls cls;
  if (cls.load_model("/no/such/cls.trt")) return 4;
  if (!cls.load_model("synthetic")) return 5;
  cls.allocate_buffers();
  std::vector<Box> ran = all;
  cls.run(img, ran, st);
  const auto scores = cls.last_scores();
  std::vector<Box> gated = all;
  pipeline::classify_angles(cls, img, gated, st);
  auto list = [](const std::vector<Box> &bs) {
    std::string o = "[";
    for (size_t k = 0; k < bs.size(); ++k) o += (k ? "," : "") + jbox(bs[k]);
    return o + "]";
  };
  std::printf("{\"in\":%s,\"out\":%s,\"gated\":%s,\"scores\":[", list(all).c_str(),
              list(ran).c_str(), list(gated).c_str());
  for (size_t k = 0; k < scores.size(); ++k)
    std::printf("%s[%.9g,%.9g]", k ? "," : "", (double)scores[k][0], (double)scores[k][1]);
  std::printf("]}\n");
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  if (argc >= 3 && std::string(argv[1]) == "host") return host_mode(argv[2]);
  if (argc >= 6 && std::string(argv[1]) == "gpu")
    return gpu_mode(argv[2], std::atoi(argv[3]), argv[4], argv[5]);
  if (argc >= 4 && std::string(argv[1]) == "cls") return cls_mode(argv[2], argv[3]);
  if (argc >= 5 && std::string(argv[1]) == "det2")
    return det2_mode(argv[2], std::atoi(argv[3]), argv[4]);
  std::fprintf(stderr, "usage: modules_test host <dict> | gpu <pages> <n> <dict> <outdir> | "
                       "det2 <pages> <n> <outdir>\n");
  return 1;
}
