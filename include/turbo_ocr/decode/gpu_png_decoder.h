// Device PNG decode for the reference's image path: what
// turbo_ocr::decode::FastPngDecoder::decode (include/turbo_ocr/decode/
// fast_png_decoder.h:12-15, src/decode/fast_png_decoder.cpp:48-128) followed
// by OcrPipeline::upload_image (src/pipeline/ocr/ocr_pipeline_runtime.cpp:
// 120-147) produce, a BGR GpuImage, made on the device from the compressed
// file. The calls follow NvJpegDecoder's device path
// (include/turbo_ocr/decode/nvjpeg_decoder.h: is_jpeg, get_dimensions,
// decode_to_gpu) so a caller can route PNG bodies the way it routes JPEG
// ones. Header-only over tocr_capi.h; the decoder owns its device scratch and
// pinned staging (grown on demand, reused), one decoder per thread.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <vector>

#include "tocr_capi.h"
#include "turbo_ocr/decode/gpu_image.h"

namespace turbo_ocr::decode {

class GpuPngDecoder {
 public:
  GpuPngDecoder() = default;
  GpuPngDecoder(const GpuPngDecoder &) = delete;
  GpuPngDecoder &operator=(const GpuPngDecoder &) = delete;
  ~GpuPngDecoder() noexcept {
    if (d_buf_) cudaFree(d_buf_);
    if (h_buf_) cudaFreeHost(h_buf_);
  }

  // FastPngDecoder::is_png (fast_png_decoder.h:18-21).
  [[nodiscard]] static bool is_png(const unsigned char *data, std::size_t len) noexcept {
    return len >= 8 && data[0] == 0x89 && data[1] == 'P' && data[2] == 'N' && data[3] == 'G';
  }

  // {width, height}, or {0, 0} when the file is not a PNG, its IHDR is
  // malformed or the reference's caps (MAX_IMAGE_DIM, MAX_IMAGE_PIXELS_MP)
  // reject it.
  [[nodiscard]] std::pair<int, int> get_dimensions(const unsigned char *data,
                                                   std::size_t len) const {
    tocr_png_info info;
    if (tocr_png_peek(data, len, max_dim(), max_pixels(), &info) != TOCR_OK) return {0, 0};
    return {info.width, info.height};
  }

  // Decodes one file into d_output (BGR u8, `pitch` bytes per row, at least
  // w x h as get_dimensions reports). Synchronises `stream` to read the
  // device status; returns true when the pixels match the reference decode,
  // false where the reference returns an empty Mat.
  [[nodiscard]] bool decode_to_gpu(const unsigned char *data, std::size_t len, void *d_output,
                                   std::size_t pitch, int w, int h, cudaStream_t stream = 0) {
    std::vector<GpuImage> out{GpuImage{d_output, pitch, h, w}};
    std::vector<std::pair<const unsigned char *, std::size_t>> in{{data, len}};
    std::vector<int> status;
    return decode_batch_to_gpu(in, out, status, stream) == 1;
  }

  // Decodes a batch: out[i] is the caller's device image for file i (its
  // rows/cols must equal get_dimensions). status[i] receives TOCR_PNG_*
  // (or -1 when the host rejects the file). Returns the number decoded.
  int decode_batch_to_gpu(const std::vector<std::pair<const unsigned char *, std::size_t>> &files,
                          const std::vector<GpuImage> &out, std::vector<int> &status,
                          cudaStream_t stream = 0) {
    const std::size_t n = files.size();
    status.assign(n, -1);
    if (out.size() != n || n == 0) return 0;
    std::vector<tocr_png_job> jobs;
    std::vector<std::size_t> which;
    std::size_t src = 0, scr = 0;
    std::uint8_t *dst_base = nullptr;
    for (std::size_t i = 0; i < n; ++i) {
      tocr_png_info info;
      if (tocr_png_peek(files[i].first, files[i].second, max_dim(), max_pixels(), &info) != TOCR_OK)
        continue;
      if (out[i].data == nullptr || out[i].rows != info.height || out[i].cols != info.width ||
          out[i].step < 3 * static_cast<std::size_t>(info.width))
        continue;
      tocr_png_job j{};
      j.src_off = src;
      j.src_len = files[i].second;
      j.dst_pitch = out[i].step;
      j.scratch_off = scr;
      j.width = info.width;
      j.height = info.height;
      // Outputs are separate buffers: each job addresses its own through
      // dst_off relative to the lowest output pointer of the batch.
      jobs.push_back(j);
      which.push_back(i);
      src += files[i].second;
      scr += (info.scratch_bytes + 15) & ~std::size_t(15);
    }
    if (jobs.empty()) return 0;
    for (std::size_t k = 0; k < jobs.size(); ++k) {
      auto *p = static_cast<std::uint8_t *>(out[which[k]].data);
      if (!dst_base || p < dst_base) dst_base = p;
    }
    for (std::size_t k = 0; k < jobs.size(); ++k)
      jobs[k].dst_off = static_cast<std::uint64_t>(static_cast<std::uint8_t *>(out[which[k]].data) -
                                                   dst_base);
    const std::size_t src_pad = (src + 15) & ~std::size_t(15);
    const std::size_t jobs_bytes = jobs.size() * sizeof(tocr_png_job);
    const std::size_t status_bytes = jobs.size() * sizeof(std::int32_t);
    const std::size_t host_need = src_pad + jobs_bytes + status_bytes;
    const std::size_t dev_need = src_pad + jobs_bytes + ((status_bytes + 15) & ~std::size_t(15)) + scr;
    if (!reserve(host_need, dev_need)) return 0;
    for (std::size_t k = 0; k < jobs.size(); ++k)
      std::memcpy(h_buf_ + jobs[k].src_off, files[which[k]].first, files[which[k]].second);
    std::memcpy(h_buf_ + src_pad, jobs.data(), jobs_bytes);
    std::uint8_t *d_src = d_buf_, *d_jobs = d_buf_ + src_pad;
    std::uint8_t *d_status = d_jobs + jobs_bytes;
    std::uint8_t *d_scratch = d_status + ((status_bytes + 15) & ~std::size_t(15));
    // d_scratch must be 16-byte aligned: src_pad, jobs (48 B each) and the
    // padded status block keep it so.
    if (cudaMemcpyAsync(d_buf_, h_buf_, src_pad + jobs_bytes, cudaMemcpyHostToDevice, stream) !=
        cudaSuccess)
      return 0;
    if (tocr_png_decode_batch(d_src, reinterpret_cast<const tocr_png_job *>(d_jobs),
                              static_cast<int>(jobs.size()), dst_base, d_scratch,
                              reinterpret_cast<std::int32_t *>(d_status), stream) != TOCR_OK)
      return 0;
    auto *h_status = reinterpret_cast<std::int32_t *>(h_buf_ + src_pad + jobs_bytes);
    if (cudaMemcpyAsync(h_status, d_status, status_bytes, cudaMemcpyDeviceToHost, stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return 0;
    int good = 0;
    for (std::size_t k = 0; k < jobs.size(); ++k) {
      status[which[k]] = h_status[k];
      good += h_status[k] == TOCR_PNG_OK;
    }
    return good;
  }

  // image_config.h:13-16 and :31-36 (env::env_int semantics).
  [[nodiscard]] static int max_dim() { return env_int("MAX_IMAGE_DIM", 16384, 64, 65535); }
  [[nodiscard]] static long long max_pixels() {
    return static_cast<long long>(env_int("MAX_IMAGE_PIXELS_MP", 128, 1, 4096)) * 1000000;
  }

 private:
  static int env_int(const char *name, int def, int lo, int hi) {
    const char *v = std::getenv(name);
    if (!v || !*v) return def;
    char *end = nullptr;
    const long x = std::strtol(v, &end, 10);
    if (end == v || *end != '\0') return def;
    return x < lo ? lo : x > hi ? hi : static_cast<int>(x);
  }

  bool reserve(std::size_t host, std::size_t dev) {
    if (host > h_cap_) {
      if (h_buf_) cudaFreeHost(h_buf_);
      h_buf_ = nullptr;
      h_cap_ = 0;
      if (cudaMallocHost(reinterpret_cast<void **>(&h_buf_), host) != cudaSuccess) return false;
      h_cap_ = host;
    }
    if (dev > d_cap_) {
      if (d_buf_) cudaFree(d_buf_);
      d_buf_ = nullptr;
      d_cap_ = 0;
      if (cudaMalloc(reinterpret_cast<void **>(&d_buf_), dev) != cudaSuccess) return false;
      d_cap_ = dev;
    }
    return true;
  }

  std::uint8_t *d_buf_ = nullptr, *h_buf_ = nullptr;
  std::size_t d_cap_ = 0, h_cap_ = 0;
};

}  // namespace turbo_ocr::decode
