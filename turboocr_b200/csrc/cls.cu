// Text-line angle classifier network pieces (the reference runs PP-LCNet
// textline orientation in TensorRT, src/classification/paddle_cls.cpp:43-103;
// its weights are not available, so the model here is a synthetic-weight
// network of the same role built from this library's kernels):
//   crops fp16 NCHW [n][3][80][160] (tocr_roi_warp_f16)
//   -> cls_stem_kernel: 3x3 stride-2 conv 3->32 + bias + hardswish, NHWC fp16
//   -> DW+PW blocks (tocr_dwpw_block)
//   -> cls_head_kernel: global average pool + FC C->2 + softmax, fp32 [n][2]
// plus the seeded generator of the synthetic weights (host).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "tocr_common.cuh"

namespace tocr {
namespace {

constexpr int kStemC = 32;       // stem output channels
constexpr int kStemRows = 8;     // output rows per CTA
constexpr int kStemCols = 32;    // output columns per CTA
constexpr int kWinR = 2 * kStemRows + 1, kWinC = 2 * kStemCols + 1;

__device__ __forceinline__ float hardswish(float v) {
  return v * fminf(fmaxf(v + 3.0f, 0.0f), 6.0f) * (1.0f / 6.0f);
}

// One CTA per (crop, 8 x 32 output tile): the 17 x 65 x 3 input window and
// the weights go to shared memory; every thread makes one output pixel's 32
// channels from its 27 taps (sum over taps in weight order) and stores them
// as four 16-byte vectors.
__global__ void __launch_bounds__(kStemRows * kStemCols)
cls_stem_kernel(const __half *__restrict__ x, int H, int W, int Ho, int Wo,
                const float *__restrict__ w, const float *__restrict__ b,
                __half *__restrict__ y) {
  __shared__ float s_x[3][kWinR][kWinC];
  __shared__ float s_w[kStemC * 27];
  __shared__ float s_b[kStemC];
  const int n = blockIdx.z, oy0 = blockIdx.y * kStemRows, ox0 = blockIdx.x * kStemCols;
  const int iy0 = 2 * oy0 - 1, ix0 = 2 * ox0 - 1;
  const __half *xn = x + (long long)n * 3 * H * W;
  for (int i = threadIdx.x; i < 3 * kWinR * kWinC; i += blockDim.x) {
    const int c = i / (kWinR * kWinC), r = (i / kWinC) % kWinR, col = i % kWinC;
    const int iy = iy0 + r, ix = ix0 + col;
    float v = 0.0f;
    if (iy >= 0 && iy < H && ix >= 0 && ix < W) v = __half2float(xn[((long long)c * H + iy) * W + ix]);
    s_x[c][r][col] = v;
  }
  for (int i = threadIdx.x; i < kStemC * 27; i += blockDim.x) s_w[i] = w[i];
  if (threadIdx.x < kStemC) s_b[threadIdx.x] = b[threadIdx.x];
  __syncthreads();
  const int ty = threadIdx.x / kStemCols, tx = threadIdx.x % kStemCols;
  const int oy = oy0 + ty, ox = ox0 + tx;
  if (oy >= Ho || ox >= Wo) return;
  float tap[27];
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) tap[c * 9 + ky * 3 + kx] = s_x[c][2 * ty + ky][2 * tx + kx];
  uint4 out[4];
  __half *o = reinterpret_cast<__half *>(out);
#pragma unroll 4
  for (int co = 0; co < kStemC; ++co) {
    float acc = s_b[co];
#pragma unroll
    for (int t = 0; t < 27; ++t) acc = fmaf(s_w[co * 27 + t], tap[t], acc);
    o[co] = __float2half_rn(hardswish(acc));
  }
  uint4 *dst = reinterpret_cast<uint4 *>(y + (((long long)n * Ho + oy) * Wo + ox) * kStemC);
#pragma unroll
  for (int k = 0; k < 4; ++k) dst[k] = out[k];
}

// One CTA per crop: channel means over the hw pixels (fp16 NHWC, thread =
// channel, consecutive threads read consecutive channels), two logits, and
// their softmax.
__global__ void __launch_bounds__(256)
cls_head_kernel(const __half *__restrict__ x, int hw, int C, const float *__restrict__ w,
                const float *__restrict__ b, float *__restrict__ scores) {
  __shared__ float s_red[2][8];
  const int n = blockIdx.x;
  const __half *xn = x + (long long)n * hw * C;
  float l0 = 0.0f, l1 = 0.0f;
  const float inv = 1.0f / (float)hw;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float s = 0.0f;
    for (int p = 0; p < hw; ++p) s += __half2float(xn[(long long)p * C + c]);
    const float m = s * inv;
    l0 = fmaf(w[c], m, l0);
    l1 = fmaf(w[C + c], m, l1);
  }
  for (int o = 16; o; o >>= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_red[0][warp] = l0;
    s_red[1][warp] = l1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = b[0], c1 = b[1];
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) {
      a += s_red[0][k];
      c1 += s_red[1][k];
    }
    const float m = fmaxf(a, c1);
    const float e0 = expf(a - m), e1 = expf(c1 - m);
    const float s = e0 + e1;
    scores[2 * n] = e0 / s;
    scores[2 * n + 1] = e1 / s;
  }
}

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API int tocr_cls_stem_f16(const void *d_x, int n, int h, int w, const float *d_w,
                               const float *d_b, void *d_y, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && h > 0 && w > 0 && n <= 65535 && h <= (1 << 20) && w <= (1 << 20),
               "tocr_cls_stem_f16: bad sizes n=%d h=%d w=%d", n, h, w);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_x && d_w && d_b && d_y, "tocr_cls_stem_f16: null pointer");
  TOCR_REQUIRE(aligned(d_y, 16), "tocr_cls_stem_f16: output not 16-byte aligned");
  const int Ho = (h - 1) / 2 + 1, Wo = (w - 1) / 2 + 1;
  const dim3 grid((Wo + kStemCols - 1) / kStemCols, (Ho + kStemRows - 1) / kStemRows, n);
  cls_stem_kernel<<<grid, kStemRows * kStemCols, 0, as_stream(stream)>>>(
      static_cast<const __half *>(d_x), h, w, Ho, Wo, d_w, d_b, static_cast<__half *>(d_y));
  return check_launch("tocr_cls_stem_f16");
}

TOCR_API int tocr_cls_head_f32(const void *d_x, int n, int hw, int c, const float *d_w,
                               const float *d_b, float *d_scores, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && hw > 0 && c > 0 && n <= (1 << 30),
               "tocr_cls_head_f32: bad sizes n=%d hw=%d c=%d", n, hw, c);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_x && d_w && d_b && d_scores, "tocr_cls_head_f32: null pointer");
  cls_head_kernel<<<n, 256, 0, as_stream(stream)>>>(static_cast<const __half *>(d_x), hw, c, d_w,
                                                    d_b, d_scores);
  return check_launch("tocr_cls_head_f32");
}

// Synthetic weights: out[i] = scale * (2u - 1), u = the top 24 bits of a
// SplitMix64 finaliser of seed + (i + 1) * 0x9E3779B97F4A7C15, / 2^24.
TOCR_API int tocr_synth_weights(uint64_t seed, float scale, float *out, long long n) {
  TOCR_REQUIRE(n >= 0 && (out || n == 0), "tocr_synth_weights: bad arguments");
  for (long long i = 0; i < n; ++i) {
    uint64_t z = seed + (uint64_t)(i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float u = (float)(z >> 40) * (1.0f / 16777216.0f);
    out[i] = scale * (2.0f * u - 1.0f);
  }
  return TOCR_OK;
}

}  // extern "C"
