// DB bitmap: dst = src > thresh ? 255 : 0 (strict compare), the contract of
// cuda_threshold_to_u8 / cuda_batch_threshold_to_u8
// (src/kernels/reduce_kernels.cu:97-151). The fused DB path never
// materialises this bitmap (its labelling pass thresholds on the fly); this
// entry exists for callers that need the bitmap itself.
#include "tocr_common.cuh"

namespace tocr {
namespace {

__global__ void __launch_bounds__(256)
threshold_u8_kernel(const float *__restrict__ src, uint8_t *__restrict__ dst, long long n,
                    float thresh) {
  const long long n16 = n >> 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const float4 *s = reinterpret_cast<const float4 *>(src) + i * 4;
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 v = __ldcs(s + k);
      w[k] = (v.x > thresh ? 0xffu : 0u) | (v.y > thresh ? 0xff00u : 0u) |
             (v.z > thresh ? 0xff0000u : 0u) | (v.w > thresh ? 0xff000000u : 0u);
    }
    reinterpret_cast<uint4 *>(dst)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  // scalar tail
  const long long t = (n16 << 4) + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (blockIdx.x == 0 && t < n) dst[t] = src[t] > thresh ? 255 : 0;
}

__global__ void threshold_u8_scalar_kernel(const float *__restrict__ src,
                                           uint8_t *__restrict__ dst, long long n,
                                           float thresh) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = src[i] > thresh ? 255 : 0;
}

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" TOCR_API int tocr_threshold_u8(const float *d_src, uint8_t *d_dst, int w, int h,
                                          int batch_size, float thresh, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(w >= 0 && h >= 0 && batch_size >= 0, "tocr_threshold_u8: negative size");
  const long long n = (long long)w * h * batch_size;
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_src && d_dst, "tocr_threshold_u8: null pointer");
  const int sms = sm_count();
  if (aligned(d_src, 16) && aligned(d_dst, 16)) {
    long long need = ((n >> 4) + 255) / 256;
    if (need < 1) need = 1;
    const int grid = (int)(need < (long long)sms * 8 ? need : (long long)sms * 8);
    threshold_u8_kernel<<<grid, 256, 0, as_stream(stream)>>>(d_src, d_dst, n, thresh);
  } else {
    long long need = (n + 255) / 256;
    const int grid = (int)(need < (long long)sms * 8 ? need : (long long)sms * 8);
    threshold_u8_scalar_kernel<<<grid, 256, 0, as_stream(stream)>>>(d_src, d_dst, n, thresh);
  }
  return check_launch("threshold_u8_kernel");
}
