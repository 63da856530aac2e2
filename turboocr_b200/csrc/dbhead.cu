// The DB head of the detection network: an FPN neck over three backbone
// levels and the binarisation head (the reference runs PP-OCR's DBFPN +
// DBHead inside TensorRT, include/turbo_ocr/engine/trt/trt_engine.h:37; no
// trained weights exist here, the module draws seeded ones):
//
//   in4 = conv1x1(c4, 256->96)                       level /16
//   out3 = conv1x1(c3, 128->96) + up2(in4)           level /8
//   out2 = conv1x1(c2, 128->96) + up2(out3)          level /4
//   p4, p3, p2 = conv3x3(in4 | out3 | out2, 96->24)  (no bias)
//   fuse = concat(up4(p4), up2(p3), p2)              72 channels at /4
//   h1 = relu(conv3x3(fuse, 72->24) + b1)            BN folded
//   h2 = relu(convT2x2 s2(h1, 24->24) + b2)          level /2, BN folded
//   prob = sigmoid(convT2x2 s2(h2, 24->1) + b3)      level /1, fp32
//
// Every convolution with a channel reduction is an implicit GEMM on the
// tensor cores (conv_tc_kernel): a CTA tile is 8 x 16 output pixels (MMA
// M = 128), its A operand is the input window of one 3x3 tap and one
// 64-channel slice, fetched by a 4-D TMA load straight into the 128-byte
// swizzled K-major layout (the shift of the tap and the zero padding come
// from the TMA coordinates and its out-of-bounds fill), the weights of all
// taps stay in shared memory, tcgen05.mma kind::f16 accumulates in TMEM
// (double-buffered across the persistent CTA's tiles), and the epilogue adds
// the bias and the upsampled coarser level, applies ReLU and stores fp16
// NHWC. The concatenation and the two transposed convolutions are small
// per-pixel kernels on the CUDA cores.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "tc_ptx.cuh"
#include "tocr_common.cuh"

namespace tocr {
namespace dbh {

using namespace ptx;

constexpr int TH = 8, TW = 16, TP = 128;  // output tile (MMA M)
constexpr int kStages = 4;                 // A ring
constexpr int kThreads = 192;              // producer, MMA, 4 epilogue warps

template <int TAPS, int KA, int NOUT, int COUT, bool RELU, bool ADD_UP>
struct Cfg {
  static constexpr int A_BYTES = TP * 128;                  // one tap x 64 channels
  static constexpr int B_BLOCK = NOUT * 128;                // one tap x 64 channels of weights
  static constexpr int B_BYTES = TAPS * KA * B_BLOCK;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + kStages * A_BYTES;
  static constexpr int OFF_BAR = OFF_B + B_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + 16 * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = 2 * NOUT <= 32 ? 32 : (2 * NOUT <= 64 ? 64 : (2 * NOUT <= 128 ? 128 : 256));
  static constexpr int STEPS = TAPS * KA;              // A boxes per tile
  static_assert(NOUT % 32 == 0 && COUT <= NOUT && COUT % 8 == 0, "output channels");
  static_assert(B_BYTES % 16 == 0 && OFF_B % 1024 == 0, "operand alignment");
  static_assert(SMEM <= 232448, "shared memory");
};

struct ConvParams {
  const uint8_t *wblob;   // packed weights (B image)
  const float *bias;      // [COUT] or null
  const __half *up;       // coarser level [N][H/2][W/2][COUT] or null
  __half *y;              // [N][H][W][COUT]
  int N, H, W, tiles_x, tiles_y, ntiles;
  int *err;
};

template <class K, int TAPS, int KA, int NOUT, int COUT, bool RELU, bool ADD_UP>
__global__ void __launch_bounds__(kThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap xmap, const ConvParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sa = smem + K::OFF_A;
  uint8_t *sb = smem + K::OFF_B;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + K::OFF_BAR);
  uint64_t *a_full = bars;                 // [kStages]
  uint64_t *a_empty = bars + kStages;      // [kStages]
  uint64_t *acc_full = bars + 2 * kStages; // [2]
  uint64_t *acc_empty = bars + 2 * kStages + 2;
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + K::OFF_MISC);
  volatile int *s_abort = reinterpret_cast<volatile int *>(smem + K::OFF_MISC + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // weights of every tap into shared memory (already in the swizzled image)
  for (int i = threadIdx.x; i < K::B_BYTES / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(sb)[i] = __ldg(reinterpret_cast<const uint4 *>(prm.wblob) + i);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, K::TMEM_COLS);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int tiles_per_img = prm.tiles_x * prm.tiles_y;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------- TMA producer
      tma_prefetch_desc(&xmap);
      uint32_t l = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < prm.ntiles; t += gridDim.x) {
        const int n = t / tiles_per_img, r = t % tiles_per_img;
        const int y0 = (r / prm.tiles_x) * TH, x0 = (r % prm.tiles_x) * TW;
        for (int st = 0; st < K::STEPS; ++st, ++l) {
          const int s = l % kStages, u = l / kStages;
          if (u > 0 && !mbar_wait_bounded(&a_empty[s], (u - 1) & 1, s_abort, prm.err, 61)) {
            ok = false;
            break;
          }
          const int tap = st / KA, a = st % KA;
          const int dy = TAPS == 9 ? tap / 3 - 1 : 0, dx = TAPS == 9 ? tap % 3 - 1 : 0;
          mbar_arrive_expect_tx(&a_full[s], K::A_BYTES);
          tma_load_4d(sa + s * K::A_BYTES, &xmap, &a_full[s], 64 * a, x0 + dx, y0 + dy, n);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ------------------------------------------- MMA
      constexpr uint32_t idesc = idesc_f16(TP, NOUT);
      uint32_t l = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < prm.ntiles; t += gridDim.x, ++i) {
        const int b = i & 1, u2 = i >> 1;
        if (u2 > 0 && !mbar_wait_bounded(&acc_empty[b], (u2 - 1) & 1, s_abort, prm.err, 62)) break;
        const uint32_t d = tmem + (uint32_t)(b * NOUT);
        for (int st = 0; st < K::STEPS; ++st, ++l) {
          const int s = l % kStages, u = l / kStages;
          if (!mbar_wait_bounded(&a_full[s], u & 1, s_abort, prm.err, 63)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sa + s * K::A_BYTES);
          const uint32_t b_addr = smem_u32(sb + st * K::B_BLOCK);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16(d, sw128_kmajor_desc(a_addr + 32 * k), sw128_kmajor_desc(b_addr + 32 * k),
                    idesc, (st > 0 || k > 0) ? 1u : 0u);
          mma_commit(&a_empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int p = quad * 32 + lane;  // pixel of the tile = TMEM lane
    uint32_t i = 0;
    for (int t = blockIdx.x; t < prm.ntiles; t += gridDim.x, ++i) {
      const int b = i & 1, u2 = i >> 1;
      if (!mbar_wait_bounded(&acc_full[b], u2 & 1, s_abort, prm.err, 64)) break;
      tc_fence_after();
      const int n = t / tiles_per_img, r = t % tiles_per_img;
      const int y = (r / prm.tiles_x) * TH + p / TW, x = (r % prm.tiles_x) * TW + p % TW;
      const bool valid = y < prm.H && x < prm.W;
      const long long pix = ((long long)n * prm.H + y) * prm.W + x;
      const __half *upp = nullptr;
      if (ADD_UP && valid)
        upp = prm.up + (((long long)n * (prm.H >> 1) + (y >> 1)) * (prm.W >> 1) + (x >> 1)) * COUT;
#pragma unroll
      for (int c0 = 0; c0 < COUT; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * NOUT + c0), v);
        tmem_ld_wait(v);
        if (!valid) continue;
        const int cn = COUT - c0 < 32 ? COUT - c0 : 32;
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          f[j] = __uint_as_float(v[j]);
          if (prm.bias && j < cn) f[j] += __ldg(prm.bias + c0 + j);
        }
        if (ADD_UP) {
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8) {
            if (8 * j8 >= cn) break;
            const uint4 u = *reinterpret_cast<const uint4 *>(upp + c0 + 8 * j8);
            const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 g = __half22float2(h[q]);
              f[8 * j8 + 2 * q] += g.x;
              f[8 * j8 + 2 * q + 1] += g.y;
            }
          }
        }
        __half *dst = prm.y + pix * COUT + c0;
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          if (8 * j8 >= cn) break;
          uint32_t w4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float a0 = f[8 * j8 + 2 * q], a1 = f[8 * j8 + 2 * q + 1];
            if (RELU) {
              a0 = fmaxf(a0, 0.f);
              a1 = fmaxf(a1, 0.f);
            }
            const __half2 h = __floats2half2_rn(a0, a1);
            w4[q] = *reinterpret_cast<const uint32_t *>(&h);
          }
          *reinterpret_cast<uint4 *>(dst + 8 * j8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, K::TMEM_COLS);
  }
}

// fuse [N][H][W][72] = (p4 at (y/4, x/4), p3 at (y/2, x/2), p2 at (y, x)), 24 channels each
__global__ void __launch_bounds__(256)
concat_kernel(const __half *__restrict__ p4, const __half *__restrict__ p3,
              const __half *__restrict__ p2, int N, int H, int W, __half *__restrict__ fuse) {
  const long long total = (long long)N * H * W * 9;  // 9 vectors of 8 channels per pixel
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int v = (int)(i % 9);
    const long long pix = i / 9;
    const int x = (int)(pix % W), y = (int)((pix / W) % H), n = (int)(pix / ((long long)W * H));
    const __half *src;
    if (v < 3)
      src = p4 + (((long long)n * (H >> 2) + (y >> 2)) * (W >> 2) + (x >> 2)) * 24 + 8 * v;
    else if (v < 6)
      src = p3 + (((long long)n * (H >> 1) + (y >> 1)) * (W >> 1) + (x >> 1)) * 24 + 8 * (v - 3);
    else
      src = p2 + pix * 24 + 8 * (v - 6);
    reinterpret_cast<uint4 *>(fuse + pix * 72)[v] = *reinterpret_cast<const uint4 *>(src);
  }
}

// The two transposed convolutions and the sigmoid: one thread per two /4
// pixels of h1 (24 channels each; every weight read from shared memory feeds
// both) writes their 4 x 4 blocks of the /1 probability map.
// w2 [24 in][24 out][2][2], w3 [24 in][2][2] (PyTorch ConvTranspose2d order).
constexpr int kUpPix = 2;
__global__ void __launch_bounds__(256)
head_up_kernel(const __half *__restrict__ h1, int N, int H, int W, const float *__restrict__ w2,
               const float *__restrict__ b2, const float *__restrict__ w3, float b3,
               float *__restrict__ prob) {
  __shared__ float s_w2[24 * 24 * 4];
  __shared__ float s_b2[24];
  __shared__ float s_w3[24 * 4];
  for (int i = threadIdx.x; i < 24 * 24 * 4; i += blockDim.x) s_w2[i] = w2[i];
  if (threadIdx.x < 24) s_b2[threadIdx.x] = b2[threadIdx.x];
  if (threadIdx.x < 96) s_w3[threadIdx.x] = w3[threadIdx.x];
  __syncthreads();
  const int Wg = (W + kUpPix - 1) / kUpPix;
  const long long total = (long long)N * H * Wg;
  const int Wo = 4 * W;
  for (long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x; gi < total;
       gi += (long long)gridDim.x * blockDim.x) {
    const int xg = (int)(gi % Wg), y = (int)((gi / Wg) % H), n = (int)(gi / ((long long)Wg * H));
    const int x0 = xg * kUpPix;
    const int np = min(kUpPix, W - x0);
    float in[kUpPix][24];
#pragma unroll
    for (int q = 0; q < kUpPix; ++q) {
      const long long pix = ((long long)n * H + y) * W + min(x0 + q, W - 1);
      const uint4 *src = reinterpret_cast<const uint4 *>(h1 + pix * 24);
#pragma unroll
      for (int v = 0; v < 3; ++v) {
        const uint4 u = src[v];
        const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 g = __half22float2(h[e]);
          in[q][8 * v + 2 * e] = g.x;
          in[q][8 * v + 2 * e + 1] = g.y;
        }
      }
    }
    float out[kUpPix][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float acc[kUpPix][4];
#pragma unroll
        for (int q = 0; q < kUpPix; ++q)
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[q][k] = b3;
        for (int c = 0; c < 24; ++c) {
          float hq[kUpPix];
#pragma unroll
          for (int q = 0; q < kUpPix; ++q) hq[q] = s_b2[c];
#pragma unroll
          for (int ci = 0; ci < 24; ++ci) {
            const float wv = s_w2[((ci * 24 + c) * 2 + i) * 2 + j];
#pragma unroll
            for (int q = 0; q < kUpPix; ++q) hq[q] = fmaf(in[q][ci], wv, hq[q]);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float w3v = s_w3[c * 4 + k];
#pragma unroll
            for (int q = 0; q < kUpPix; ++q) acc[q][k] = fmaf(fmaxf(hq[q], 0.f), w3v, acc[q][k]);
          }
        }
#pragma unroll
        for (int q = 0; q < kUpPix; ++q)
#pragma unroll
          for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int l = 0; l < 2; ++l)
              out[q][2 * i + k][2 * j + l] = 1.f / (1.f + expf(-acc[q][2 * k + l]));
      }
#pragma unroll
    for (int q = 0; q < kUpPix; ++q) {
      if (q >= np) break;
      float *o = prob + ((long long)n * 4 * H + 4 * y) * Wo + 4 * (x0 + q);
#pragma unroll
      for (int r = 0; r < 4; ++r)
        *reinterpret_cast<float4 *>(o + (long long)r * Wo) =
            make_float4(out[q][r][0], out[q][r][1], out[q][r][2], out[q][r][3]);
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// x fp16 NHWC [N][H][W][C] as a 4-D map with boxes of 64 channels x 16 x 8 x 1,
// 128-byte swizzle (the K-major MMA layout), zero fill out of bounds.
int make_xmap(CUtensorMap *m, const void *x, int N, int H, int W, int C) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(TOCR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N};
  const cuuint64_t strides[3] = {(cuuint64_t)C * 2, (cuuint64_t)C * W * 2, (cuuint64_t)C * W * H * 2};
  const cuuint32_t box[4] = {64, TW, TH, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(x), dims, strides, box,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TOCR_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TOCR_OK;
}

template <int TAPS, int KA, int NOUT, int COUT, bool RELU, bool ADD_UP>
int launch_conv(const void *x, int N, int H, int W, int C, const void *wblob, const float *bias,
                const void *up, void *y, int *err, cudaStream_t st) {
  using K = Cfg<TAPS, KA, NOUT, COUT, RELU, ADD_UP>;
  auto kern = conv_tc_kernel<K, TAPS, KA, NOUT, COUT, RELU, ADD_UP>;
  CUtensorMap xm;
  int rc = make_xmap(&xm, x, N, H, W, C);
  if (rc) return rc;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM);
  if (e != cudaSuccess) return set_error(TOCR_ERR_CUDA, "conv_tc smem: %s", cudaGetErrorString(e));
  ConvParams p;
  p.wblob = static_cast<const uint8_t *>(wblob);
  p.bias = bias;
  p.up = static_cast<const __half *>(up);
  p.y = static_cast<__half *>(y);
  p.N = N;
  p.H = H;
  p.W = W;
  p.tiles_x = (W + TW - 1) / TW;
  p.tiles_y = (H + TH - 1) / TH;
  p.ntiles = N * p.tiles_x * p.tiles_y;
  p.err = err;
  if (p.ntiles == 0) return TOCR_OK;
  const int grid = p.ntiles < sm_count() ? p.ntiles : sm_count();
  kern<<<grid, kThreads, K::SMEM, st>>>(xm, p);
  return check_launch("conv_tc_kernel");
}

// Host: weights [Cout][Cin][k][k] (fp32, PyTorch Conv2d order) into the B
// image of conv_tc_kernel: per (tap, 64-channel slice) a block of NOUT rows
// of 128 bytes (K-major, 128-byte swizzle), rows >= Cout and channels >= Cin zero.
void pack_weights(const float *w, int cout, int cin, int taps, int nout, uint8_t *out) {
  const int ka = (cin + 63) / 64;
  const size_t block = (size_t)nout * 128;
  std::memset(out, 0, (size_t)taps * ka * block);
  for (int t = 0; t < taps; ++t)
    for (int a = 0; a < ka; ++a) {
      uint8_t *blk = out + (size_t)(t * ka + a) * block;
      for (int o = 0; o < cout; ++o)
        for (int k = 0; k < 64; ++k) {
          const int c = 64 * a + k;
          if (c >= cin) break;
          const float v = w[((size_t)o * cin + c) * taps + t];
          const __half h = __float2half_rn(v);
          const int chunk = k / 8, e = k % 8;
          const size_t off = (size_t)(o / 8) * 1024 + (o % 8) * 128 + ((chunk ^ (o % 8)) * 16) + 2 * e;
          std::memcpy(blk + off, &h, 2);
        }
    }
}

size_t packed_bytes(int cin, int taps, int nout) { return (size_t)taps * ((cin + 63) / 64) * nout * 128; }

int nout_for(int cout) { return cout <= 32 ? 32 : 96; }

}  // namespace dbh
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API size_t tocr_conv_tc_packed_bytes(int cin, int cout, int ksize) {
  if (cin <= 0 || cout <= 0 || (ksize != 1 && ksize != 3)) return 0;
  return dbh::packed_bytes(cin, ksize * ksize, dbh::nout_for(cout));
}

TOCR_API int tocr_conv_tc_pack(int cin, int cout, int ksize, const float *w, void *out,
                               size_t out_bytes) {
  TOCR_REQUIRE(cin > 0 && cout > 0 && (ksize == 1 || ksize == 3) && w && out,
               "tocr_conv_tc_pack: bad arguments");
  TOCR_REQUIRE(out_bytes >= tocr_conv_tc_packed_bytes(cin, cout, ksize),
               "tocr_conv_tc_pack: output too small");
  dbh::pack_weights(w, cout, cin, ksize * ksize, dbh::nout_for(cout), static_cast<uint8_t *>(out));
  return TOCR_OK;
}

TOCR_API int tocr_conv_tc_f16(const void *d_x, int n, int h, int w, int cin, int cout, int ksize,
                              const void *d_packed, const float *d_bias, int relu,
                              const void *d_up, void *d_y, int *d_err, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && h > 0 && w > 0 && n <= 65535 && (long long)n * h * w < (1ll << 31),
               "tocr_conv_tc_f16: bad sizes n=%d h=%d w=%d", n, h, w);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_x && d_packed && d_y && d_err, "tocr_conv_tc_f16: null pointer");
  TOCR_REQUIRE(aligned(d_x, 16) && aligned(d_y, 16) && aligned(d_packed, 16) &&
                   (!d_up || aligned(d_up, 16)),
               "tocr_conv_tc_f16: buffers must be 16-byte aligned");
  TOCR_REQUIRE(!d_up || (h % 2 == 0 && w % 2 == 0), "tocr_conv_tc_f16: the upsampled add needs even sizes");
  cudaStream_t st = as_stream(stream);
  if (ksize == 1 && cin == 256 && cout == 96 && !relu && !d_up)
    return dbh::launch_conv<1, 4, 96, 96, false, false>(d_x, n, h, w, cin, d_packed, d_bias, d_up, d_y, d_err, st);
  if (ksize == 1 && cin == 128 && cout == 96 && !relu && !d_up)
    return dbh::launch_conv<1, 2, 96, 96, false, false>(d_x, n, h, w, cin, d_packed, d_bias, d_up, d_y, d_err, st);
  if (ksize == 1 && cin == 128 && cout == 96 && !relu && d_up)
    return dbh::launch_conv<1, 2, 96, 96, false, true>(d_x, n, h, w, cin, d_packed, d_bias, d_up, d_y, d_err, st);
  if (ksize == 3 && cin == 96 && cout == 24 && !relu && !d_up)
    return dbh::launch_conv<9, 2, 32, 24, false, false>(d_x, n, h, w, cin, d_packed, d_bias, d_up, d_y, d_err, st);
  if (ksize == 3 && cin == 72 && cout == 24 && relu && !d_up)
    return dbh::launch_conv<9, 2, 32, 24, true, false>(d_x, n, h, w, cin, d_packed, d_bias, d_up, d_y, d_err, st);
  return set_error(TOCR_ERR_INVALID,
                   "tocr_conv_tc_f16: unsupported shape k=%d cin=%d cout=%d relu=%d up=%d", ksize,
                   cin, cout, relu, d_up != nullptr);
}

TOCR_API int tocr_fpn_concat_f16(const void *d_p4, const void *d_p3, const void *d_p2, int n, int h,
                                 int w, void *d_fuse, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && h > 0 && w > 0 && h % 4 == 0 && w % 4 == 0,
               "tocr_fpn_concat_f16: bad sizes n=%d h=%d w=%d (multiples of 4)", n, h, w);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_p4 && d_p3 && d_p2 && d_fuse, "tocr_fpn_concat_f16: null pointer");
  TOCR_REQUIRE(aligned(d_p4, 16) && aligned(d_p3, 16) && aligned(d_p2, 16) && aligned(d_fuse, 16),
               "tocr_fpn_concat_f16: buffers must be 16-byte aligned");
  const long long total = (long long)n * h * w * 9;
  const unsigned grid = (unsigned)std::min<long long>((total + 255) / 256, (long long)sm_count() * 16);
  dbh::concat_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      static_cast<const __half *>(d_p4), static_cast<const __half *>(d_p3),
      static_cast<const __half *>(d_p2), n, h, w, static_cast<__half *>(d_fuse));
  return check_launch("tocr_fpn_concat_f16");
}

TOCR_API int tocr_db_head_up_f32(const void *d_h1, int n, int h, int w, const float *d_w2,
                                 const float *d_b2, const float *d_w3, float b3, float *d_prob,
                                 void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n >= 0 && h > 0 && w > 0, "tocr_db_head_up_f32: bad sizes n=%d h=%d w=%d", n, h, w);
  if (n == 0) return TOCR_OK;
  TOCR_REQUIRE(d_h1 && d_w2 && d_b2 && d_w3 && d_prob, "tocr_db_head_up_f32: null pointer");
  TOCR_REQUIRE(aligned(d_h1, 16) && aligned(d_prob, 16), "tocr_db_head_up_f32: alignment");
  const long long total = (long long)n * h * ((w + dbh::kUpPix - 1) / dbh::kUpPix);
  const unsigned grid = (unsigned)std::min<long long>((total + 255) / 256, (long long)sm_count() * 16);
  dbh::head_up_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const __half *>(d_h1), n, h,
                                                           w, d_w2, d_b2, d_w3, b3, d_prob);
  return check_launch("tocr_db_head_up_f32");
}

}  // extern "C"
