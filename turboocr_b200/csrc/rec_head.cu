// The recognizer's CTC head fused with the greedy decode, on the tensor cores.
//
// The reference's recognizer ends in a linear layer over every timestep's
// feature vector (the logits [N, T, V] of paddle_rec.cpp:48-90, V = 18385
// for the shipped dictionary) that TensorRT writes to memory; argmax and
// the max softmax probability are then read back per timestep
// (reduce_kernels.cu:15-93, ctc_decode.cpp:25-88). Here the logits never
// leave the SM: one CTA owns 128 timestep rows, streams the [V][K] weight
// matrix through shared memory in chunks of 256 vocabulary rows (TMA,
// 128-byte swizzle, L2-resident across CTAs), computes each 128 x 256
// logit tile with tcgen05.mma (kind::f16, fp32 accumulators in TMEM,
// double-buffered so the MMA of chunk c+1 overlaps the epilogue of chunk c),
// and the epilogue keeps an online (max, first argmax, sum of exp) per row.
// Output per row: the argmax (lowest index on ties) and p = 1 / sum_j
// exp(l_j - l_max), the same definitions as tocr_ctc_greedy_f16 on stored
// logits; then the same collapse kernel makes tokens and line scores.
//
// Roles (18 warps): warp 0 issues the TMA loads (the A tile once, then the
// weight chunks into a 2-stage ring), warp 1 owns TMEM and one lane issues
// the MMAs, warps 2..17 are the epilogue: four warps per TMEM lane quadrant,
// each on one quarter (64 columns) of every chunk; the quarters are combined
// at the end. The epilogue works in the log2 domain, y = l * log2(e): each
// warp stages bias * log2(e) of its next 32 columns in its own slice of
// shared memory (one coalesced load, -inf past the vocabulary, so no column
// test is left in the loop); per logit one multiply-add makes y, a max tree gives
// the group maximum (its first index is only looked for when it beats the
// running maximum), and exp2(y - base) goes into four partial sums, where
// base is 0 while the row's maximum stays within 2^64 of it (no subtraction
// then) and follows the maximum otherwise. Every
// wait is bounded (about a second); a wait that gives up sets the error
// word, every role unwinds and TMEM is released.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "ctc_internal.h"
#include "tc_ptx.cuh"
#include "tocr_common.cuh"

namespace tocr {
namespace {

using namespace ptx;

constexpr int kRows = 128;         // timestep rows per CTA (MMA M, TMEM lanes)
constexpr int kChunk = 256;        // vocabulary rows per chunk (MMA N)
constexpr int kEpiWarp0 = 2;
constexpr int kEpiWarps = 16;      // four per TMEM lane quadrant
constexpr int kParts = kEpiWarps / 4;            // column parts of a chunk
constexpr int kPartCols = kChunk / kParts;       // 64
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kTmemCols = 2 * kChunk;
constexpr float kLog2e = 1.4426950408889634f;

template <int KA>  // K = 64 * KA fp16 features per row
struct Cfg {
  static constexpr int K = 64 * KA;
  static constexpr int STAGES = 2;
  static constexpr int A_BYTES = KA * kRows * 128;
  static constexpr int B_BYTES = KA * kChunk * 128;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = A_BYTES;
  static constexpr int OFF_BAR = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + 16 * 8;
  static constexpr int OFF_COMB = OFF_MISC + 16;
  static constexpr int OFF_BIAS = OFF_COMB + (kParts - 1) * 3 * kRows * 4;
  static constexpr int SMEM = OFF_BIAS + kEpiWarps * 32 * 4 + 1024;  // + alignment slack
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *m, uint64_t *bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

struct HeadParams {
  const float *bias;
  int rows, V, n_chunks;
  int *step_idx;
  float *step_prob;
  int *err;
};

template <int KA>
__global__ void __launch_bounds__(kThreads, 1)
rec_head_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                const HeadParams prm) {
  using C = Cfg<KA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sa = smem + C::OFF_A;
  uint8_t *sb = smem + C::OFF_B;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
  uint64_t *a_full = bars + 0;
  uint64_t *b_full = bars + 1;               // [STAGES]
  uint64_t *b_empty = bars + 1 + C::STAGES;  // [STAGES]
  uint64_t *acc_full = bars + 1 + 2 * C::STAGES;   // [2]
  uint64_t *acc_empty = bars + 3 + 2 * C::STAGES;  // [2]
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + C::OFF_MISC);
  volatile int *s_abort = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 4);
  float *comb = reinterpret_cast<float *>(smem + C::OFF_COMB);  // [kParts-1][3][kRows]
  float *sbias = reinterpret_cast<float *>(smem + C::OFF_BIAS);  // [kEpiWarps][32], bias*log2(e)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRows;
  const int NC = prm.n_chunks;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiThreads / 32);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ---------------------------------------------------------- producer --
    if (lane == 0) {
      tma_prefetch_desc(&amap);
      tma_prefetch_desc(&bmap);
      mbar_arrive_expect_tx(a_full, C::A_BYTES);
      for (int k = 0; k < KA; ++k) tma_load_2d(sa + k * kRows * 128, &amap, a_full, 64 * k, row0);
      for (int c = 0; c < NC; ++c) {
        const int s = c % C::STAGES, u = c / C::STAGES;
        if (u > 0 && !mbar_wait_bounded(&b_empty[s], (u - 1) & 1, s_abort, prm.err, 51)) break;
        mbar_arrive_expect_tx(&b_full[s], C::B_BYTES);
        uint8_t *dst = sb + s * C::B_BYTES;
        for (int k = 0; k < KA; ++k)
          tma_load_2d(dst + k * kChunk * 128, &bmap, &b_full[s], 64 * k, c * kChunk);
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kRows, kChunk);
      bool ok = mbar_wait_bounded(a_full, 0, s_abort, prm.err, 52);
      const uint32_t a_addr = smem_u32(sa);
      for (int c = 0; ok && c < NC; ++c) {
        const int s = c % C::STAGES, u = c / C::STAGES;
        const int b = c & 1, u2 = c >> 1;
        if (!mbar_wait_bounded(&b_full[s], u & 1, s_abort, prm.err, 53)) break;
        if (u2 > 0 && !mbar_wait_bounded(&acc_empty[b], (u2 - 1) & 1, s_abort, prm.err, 54)) break;
        tc_fence_after();
        const uint32_t b_addr = smem_u32(sb + s * C::B_BYTES);
        const uint32_t d = tmem + (uint32_t)(b * kChunk);
#pragma unroll
        for (int k = 0; k < 4 * KA; ++k) {
          const uint32_t off = 32u * (k & 3);  // K = 16 step within the 128-byte row
          const uint64_t ad = sw128_kmajor_desc(a_addr + (k >> 2) * (kRows * 128) + off);
          const uint64_t bd = sw128_kmajor_desc(b_addr + (k >> 2) * (kChunk * 128) + off);
          mma_f16(d, ad, bd, idesc, k > 0 ? 1u : 0u);
        }
        mma_commit(&b_empty[s]);
        mma_commit(&acc_full[b]);
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int ew = warp - kEpiWarp0;     // 0..15
    const int part = ew >> 2;            // column part of every chunk
    const int quad = warp & 3;           // TMEM lane quadrant this warp may read
    const int r = quad * 32 + lane;      // row within the tile
    // running max of y = l*log2(e), its first column, and sum of exp2(y - base)
    float my = -INFINITY, sum = 0.0f, base = 0.0f;
    int idx = 0;
    bool ok = true;
    float *b2 = sbias + ew * 32;          // this warp's staged bias * log2(e)
    for (int c = 0; c < NC; ++c) {
      const int b = c & 1, u2 = c >> 1;
      const int col0 = c * kChunk + part * kPartCols;
      float bl[kPartCols / 32];  // this lane's bias of each group, loaded before the wait
#pragma unroll
      for (int g = 0; g < kPartCols / 32; ++g) {
        const int col = col0 + 32 * g + lane;
        bl[g] = col < prm.V ? __ldg(prm.bias + col) : 0.0f;
      }
      ok = mbar_wait_bounded(&acc_full[b], u2 & 1, s_abort, prm.err, 55);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * kChunk + part * kPartCols);
      uint32_t va[32], vb[32];
      tmem_ld32(taddr, va);
#pragma unroll
      for (int g = 0; g < kPartCols / 32; ++g) {
        uint32_t(&v)[32] = (g & 1) ? vb : va;
        const int cb = col0 + 32 * g;
        __syncwarp();  // the previous group's reads of b2 are done
        b2[lane] = cb + lane < prm.V ? bl[g] * kLog2e : -INFINITY;
        __syncwarp();
        tmem_ld_wait(v);
        if (g + 1 < kPartCols / 32) tmem_ld32(taddr + 32 * (g + 1), (g & 1) ? va : vb);
        if (cb >= prm.V) continue;
        float y[32];
        const float4 *bq = reinterpret_cast<const float4 *>(b2);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          const float4 bb = bq[j4];
          y[4 * j4 + 0] = fmaf(__uint_as_float(v[4 * j4 + 0]), kLog2e, bb.x);
          y[4 * j4 + 1] = fmaf(__uint_as_float(v[4 * j4 + 1]), kLog2e, bb.y);
          y[4 * j4 + 2] = fmaf(__uint_as_float(v[4 * j4 + 2]), kLog2e, bb.z);
          y[4 * j4 + 3] = fmaf(__uint_as_float(v[4 * j4 + 3]), kLog2e, bb.w);
        }
        // group maximum by a tree (depth 5)
        float t16[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) t16[j] = fmaxf(y[j], y[j + 16]);
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int j = 0; j < w; ++j) t16[j] = fmaxf(t16[j], t16[j + w]);
        const float gm = t16[0];
        if (gm > my) {  // a new running maximum: its first column
          uint32_t eq = 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) eq |= (y[j] == gm ? 1u : 0u) << j;
          my = gm;
          idx = cb + __ffs(eq) - 1;
          if (my > base + 64.0f || my < base - 64.0f) {  // keep exp2(y - base) in range
            sum *= ex2_approx(base - my);
            base = my;
          }
        }
        float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (__any_sync(0xffffffffu, base != 0.0f)) {
#pragma unroll
          for (int j = 0; j < 32; ++j) s8[j & 7] += ex2_approx(y[j] - base);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) s8[j & 7] += ex2_approx(y[j]);
        }
        sum += ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    // the row's sum relative to its maximum: sum_j exp2(y_j - my)
    sum = my == -INFINITY ? 0.0f : sum * ex2_approx(base - my);
    // combine the column parts of every row (the lower index wins a tie)
    if (part > 0) {
      float *cp = comb + (size_t)(part - 1) * 3 * kRows;
      cp[r] = my;
      cp[kRows + r] = sum;
      reinterpret_cast<int *>(cp)[2 * kRows + r] = idx;
    }
    const bool all_ok = named_bar_and(1, kEpiThreads, ok);
    if (part == 0 && all_ok) {
      float pm[kParts], ps[kParts];
      int pi[kParts];
      pm[0] = my;
      ps[0] = sum;
      pi[0] = idx;
#pragma unroll
      for (int q = 1; q < kParts; ++q) {
        const float *cp = comb + (size_t)(q - 1) * 3 * kRows;
        pm[q] = cp[r];
        ps[q] = cp[kRows + r];
        pi[q] = reinterpret_cast<const int *>(cp)[2 * kRows + r];
      }
      float M = pm[0];
      int I = pi[0];
#pragma unroll
      for (int q = 1; q < kParts; ++q)
        if (pm[q] > M || (pm[q] == M && pi[q] < I)) {
          M = pm[q];
          I = pi[q];
        }
      float S = 0.f;
#pragma unroll
      for (int q = 0; q < kParts; ++q)
        if (pm[q] != -INFINITY) S += ps[q] * ex2_approx(pm[q] - M);
      const int row = row0 + r;
      if (row < prm.rows) {
        prm.step_idx[row] = M == -INFINITY ? 0 : I;
        prm.step_prob[row] = S > 0.f ? 1.0f / S : 0.f;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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

// fp16 [rows][K] row-major, boxes of 64 x box_rows with the 128-byte swizzle.
int make_map(CUtensorMap *m, const void *base, int K, int rows, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(TOCR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TOCR_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TOCR_OK;
}

template <int KA>
int launch_head(const void *feat, int rows, const void *w, const float *bias, int V,
                int *step_idx, float *step_prob, int *err, cudaStream_t st) {
  using C = Cfg<KA>;
  CUtensorMap am, bm;
  int rc = make_map(&am, feat, C::K, rows, kRows);
  if (rc) return rc;
  rc = make_map(&bm, w, C::K, V, kChunk);
  if (rc) return rc;
  cudaError_t e = cudaFuncSetAttribute(rec_head_kernel<KA>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess)
    return set_error(TOCR_ERR_CUDA, "tocr_rec_head_ctc_f16: %s", cudaGetErrorString(e));
  HeadParams p;
  p.bias = bias;
  p.rows = rows;
  p.V = V;
  p.n_chunks = (V + kChunk - 1) / kChunk;
  p.step_idx = step_idx;
  p.step_prob = step_prob;
  p.err = err;
  const int grid = (rows + kRows - 1) / kRows;
  rec_head_kernel<KA><<<grid, kThreads, C::SMEM, st>>>(am, bm, p);
  return check_launch("rec_head_kernel");
}

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API int tocr_rec_head_ctc_f16(const void *d_feat, int batch_size, int seq_len, int K,
                                   const void *d_w, const float *d_bias, int num_classes,
                                   int num_labels, int *d_tokens, int *d_lengths,
                                   float *d_line_scores, int *d_step_idx, float *d_step_prob,
                                   int *d_err, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(batch_size >= 0 && seq_len > 0 && num_classes > 0 &&
                   (long long)batch_size * seq_len < (1ll << 31),
               "tocr_rec_head_ctc_f16: bad sizes batch=%d seq_len=%d classes=%d", batch_size,
               seq_len, num_classes);
  TOCR_REQUIRE(K == 64 || K == 128, "tocr_rec_head_ctc_f16: K must be 64 or 128 (got %d)", K);
  if (batch_size == 0) return TOCR_OK;
  TOCR_REQUIRE(d_feat && d_w && d_bias && d_tokens && d_lengths && d_line_scores && d_step_idx &&
                   d_step_prob && d_err,
               "tocr_rec_head_ctc_f16: null pointer");
  TOCR_REQUIRE(aligned(d_feat, 16) && aligned(d_w, 16) && aligned(d_bias, 16),
               "tocr_rec_head_ctc_f16: features, weights and bias must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int rows = batch_size * seq_len;
  const int rc = K == 64 ? launch_head<1>(d_feat, rows, d_w, d_bias, num_classes, d_step_idx,
                                          d_step_prob, d_err, st)
                         : launch_head<2>(d_feat, rows, d_w, d_bias, num_classes, d_step_idx,
                                          d_step_prob, d_err, st);
  if (rc != TOCR_OK) return rc;
  return launch_ctc_collapse(d_step_idx, d_step_prob, batch_size, seq_len, num_labels, d_tokens,
                             d_lengths, d_line_scores, nullptr, st);
}

}  // extern "C"
