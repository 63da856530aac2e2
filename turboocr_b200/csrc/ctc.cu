// Subsystem 4 — CTC greedy decode on B200.
//
// Reference behaviour (TurboOCR):
//   argmax per timestep, lowest index on ties ....... src/kernels/reduce_kernels.cu:15-83
//   collapse: emit idx if idx != last && idx != 0 && idx < |labels|,
//             score = sequential fp32 mean of emitted maxima ... src/recognition/ctc_decode.cpp:25-92
//
// B200 design: the logits tensor is read exactly once from HBM. One warp owns
// one (line, timestep) row; lanes stream 16-byte chunks of the row with
// L1-bypassing vector loads (four chunks in flight per lane) and keep an
// online (max, argmax, sum exp(x - max)) triple, so the argmax and the max
// softmax probability come out of the same pass. Rows are 2-byte aligned
// only (num_classes is odd for the PP-OCR dictionaries), so each row is split
// into a scalar head up to the first 16-byte boundary, an aligned body and a
// scalar tail. A second, tiny launch collapses each line with one warp.
#include "ctc_internal.h"
#include "tocr_common.cuh"

#include <cmath>

namespace tocr {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kRowsThreads = 256;  // 8 warps per CTA, one row per warp at a time

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Streaming 16-byte load: read-only, no L1 allocation, 256-byte L2 prefetch.
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Running state of one lane over the elements it has seen, in increasing
// index order: maximum m, its (lowest) index mi, and s = sum exp(x - m).
struct SoftAcc {
  float m;
  int mi;
  float s;
};

__device__ __forceinline__ void soft_scalar(SoftAcc &a, float x, int idx) {
  if (x > a.m) {
    a.s = (a.m == -INFINITY) ? 0.f : a.s * ex2_approx((a.m - x) * kLog2e);
    a.m = x;
    a.mi = idx;
  }
  if (a.m != -INFINITY) a.s += ex2_approx(x * kLog2e - a.m * kLog2e);
}

__device__ __forceinline__ __half2 as_h2(uint32_t u) {
  return *reinterpret_cast<__half2 *>(&u);
}

// Eight consecutive fp16 logits starting at element `base`.
__device__ __forceinline__ void soft_chunk8(SoftAcc &a, uint4 v, int base) {
  const __half2 h0 = as_h2(v.x), h1 = as_h2(v.y), h2 = as_h2(v.z), h3 = as_h2(v.w);
  const __half2 mx = __hmax2(__hmax2(h0, h1), __hmax2(h2, h3));
  const float cm = fmaxf(__low2float(mx), __high2float(mx));
  const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
  const float2 f2 = __half22float2(h2), f3 = __half22float2(h3);
  if (cm > a.m) {  // strictly greater: an equal later value never wins
    int j = 7;
    if (f3.x == cm) j = 6;
    if (f2.y == cm) j = 5;
    if (f2.x == cm) j = 4;
    if (f1.y == cm) j = 3;
    if (f1.x == cm) j = 2;
    if (f0.y == cm) j = 1;
    if (f0.x == cm) j = 0;
    a.s = (a.m == -INFINITY) ? 0.f : a.s * ex2_approx((a.m - cm) * kLog2e);
    a.m = cm;
    a.mi = base + j;
  }
  if (a.m != -INFINITY) {
    const float mb = a.m * kLog2e;
    float t0 = ex2_approx(fmaf(f0.x, kLog2e, -mb)) + ex2_approx(fmaf(f0.y, kLog2e, -mb));
    float t1 = ex2_approx(fmaf(f1.x, kLog2e, -mb)) + ex2_approx(fmaf(f1.y, kLog2e, -mb));
    float t2 = ex2_approx(fmaf(f2.x, kLog2e, -mb)) + ex2_approx(fmaf(f2.y, kLog2e, -mb));
    float t3 = ex2_approx(fmaf(f3.x, kLog2e, -mb)) + ex2_approx(fmaf(f3.y, kLog2e, -mb));
    a.s += (t0 + t1) + (t2 + t3);
  }
}

// Merge two lane states; ties on the maximum keep the lower index.
__device__ __forceinline__ void soft_merge(SoftAcc &a, float om, int omi, float os) {
  const float M = fmaxf(a.m, om);
  const float sa = (a.m == -INFINITY) ? 0.f : a.s * ex2_approx((a.m - M) * kLog2e);
  const float sb = (om == -INFINITY) ? 0.f : os * ex2_approx((om - M) * kLog2e);
  if (om > a.m || (om == a.m && omi < a.mi)) a.mi = omi;
  a.m = M;
  a.s = sa + sb;
}

__global__ void __launch_bounds__(kRowsThreads)
ctc_rows_f16_kernel(const __half *__restrict__ logits, long long rows, int V,
                    int *__restrict__ step_idx, float *__restrict__ step_prob,
                    const int *__restrict__ d_batch = nullptr, int T = 0) {
  const int lane = threadIdx.x & 31;
  if (d_batch) rows = min(rows, (long long)(*d_batch) * T);
  const long long warps_total = (long long)gridDim.x * (kRowsThreads / 32);
  for (long long r = (long long)blockIdx.x * (kRowsThreads / 32) + (threadIdx.x >> 5);
       r < rows; r += warps_total) {
    const __half *row = logits + r * (long long)V;
    int head = (int)(((16u - (unsigned)(reinterpret_cast<uintptr_t>(row) & 15u)) & 15u) >> 1);
    if (head > V) head = V;
    const int nchunks = (V - head) >> 3;
    const int tail0 = head + (nchunks << 3);

    SoftAcc a{-INFINITY, INT_MAX, 0.f};
    if (lane < head) soft_scalar(a, __half2float(row[lane]), lane);

    const uint4 *body = reinterpret_cast<const uint4 *>(row + head);
    int c = lane;
    for (; c + 96 < nchunks; c += 128) {
      const uint4 v0 = ld_stream16(body + c);
      const uint4 v1 = ld_stream16(body + c + 32);
      const uint4 v2 = ld_stream16(body + c + 64);
      const uint4 v3 = ld_stream16(body + c + 96);
      soft_chunk8(a, v0, head + (c << 3));
      soft_chunk8(a, v1, head + ((c + 32) << 3));
      soft_chunk8(a, v2, head + ((c + 64) << 3));
      soft_chunk8(a, v3, head + ((c + 96) << 3));
    }
    for (; c < nchunks; c += 32) soft_chunk8(a, ld_stream16(body + c), head + (c << 3));

    if (tail0 + lane < V) soft_scalar(a, __half2float(row[tail0 + lane]), tail0 + lane);

#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, a.m, off);
      const int omi = __shfl_xor_sync(0xffffffffu, a.mi, off);
      const float os = __shfl_xor_sync(0xffffffffu, a.s, off);
      soft_merge(a, om, omi, os);
    }
    if (lane == 0) {
      step_idx[r] = (a.mi == INT_MAX) ? 0 : a.mi;
      step_prob[r] = (a.s > 0.f) ? __frcp_rn(a.s) : 0.f;
    }
  }
}

// fp32 variant for the reference cuda_argmax contract: max VALUE (not a
// softmax) and its lowest index.
__global__ void __launch_bounds__(kRowsThreads)
argmax_rows_f32_kernel(const float *__restrict__ probs, long long rows, int V,
                       int *__restrict__ out_idx, float *__restrict__ out_val) {
  const int lane = threadIdx.x & 31;
  const long long warps_total = (long long)gridDim.x * (kRowsThreads / 32);
  for (long long r = (long long)blockIdx.x * (kRowsThreads / 32) + (threadIdx.x >> 5);
       r < rows; r += warps_total) {
    const float *row = probs + r * (long long)V;
    int head = (int)(((16u - (unsigned)(reinterpret_cast<uintptr_t>(row) & 15u)) & 15u) >> 2);
    if (head > V) head = V;
    const int nchunks = (V - head) >> 2;
    const int tail0 = head + (nchunks << 2);
    float m = -INFINITY;
    int mi = INT_MAX;
    auto take = [&](float x, int i) {
      if (x > m) { m = x; mi = i; }
    };
    if (lane < head) take(row[lane], lane);
    const uint4 *body = reinterpret_cast<const uint4 *>(row + head);
    int c = lane;
    for (; c + 96 < nchunks; c += 128) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = ld_stream16(body + c + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int b = head + ((c + 32 * u) << 2);
        take(__uint_as_float(v[u].x), b);
        take(__uint_as_float(v[u].y), b + 1);
        take(__uint_as_float(v[u].z), b + 2);
        take(__uint_as_float(v[u].w), b + 3);
      }
    }
    for (; c < nchunks; c += 32) {
      const uint4 v = ld_stream16(body + c);
      const int b = head + (c << 2);
      take(__uint_as_float(v.x), b);
      take(__uint_as_float(v.y), b + 1);
      take(__uint_as_float(v.z), b + 2);
      take(__uint_as_float(v.w), b + 3);
    }
    if (tail0 + lane < V) take(row[tail0 + lane], tail0 + lane);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, off);
      const int omi = __shfl_xor_sync(0xffffffffu, mi, off);
      if (om > m || (om == m && omi < mi)) { m = om; mi = omi; }
    }
    if (lane == 0) {
      // A row with no value above -FLT_MAX keeps index 0, like the reference
      // loop whose initial best is (-FLT_MAX, 0).
      if (mi == INT_MAX || !(m > -3.402823466e38f)) { mi = 0; m = -3.402823466e38f; }
      out_idx[r] = mi;
      out_val[r] = m;
    }
  }
}

constexpr int kCollapseWarps = 4;

// One warp per line: the greedy collapse of ctc_decode.cpp:25-48, with the
// score summed sequentially in timestep order (same fp32 rounding order).
__global__ void __launch_bounds__(kCollapseWarps * 32)
ctc_collapse_kernel(const int *__restrict__ step_idx, const float *__restrict__ step_prob,
                    int batch, int T, int num_labels, int *__restrict__ tokens,
                    int *__restrict__ lengths, float *__restrict__ scores,
                    const int *__restrict__ d_batch = nullptr) {
  __shared__ float s_prob[kCollapseWarps][32];
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int line = blockIdx.x * kCollapseWarps + w;
  if (d_batch) batch = min(batch, *d_batch);
  if (line >= batch) return;
  const long long base = (long long)line * T;
  int carry = -1;  // last_index before the first step
  int count = 0;
  float sum = 0.f;
  for (int t0 = 0; t0 < T; t0 += 32) {
    const int t = t0 + lane;
    const bool valid = t < T;
    const int idx = valid ? step_idx[base + t] : -2;
    const float p = valid ? step_prob[base + t] : 0.f;
    int prev = __shfl_up_sync(0xffffffffu, idx, 1);
    if (lane == 0) prev = carry;
    const bool emit = valid && idx != prev && idx != 0 && idx < num_labels;
    const unsigned mask = __ballot_sync(0xffffffffu, emit);
    const int pos = count + __popc(mask & ((1u << lane) - 1u));
    if (emit) {
      tokens[base + pos] = idx;
      s_prob[w][lane] = p;
    }
    __syncwarp();
    if (lane == 0) {
      unsigned m = mask;
      while (m) {
        const int l = __ffs(m) - 1;
        sum = __fadd_rn(sum, s_prob[w][l]);
        m &= m - 1u;
      }
    }
    __syncwarp();
    count += __popc(mask);
    carry = __shfl_sync(0xffffffffu, idx, 31);
  }
  if (lane == 0) {
    lengths[line] = count;
    scores[line] = count > 0 ? __fdiv_rn(sum, (float)count) : 0.f;
  }
}

// Enough CTAs to fill every SM at the kernel's occupancy; warps then
// grid-stride over rows.
template <typename K>
int rows_grid(K kernel, long long rows) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kRowsThreads, 0) !=
          cudaSuccess || per_sm <= 0)
    per_sm = 4;
  const long long need = (rows + (kRowsThreads / 32) - 1) / (kRowsThreads / 32);
  const long long cap = (long long)sm_count() * per_sm;
  return (int)(need < cap ? need : cap);
}

}  // namespace

int launch_ctc_collapse(const int *step_idx, const float *step_prob, int batch, int T,
                        int num_labels, int *tokens, int *lengths, float *scores,
                        const int *d_batch, cudaStream_t stream) {
  if (batch <= 0) return TOCR_OK;
  const int blocks = (batch + kCollapseWarps - 1) / kCollapseWarps;
  ctc_collapse_kernel<<<blocks, kCollapseWarps * 32, 0, stream>>>(
      step_idx, step_prob, batch, T, num_labels, tokens, lengths, scores, d_batch);
  return check_launch("ctc_collapse_kernel");
}

}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API int tocr_argmax_f32(const float *d_probs, int *d_indices, float *d_scores,
                             int batch_size, int seq_len, int num_classes, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(batch_size >= 0 && seq_len >= 0 && num_classes > 0,
               "tocr_argmax_f32: bad sizes batch=%d seq_len=%d classes=%d", batch_size,
               seq_len, num_classes);
  const long long rows = (long long)batch_size * seq_len;
  if (rows == 0) return TOCR_OK;
  TOCR_REQUIRE(d_probs && d_indices && d_scores, "tocr_argmax_f32: null pointer");
  TOCR_REQUIRE(aligned(d_probs, 4), "tocr_argmax_f32: probs must be 4-byte aligned");
  argmax_rows_f32_kernel<<<rows_grid(argmax_rows_f32_kernel, rows), kRowsThreads, 0, as_stream(stream)>>>(
      d_probs, rows, num_classes, d_indices, d_scores);
  return check_launch("argmax_rows_f32_kernel");
}

TOCR_API int tocr_ctc_greedy_f16(const void *d_logits, int batch_size, int seq_len,
                                 int num_classes, int num_labels, int *d_tokens,
                                 int *d_lengths, float *d_line_scores, int *d_step_idx,
                                 float *d_step_prob, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(batch_size >= 0 && seq_len >= 0 && num_classes > 0,
               "tocr_ctc_greedy_f16: bad sizes batch=%d seq_len=%d classes=%d",
               batch_size, seq_len, num_classes);
  if (batch_size == 0) return TOCR_OK;
  TOCR_REQUIRE(d_lengths && d_line_scores && (d_tokens || seq_len == 0),
               "tocr_ctc_greedy_f16: null output pointer");
  if (seq_len > 0) {
    TOCR_REQUIRE(d_logits && d_step_idx && d_step_prob,
                 "tocr_ctc_greedy_f16: null logits/step pointer");
    TOCR_REQUIRE(aligned(d_logits, 2), "tocr_ctc_greedy_f16: logits must be 2-byte aligned");
    const long long rows = (long long)batch_size * seq_len;
    ctc_rows_f16_kernel<<<rows_grid(ctc_rows_f16_kernel, rows), kRowsThreads, 0, as_stream(stream)>>>(
        reinterpret_cast<const __half *>(d_logits), rows, num_classes, d_step_idx,
        d_step_prob);
    int st = check_launch("ctc_rows_f16_kernel");
    if (st != TOCR_OK) return st;
  }
  const int blocks = (batch_size + kCollapseWarps - 1) / kCollapseWarps;
  ctc_collapse_kernel<<<blocks, kCollapseWarps * 32, 0, as_stream(stream)>>>(
      d_step_idx, d_step_prob, batch_size, seq_len, num_labels, d_tokens, d_lengths,
      d_line_scores);
  return check_launch("ctc_collapse_kernel");
}

// tocr_ctc_greedy_f16 for a batch whose size lives on the device (e.g. the
// crop count of a detection stage, so the call can sit in a CUDA graph):
// lines [0, min(*d_batch, max_batch)) are decoded, the rest untouched.
TOCR_API int tocr_ctc_greedy_f16_dev(const void *d_logits, const int *d_batch, int max_batch,
                                     int seq_len, int num_classes, int num_labels,
                                     int *d_tokens, int *d_lengths, float *d_line_scores,
                                     int *d_step_idx, float *d_step_prob, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(max_batch >= 0 && seq_len > 0 && num_classes > 0,
               "tocr_ctc_greedy_f16_dev: bad sizes max_batch=%d seq_len=%d classes=%d",
               max_batch, seq_len, num_classes);
  if (max_batch == 0) return TOCR_OK;
  TOCR_REQUIRE(d_logits && d_batch && d_tokens && d_lengths && d_line_scores && d_step_idx &&
                   d_step_prob, "tocr_ctc_greedy_f16_dev: null pointer");
  TOCR_REQUIRE(aligned(d_logits, 2), "tocr_ctc_greedy_f16_dev: logits must be 2-byte aligned");
  const long long rows = (long long)max_batch * seq_len;
  ctc_rows_f16_kernel<<<rows_grid(ctc_rows_f16_kernel, rows), kRowsThreads, 0, as_stream(stream)>>>(
      reinterpret_cast<const __half *>(d_logits), rows, num_classes, d_step_idx, d_step_prob,
      d_batch, seq_len);
  int st = check_launch("ctc_rows_f16_kernel");
  if (st != TOCR_OK) return st;
  const int blocks = (max_batch + kCollapseWarps - 1) / kCollapseWarps;
  ctc_collapse_kernel<<<blocks, kCollapseWarps * 32, 0, as_stream(stream)>>>(
      d_step_idx, d_step_prob, max_batch, seq_len, num_labels, d_tokens, d_lengths,
      d_line_scores, d_batch);
  return check_launch("ctc_collapse_kernel");
}

}  // extern "C"

// ---- allocation-free variant -------------------------------------------------
// tocr_ctc_greedy_f16_noalloc keeps the per-step scratch (argmax index and
// max probability of every row) in module-scope device arrays instead of
// caller buffers. Both arrays are fully written by ctc_rows_f16_kernel before
// ctc_collapse_kernel reads them, so nothing has to be cleared between calls.
namespace {

constexpr long long kNoAllocMaxSteps = 1ll << 20;  // 4 MiB of indices + 4 MiB of probabilities

__device__ __align__(256) int g_noalloc_step_idx[kNoAllocMaxSteps];
__device__ __align__(256) float g_noalloc_step_prob[kNoAllocMaxSteps];

struct NoAllocScratch {
  int *idx = nullptr;
  float *prob = nullptr;
};

// Device addresses of the scratch arrays in the current context. They are
// looked up on every call rather than cached: a device reset or a new
// primary context reloads the module at another address, and after the
// first call (which may load the module) the lookup is cheap.
int noalloc_scratch(NoAllocScratch *out) {
  void *pi = nullptr, *pp = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&pi, g_noalloc_step_idx);
  if (e != cudaSuccess)
    return set_error(TOCR_ERR_CUDA, "cudaGetSymbolAddress(step_idx): %s", cudaGetErrorString(e));
  e = cudaGetSymbolAddress(&pp, g_noalloc_step_prob);
  if (e != cudaSuccess)
    return set_error(TOCR_ERR_CUDA, "cudaGetSymbolAddress(step_prob): %s", cudaGetErrorString(e));
  out->idx = static_cast<int *>(pi);
  out->prob = static_cast<float *>(pp);
  return TOCR_OK;
}

}  // namespace

extern "C" TOCR_API int tocr_ctc_greedy_f16_noalloc(const void *d_logits, int batch_size,
                                                    int seq_len, int num_classes,
                                                    int num_labels, int *d_tokens,
                                                    int *d_lengths, float *d_line_scores,
                                                    void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(batch_size >= 0 && seq_len >= 0 && num_classes > 0,
               "tocr_ctc_greedy_f16_noalloc: bad sizes batch=%d seq_len=%d classes=%d",
               batch_size, seq_len, num_classes);
  const long long rows = (long long)batch_size * seq_len;
  TOCR_REQUIRE(rows <= kNoAllocMaxSteps,
               "tocr_ctc_greedy_f16_noalloc: batch*seq_len = %lld exceeds the static scratch of "
               "%lld steps; use tocr_ctc_greedy_f16 with caller buffers",
               rows, kNoAllocMaxSteps);
  if (batch_size == 0) return TOCR_OK;
  TOCR_REQUIRE(d_lengths && d_line_scores && (d_tokens || seq_len == 0),
               "tocr_ctc_greedy_f16_noalloc: null output pointer");
  NoAllocScratch scr;
  int st = noalloc_scratch(&scr);
  if (st != TOCR_OK) return st;
  if (seq_len > 0) {
    TOCR_REQUIRE(d_logits, "tocr_ctc_greedy_f16_noalloc: null logits pointer");
    TOCR_REQUIRE(aligned(d_logits, 2),
                 "tocr_ctc_greedy_f16_noalloc: logits must be 2-byte aligned");
    ctc_rows_f16_kernel<<<rows_grid(ctc_rows_f16_kernel, rows), kRowsThreads, 0,
                          as_stream(stream)>>>(reinterpret_cast<const __half *>(d_logits), rows,
                                               num_classes, scr.idx, scr.prob);
    st = check_launch("ctc_rows_f16_kernel");
    if (st != TOCR_OK) return st;
  }
  const int blocks = (batch_size + kCollapseWarps - 1) / kCollapseWarps;
  ctc_collapse_kernel<<<blocks, kCollapseWarps * 32, 0, as_stream(stream)>>>(
      scr.idx, scr.prob, batch_size, seq_len, num_labels, d_tokens, d_lengths, d_line_scores);
  return check_launch("ctc_collapse_kernel");
}
