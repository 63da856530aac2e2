// Seeded synthetic inputs for the parity tests and bench.py, built as
// libtocr_synth.so beside the product library. The end-to-end page pipeline
// (turboocr_b200/pipeline.py) loads it for one stage: the recognition network
// is out of scope, so tocr_synth_rec_logits writes stand-in CTC logits per
// crop. Every other entry here only makes test and benchmark inputs.
//
// One counter-based generator everywhere: value i of stream s under seed k is
// mix64(k + golden * (mix64(s) + i + 1)) (splitmix64 finaliser), so any
// element can be produced independently on host or device. Config seeds are
// 0x7EC00000 + config index.
#include "tocr_common.cuh"

#include <cmath>

namespace synth {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t hash3(uint64_t seed, uint64_t stream, uint64_t i) {
  return mix64(seed + 0x9E3779B97F4A7C15ULL * (mix64(stream) + i + 1));
}
// uniform in [0,1) with 24 bits
__host__ __device__ __forceinline__ float unif(uint64_t h) {
  return (float)(h >> 40) * (1.0f / 16777216.0f);
}
// uniform integer in [lo, hi]
__host__ __device__ __forceinline__ int unif_int(uint64_t h, int lo, int hi) {
  return lo + (int)((h >> 32) % (uint64_t)(hi - lo + 1));
}

// ---- uniform bytes ---------------------------------------------------------
__global__ void fill_u8_kernel(uint8_t *d, long long n, uint64_t seed, uint64_t stream) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i * 8 < n; i += stride) {
    const uint64_t h = hash3(seed, stream, (uint64_t)i);
    for (int k = 0; k < 8 && i * 8 + k < n; ++k) d[i * 8 + k] = (uint8_t)(h >> (8 * k));
  }
}

// ---- CTC logits (config 2) ---------------------------------------------------
// Plan per line: n_tok ~ U{5..40} tokens ~ U{1..V-1}, each a run of U{1..4}
// steps, a blank run (index 0) of U{1..3} steps before every token and none
// after; runs shrink to 1 step when the line would exceed T. plan[b*T+t] is
// the planted index of step t or -1 (left random).
__global__ void ctc_plan_kernel(int *plan, int B, int T, int V, uint64_t seed) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  uint64_t ctr = 0;
  const uint64_t st = 1000 + (uint64_t)b;
  const int n_tok = unif_int(hash3(seed, st, ctr++), 5, 40);
  int tok[40], run[40], gap[40];
  int total = 0;
  for (int k = 0; k < n_tok; ++k) {
    tok[k] = unif_int(hash3(seed, st, ctr++), 1, V - 1);
    run[k] = unif_int(hash3(seed, st, ctr++), 1, 4);
    gap[k] = unif_int(hash3(seed, st, ctr++), 1, 3);
    total += run[k] + gap[k];
  }
  for (int k = 0; k < n_tok && total > T; ++k) { total -= gap[k] - 1; gap[k] = 1; }
  for (int k = 0; k < n_tok && total > T; ++k) { total -= run[k] - 1; run[k] = 1; }
  int t = 0;
  int *p = plan + (long long)b * T;
  for (int k = 0; k < n_tok && t < T; ++k) {
    for (int g = 0; g < gap[k] && t < T; ++g) p[t++] = 0;
    for (int r = 0; r < run[k] && t < T; ++r) p[t++] = tok[k];
  }
  for (; t < T; ++t) p[t] = -1;
}

__global__ void normal_f16_kernel(__half *d, long long n, float sigma, uint64_t seed,
                                  uint64_t stream) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; 2 * i < n; i += stride) {
    const uint64_t h = hash3(seed, stream, (uint64_t)i);
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1)) * sigma;
    float s, c;
    sincospif(2.0f * u2, &s, &c);
    d[2 * i] = __float2half_rn(r * c);
    if (2 * i + 1 < n) d[2 * i + 1] = __float2half_rn(r * s);
  }
}

// One warp per row: planted index gets (row max + 2.0).
__global__ void ctc_plant_kernel(__half *logits, const int *plan, long long rows, int V) {
  const int lane = threadIdx.x & 31;
  const long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= rows) return;
  const int pi = plan[r];
  if (pi < 0) return;
  __half *row = logits + r * V;
  float m = -INFINITY;
  for (int j = lane; j < V; j += 32) m = fmaxf(m, __half2float(row[j]));
  for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  __syncwarp();
  if (lane == 0) row[pi] = __float2half_rn(m + 2.0f);
}

// ---- config-5 pages ------------------------------------------------------------
// Page m: white (255) u8 HWC. n_lines ~ U{30..80} text lines at a pitch of
// H / n_lines; line i: glyph height ~ U{6..min(14, pitch - 3)}, left margin
// U{16..160}, length U{120..W - 40 - left}; glyphs are black (0) rectangles of
// width U{4..10} separated by 2 px inside a word; words of U{2..8} glyphs are
// separated by U{6..12} px. One CTA per (line slot, page); thread 0 lays the
// line out, all threads paint it.
constexpr int kMaxGlyphs = 512;

__global__ void __launch_bounds__(256)
page_lines_kernel(uint8_t *pages, int H, int W, uint64_t seed, long long first_page) {
  const long long m = blockIdx.y;
  const int line = blockIdx.x;
  const uint64_t st = 5000 + (uint64_t)(first_page + m);
  const int n_lines = unif_int(hash3(seed, st, 0), 30, 80);
  if (line >= n_lines) return;
  __shared__ int gx0[kMaxGlyphs], gx1[kMaxGlyphs];
  __shared__ int s_ng, s_y0, s_y1;
  if (threadIdx.x == 0) {
    const uint64_t ls = ((uint64_t)(first_page + m) << 8) + (uint64_t)line;
    uint64_t ctr = 0;
    const float pitch = (float)H / (float)n_lines;
    const int hmax = min(14, (int)pitch - 3);
    const int gh = unif_int(hash3(seed, ls, ctr++), 6, max(6, hmax));
    const int yc = (int)((line + 0.5f) * pitch);
    s_y0 = max(0, yc - gh / 2);
    s_y1 = min(H, s_y0 + gh);
    const int left = unif_int(hash3(seed, ls, ctr++), 16, 160);
    const int len = unif_int(hash3(seed, ls, ctr++), 120, max(120, W - 40 - left));
    const int end = min(W - 8, left + len);
    int x = left, ng = 0;
    while (x < end && ng < kMaxGlyphs) {
      const int nw = unif_int(hash3(seed, ls, ctr++), 2, 8);
      for (int g = 0; g < nw && x < end && ng < kMaxGlyphs; ++g) {
        const int gw = unif_int(hash3(seed, ls, ctr++), 4, 10);
        gx0[ng] = x;
        gx1[ng] = min(end, x + gw);
        ++ng;
        x += gw + 2;
      }
      x += unif_int(hash3(seed, ls, ctr++), 6, 12) - 2;
    }
    s_ng = ng;
  }
  __syncthreads();
  uint8_t *pg = pages + m * (long long)H * W * 3;
  const int rows = s_y1 - s_y0;
  for (int g = 0; g < s_ng; ++g) {
    const int w = gx1[g] - gx0[g];
    for (int i = threadIdx.x; i < w * rows * 3; i += blockDim.x) {
      const int c = i % 3, px = (i / 3) % w, ry = (i / 3) / w;
      pg[((long long)(s_y0 + ry) * W + gx0[g] + px) * 3 + c] = 0;
    }
  }
}

// ---- stand-in recognition logits for the crops of config 5 ----------------------
// Row (crop c, step t): noise in [-4, 4) from a fixed 8192-entry table read
// in flat 16-byte chunks (a pure streaming write), then a planted value 8 at
// the row's token: a blank (0) or a label in U{1..V-1}, held for 3 steps.
// Rows of crops >= *n_crops are not written.
__device__ __forceinline__ int rec_token(uint64_t seed, long long c, int t, int V) {
  const uint64_t th = hash3(seed, 7000 + (uint64_t)c, (uint64_t)(t / 3));
  return (th & 1) ? 0 : unif_int(th, 1, V - 1);
}

constexpr int kNoiseChunks = 1024;  // table of 1024 x 8 halves

__global__ void __launch_bounds__(256)
rec_noise_kernel(__half *logits, const int *n_crops, int max_crops, int T, int V, uint64_t seed) {
  __shared__ uint4 table[kNoiseChunks];
  for (int i = threadIdx.x; i < kNoiseChunks; i += blockDim.x) {
    const uint64_t h = hash3(seed, 9000, (uint64_t)i);
    __align__(16) __half v[8];
    for (int k = 0; k < 8; ++k)
      v[k] = __float2half_rn((float)((h >> (8 * k)) & 0xFF) * (8.0f / 256.0f) - 4.0f);
    table[i] = *reinterpret_cast<const uint4 *>(v);
  }
  __syncthreads();
  const long long n_el = (long long)min(*n_crops, max_crops) * T * V;
  const long long n_full = n_el / 8;
  uint4 *out = reinterpret_cast<uint4 *>(logits);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n_full; i += stride)
    out[i] = table[(i * 7 + (i >> 10)) & (kNoiseChunks - 1)];
  if (blockIdx.x == 0 && threadIdx.x < (int)(n_el - n_full * 8))
    logits[n_full * 8 + threadIdx.x] = __float2half_rn(0.0f);
}

__global__ void __launch_bounds__(256)
rec_plant_kernel(__half *logits, const int *n_crops, int max_crops, int T, int V, uint64_t seed) {
  const long long rows = (long long)min(*n_crops, max_crops) * T;
  const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  logits[r * V + rec_token(seed, r / T, (int)(r % T), V)] = __float2half_rn(8.0f);
}

}  // namespace synth

using namespace synth;

extern "C" {

TOCR_API uint64_t tocr_synth_hash(uint64_t seed, uint64_t stream, uint64_t i) {
  return hash3(seed, stream, i);
}

TOCR_API int tocr_synth_fill_u8(void *d, long long n, uint64_t seed, uint64_t stream,
                                void *cuda_stream) {
  if (n <= 0) return 0;
  const long long need = (n / 8 + 256) / 256;
  const int grid = (int)(need < 148 * 16 ? need : 148 * 16);
  fill_u8_kernel<<<grid, 256, 0, (cudaStream_t)cuda_stream>>>((uint8_t *)d, n, seed, stream);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

TOCR_API int tocr_synth_normal_f16(void *d, long long n, float sigma, uint64_t seed,
                                   uint64_t stream, void *cuda_stream) {
  if (n <= 0) return 0;
  const long long need = (n / 2 + 256) / 256;
  const int grid = (int)(need < 148 * 16 ? need : 148 * 16);
  normal_f16_kernel<<<grid, 256, 0, (cudaStream_t)cuda_stream>>>((__half *)d, n, sigma, seed,
                                                                  stream);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// Config-2 logits: fills d_logits [B,T,V] fp16 and d_plan [B*T].
TOCR_API int tocr_synth_ctc_logits(void *d_logits, int *d_plan, int B, int T, int V,
                                   uint64_t seed, void *cuda_stream) {
  cudaStream_t s = (cudaStream_t)cuda_stream;
  const long long n = (long long)B * T * V;
  ctc_plan_kernel<<<(B + 127) / 128, 128, 0, s>>>(d_plan, B, T, V, seed);
  tocr_synth_normal_f16(d_logits, n, 4.0f, seed, 1, cuda_stream);
  const long long rows = (long long)B * T;
  ctc_plant_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>((__half *)d_logits,
                                                                       d_plan, rows, V);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// Config-1 DB probability maps (host): background U[0, 0.1]; k ~ U{kmin..kmax}
// rotated rectangles (width U[20,400], height U[8,60], angle U[-15,15] deg,
// centre uniform in the map) filled with U[0.6, 1.0]; a pixel belongs to a
// rectangle when its centre (x+0.5, y+0.5) lies inside (double arithmetic);
// later rectangles overwrite earlier ones. Returns the rectangle count.
TOCR_API int tocr_synth_db_map_host(float *out, int H, int W, int kmin, int kmax, uint64_t seed,
                                    uint64_t map_index) {
  const uint64_t st = 3000 + map_index;
  uint64_t ctr = 0;
  for (long long i = 0; i < (long long)H * W; ++i)
    out[i] = 0.1f * unif(hash3(seed, st + (1ull << 40), (uint64_t)i));
  const int k = unif_int(hash3(seed, st, ctr++), kmin, kmax);
  for (int r = 0; r < k; ++r) {
    const double w = 20.0 + 380.0 * unif(hash3(seed, st, ctr++));
    const double h = 8.0 + 52.0 * unif(hash3(seed, st, ctr++));
    const double th = (-15.0 + 30.0 * unif(hash3(seed, st, ctr++))) * 3.141592653589793 / 180.0;
    const double cx = W * (double)unif(hash3(seed, st, ctr++));
    const double cy = H * (double)unif(hash3(seed, st, ctr++));
    const double c = cos(th), s = sin(th);
    const double ex = 0.5 * (fabs(w * c) + fabs(h * s)), ey = 0.5 * (fabs(w * s) + fabs(h * c));
    const int x0 = (int)fmax(0.0, floor(cx - ex - 1)), x1 = (int)fmin(W - 1.0, ceil(cx + ex + 1));
    const int y0 = (int)fmax(0.0, floor(cy - ey - 1)), y1 = (int)fmin(H - 1.0, ceil(cy + ey + 1));
    const uint64_t fill_stream = st + (2ull << 40) + (uint64_t)r;
    for (int y = y0; y <= y1; ++y)
      for (int x = x0; x <= x1; ++x) {
        const double dx = x + 0.5 - cx, dy = y + 0.5 - cy;
        const double u = dx * c + dy * s, v = -dx * s + dy * c;
        if (fabs(u) <= 0.5 * w && fabs(v) <= 0.5 * h)
          out[(long long)y * W + x] = 0.6f + 0.4f * unif(hash3(seed, fill_stream, (uint64_t)(y * W + x)));
      }
  }
  return k;
}

// Config-5 pages u8 [n][H][W][3] (pages first_page .. first_page + n - 1).
TOCR_API int tocr_synth_pages(void *d_pages, int n, int H, int W, uint64_t seed,
                              long long first_page, void *cuda_stream) {
  if (n <= 0) return 0;
  cudaStream_t s = (cudaStream_t)cuda_stream;
  if (cudaMemsetAsync(d_pages, 255, (size_t)n * H * W * 3, s) != cudaSuccess) return 2;
  page_lines_kernel<<<dim3(80, n), 256, 0, s>>>((uint8_t *)d_pages, H, W, seed, first_page);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// Stand-in recognition logits fp16 [max_crops][T][V] for the first *d_n_crops crops.
TOCR_API int tocr_synth_rec_logits(void *d_logits, const int *d_n_crops, int max_crops, int T,
                                   int V, uint64_t seed, void *cuda_stream) {
  if (max_crops <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(d_logits) & 15) != 0) return 1;
  cudaStream_t s = (cudaStream_t)cuda_stream;
  rec_noise_kernel<<<148 * 4, 256, 0, s>>>((__half *)d_logits, d_n_crops, max_crops, T, V, seed);
  const long long rows = (long long)max_crops * T;
  rec_plant_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>((__half *)d_logits, d_n_crops,
                                                                  max_crops, T, V, seed);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // extern "C"
