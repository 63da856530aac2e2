// Mode-2 detection geometry (the reference's all-device unclip,
// src/kernels/jfa.cu:75-498, include/turbo_ocr/kernels/kernels.h:160-229):
// every component of the CCL compact-id map grows by its own distance
// e = pixel_count * ratio / crack perimeter (clamped), a background pixel
// goes to the component whose boundary pixel is nearest among those whose
// disc of radius e reaches it (ties: the smaller component id), and the
// grown regions are reduced to an axis-aligned box and a PCA-oriented
// rectangle.
//
// Results are the reference's bit for bit (same packed (d2, id) winner key,
// same float/double expressions); the work is arranged for the device:
//   * crack perimeters: warp-aggregated atomics (one per component per warp);
//   * disc stamping: boundary seeds are first compacted into a list (ballot
//     per warp), so stamping warps are dense and neighbouring lanes stamp
//     neighbouring pixels (coalesced atomicMin), instead of one mostly idle
//     thread per pixel;
//   * extraction: one thread per 32-pixel row segment reduces each run of
//     equal labels in closed form (box, count, first and second moments as
//     exact integer sums; the projections are monotone along a row, so a
//     run's extreme projections are those of its end pixels) and flushes one
//     set of atomics per run instead of one per pixel.
// Integer sums, min/max and the winner key do not depend on the order of
// the atomics, so the reduction order changes no result.
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdint>

#include "tocr_common.cuh"

namespace tocr {
namespace {

// GpuDetBox (include/turbo_ocr/kernels/kernels.h, 56 bytes).
struct DetBox {
  int xmin, ymin, xmax, ymax;
  float score;
  int pixel_count;
  float ox[4], oy[4];
};
static_assert(sizeof(DetBox) == 56, "GpuDetBox layout");

constexpr int kMaxComponents = 3000;
// Winner key of a pixel: squared distance above kLabelBits bits of component
// id, so the unsigned minimum is the nearest seed and, among equally near
// ones, the smallest id (the reference's tie rule, jfa.cu:47-62).
constexpr int kLabelBits = 13;
constexpr uint32_t kLabelMask = (1u << kLabelBits) - 1u;
constexpr uint32_t kKeyEmpty = 0xFFFFFFFFu;
constexpr int kMaxSafeExpand = 723;  // keeps d2 << kLabelBits inside 32 bits
static_assert(kMaxSafeExpand * kMaxSafeExpand < (1 << (32 - kLabelBits)), "key budget");
static_assert(kMaxComponents <= (int)kLabelMask, "component id fits the key");
constexpr int kSeg = 32;  // pixels of a row per extraction thread

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

// ---------------------------------------------------------------- perimeter --
// Exposed 4-connected crack edges of every foreground pixel (edges facing
// background or the image border), summed per component id.
__global__ void __launch_bounds__(256)
crack_kernel(const int32_t *__restrict__ cid, const uint8_t *__restrict__ bm, int w, int h,
             int num_slots, int *__restrict__ perim) {
  const long long n = (long long)w * h;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long p0 = (long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31); p0 < n;
       p0 += stride) {
    const long long p = p0 + lane_id();
    int id = -1, c = 0;
    if (p < n && bm[p]) {
      id = cid[p];
      if (id >= 0 && id < num_slots) {
        const int x = (int)(p % w), y = (int)(p / w);
        c = (x == 0 || !bm[p - 1]) + (x == w - 1 || !bm[p + 1]) + (y == 0 || !bm[p - w]) +
            (y == h - 1 || !bm[p + w]);
      } else {
        id = -1;
      }
    }
    const unsigned grp = __match_any_sync(0xffffffffu, id);
    const int s = (int)__reduce_add_sync(grp, (unsigned)c);
    if (id >= 0 && s != 0 && lane_id() == __ffs(grp) - 1) atomicAdd(&perim[id], s);
  }
}

// ------------------------------------------------------------ expand distance --
// jfa.cu:191-212: 0 for empty, small or low-scoring slots (score is the sum of
// the prediction over the component, as cuda_gpu_ccl_detect leaves it in its
// first kMaxGpuComponents records), else pixel_count * ratio / perimeter
// clamped to [min_expand, max_expand] (the bbox perimeter when no crack was
// counted).
__global__ void expand_kernel(const DetBox *__restrict__ boxes, const int *__restrict__ perim,
                              int num_slots, float unclip_ratio, float min_expand,
                              float max_expand, float box_thresh, float *__restrict__ expand) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= num_slots) return;
  const DetBox b = boxes[i];
  const int pc = b.pixel_count;
  const int bw = b.xmax - b.xmin + 1, bh = b.ymax - b.ymin + 1;
  float e = 0.0f;
  if (pc >= 3 && bw >= 3 && bh >= 3) {
    const float score = b.score / (float)pc;
    if (!(score < box_thresh)) {
      float pr = (float)perim[i];
      if (pr < 1.0f) pr = 2.0f * (float)(bw + bh);
      const float area = (float)pc;
      e = area * unclip_ratio / pr;
      if (e < min_expand) e = min_expand;
      if (e > max_expand) e = max_expand;
    }
  }
  expand[i] = e;
}

// ------------------------------------------------------------- disc stamps --
__device__ __forceinline__ bool is_seed(const uint8_t *__restrict__ bm, int x, int y, int w,
                                        int h) {
  const long long p = (long long)y * w + x;
  if (!bm[p]) return false;
  for (int dy = -1; dy <= 1; ++dy)
    for (int dx = -1; dx <= 1; ++dx) {
      if ((dx | dy) == 0) continue;
      const int nx = x + dx, ny = y + dy;
      if (nx < 0 || nx >= w || ny < 0 || ny >= h) continue;
      if (!bm[(long long)ny * w + nx]) return true;
    }
  return false;
}

// The disc of one seed: every pixel with d2 <= e^2 (in float, as the
// reference compares) takes min(key, (d2 << 13) | id).
__device__ __forceinline__ void stamp(uint32_t *__restrict__ best, int x, int y, int id, float e,
                                      int w, int h) {
  if (e > (float)kMaxSafeExpand) e = (float)kMaxSafeExpand;
  const float e2 = e * e;
  const int r = (int)ceilf(e);
  const int y0 = max(y - r, 0), y1 = min(y + r, h - 1);
  const int x0 = max(x - r, 0), x1 = min(x + r, w - 1);
  for (int ty = y0; ty <= y1; ++ty) {
    const int dy = ty - y;
    const int dy2 = dy * dy;
    uint32_t *row = best + (long long)ty * w;
    for (int tx = x0; tx <= x1; ++tx) {
      const int dx = tx - x;
      const int d2 = dx * dx + dy2;
      if ((float)d2 > e2) continue;
      atomicMin(row + tx, ((uint32_t)d2 << kLabelBits) | (uint32_t)id);
    }
  }
}

// Boundary seeds (foreground pixels with an in-bounds background 8-neighbour,
// a component id and a positive distance) as raster indices: list[0] counts,
// entries follow. A foreground pixel is needed for a seed and a background
// one for it to be a boundary, so at most w*h - 1 entries exist.
__global__ void __launch_bounds__(256)
seed_kernel(const uint8_t *__restrict__ bm, const int32_t *__restrict__ cid,
            const float *__restrict__ expand, int w, int h, uint32_t *__restrict__ list) {
  const long long n = (long long)w * h;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long p0 = (long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31); p0 < n;
       p0 += stride) {
    const long long p = p0 + lane_id();
    bool s = false;
    if (p < n) {
      const int id = bm[p] ? cid[p] : -1;
      if (id >= 0 && id < kMaxComponents && expand[id] > 0.0f)
        s = is_seed(bm, (int)(p % w), (int)(p / w), w, h);
    }
    const unsigned b = __ballot_sync(0xffffffffu, s);
    if (b == 0) continue;
    uint32_t base = 0;
    if (lane_id() == 0) base = atomicAdd(list, (uint32_t)__popc(b));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (s) {
      const uint32_t k = base + (uint32_t)__popc(b & ((1u << lane_id()) - 1u));
      if ((long long)k + 1 < n) list[k + 1] = (uint32_t)p;
    }
  }
}

__global__ void __launch_bounds__(256)
stamp_list_kernel(const uint32_t *__restrict__ list, const int32_t *__restrict__ cid,
                  const float *__restrict__ expand, int w, int h, uint32_t *__restrict__ best) {
  const long long n = (long long)w * h;
  long long cnt = list[0];
  if (cnt > n - 1) cnt = n - 1;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < cnt;
       k += (long long)gridDim.x * blockDim.x) {
    const long long p = list[k + 1];
    const int id = cid[p];
    stamp(best, (int)(p % w), (int)(p / w), id, expand[id], w, h);
  }
}

// Without a seed-list buffer: every pixel tests itself.
__global__ void __launch_bounds__(256)
stamp_pixels_kernel(const uint8_t *__restrict__ bm, const int32_t *__restrict__ cid,
                    const float *__restrict__ expand, int w, int h,
                    uint32_t *__restrict__ best) {
  const long long n = (long long)w * h;
  for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < n;
       p += (long long)gridDim.x * blockDim.x) {
    const int id = bm[p] ? cid[p] : -1;
    if (id < 0 || id >= kMaxComponents) continue;
    const float e = expand[id];
    if (!(e > 0.0f)) continue;
    const int x = (int)(p % w), y = (int)(p / w);
    if (is_seed(bm, x, y, w, h)) stamp(best, x, y, id, e, w, h);
  }
}

__global__ void __launch_bounds__(256)
fill_kernel(uint32_t *__restrict__ a, long long n, uint32_t v) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    a[i] = v;
}

// Final label per pixel: 1 + id (0 = none). Foreground keeps its own
// component (when that component has a positive distance), background takes
// the winner of its key.
__global__ void __launch_bounds__(256)
resolve_kernel(const uint32_t *__restrict__ best, const uint8_t *__restrict__ bm,
               const int32_t *__restrict__ cid, const float *__restrict__ expand, int w, int h,
               uint32_t *__restrict__ out) {
  const long long n = (long long)w * h;
  for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < n;
       p += (long long)gridDim.x * blockDim.x) {
    uint32_t l = 0;
    if (bm[p]) {
      const int id = cid[p];
      if (id >= 0 && id < kMaxComponents && expand[id] > 0.0f) l = (uint32_t)id + 1u;
    } else {
      const uint32_t key = best[p];
      if (key != kKeyEmpty) l = (key & kLabelMask) + 1u;
    }
    out[p] = l;
  }
}

// ------------------------------------------------------------- extraction --
__global__ void box_init_kernel(DetBox *__restrict__ boxes, int num_slots) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= num_slots) return;
  DetBox &b = boxes[i];
  b.xmin = INT_MAX;
  b.ymin = INT_MAX;
  b.xmax = INT_MIN;
  b.ymax = INT_MIN;
  b.pixel_count = 0;
  b.score = 0.0f;
}

// sum of k^2 for k = 0..m (m >= -1)
__device__ __forceinline__ unsigned long long sq_sum(long long m) {
  if (m < 0) return 0ull;
  const unsigned long long u = (unsigned long long)m;
  return u * (u + 1) * (2 * u + 1) / 6;
}

// A run of label `l` (> 0) on row y from xa to xb (inclusive).
template <bool kMoments>
__device__ __forceinline__ void flush_run(uint32_t l, int xa, int xb, int y, int num_slots,
                                          DetBox *__restrict__ boxes,
                                          unsigned long long *__restrict__ mom) {
  if (l == 0) return;
  const int id = (int)l - 1;
  if (id >= num_slots) return;
  DetBox &b = boxes[id];
  const int cnt = xb - xa + 1;
  atomicMin(&b.xmin, xa);
  atomicMax(&b.xmax, xb);
  atomicMin(&b.ymin, y);
  atomicMax(&b.ymax, y);
  atomicAdd(&b.pixel_count, cnt);
  if (kMoments) {
    const unsigned long long n = (unsigned long long)cnt, uy = (unsigned long long)y;
    const unsigned long long sx = ((unsigned long long)xa + (unsigned long long)xb) * n / 2;
    const unsigned long long sxx = sq_sum(xb) - sq_sum((long long)xa - 1);
    unsigned long long *m = mom + (size_t)id * 6;
    atomicAdd(&m[0], n);
    atomicAdd(&m[1], sx);
    atomicAdd(&m[2], uy * n);
    atomicAdd(&m[3], sxx);
    atomicAdd(&m[4], uy * uy * n);
    atomicAdd(&m[5], uy * sx);
  }
}

// One thread per kSeg-pixel segment of a row; runs of equal labels flush once.
template <bool kMoments>
__global__ void __launch_bounds__(256)
extract_kernel(const uint32_t *__restrict__ labels, int w, int h, int num_slots,
               DetBox *__restrict__ boxes, unsigned long long *__restrict__ mom) {
  const int segs = (w + kSeg - 1) / kSeg;
  const long long total = (long long)segs * h;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(t / segs), x0 = (int)(t % segs) * kSeg;
    const int x1 = min(x0 + kSeg, w);
    const uint32_t *row = labels + (long long)y * w;
    uint32_t cur = row[x0];
    int xa = x0;
    for (int x = x0 + 1; x < x1; ++x) {
      const uint32_t l = row[x];
      if (l != cur) {
        flush_run<kMoments>(cur, xa, x - 1, y, num_slots, boxes, mom);
        cur = l;
        xa = x;
      }
    }
    flush_run<kMoments>(cur, xa, x1 - 1, y, num_slots, boxes, mom);
  }
}

// Principal axis of every component from its moments (jfa.cu:318-345): the
// same double expressions, so the same angle; projection extents seeded.
__global__ void axis_kernel(const unsigned long long *__restrict__ mom, int num_slots,
                            float *__restrict__ orient) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= num_slots) return;
  const unsigned long long *m = mom + (size_t)i * 6;
  float *o = orient + (size_t)i * 6;
  const unsigned long long n = m[0];
  o[2] = INFINITY;
  o[3] = -INFINITY;
  o[4] = INFINITY;
  o[5] = -INFINITY;
  if (n < 3) {
    o[0] = 1.0f;
    o[1] = 0.0f;
    return;
  }
  double dn = (double)n;
  double mx = (double)m[1] / dn, my = (double)m[2] / dn;
  double cxx = (double)m[3] / dn - mx * mx;
  double cyy = (double)m[4] / dn - my * my;
  double cxy = (double)m[5] / dn - mx * my;
  double trace = cxx + cyy;
  double aniso = sqrt((cxx - cyy) * (cxx - cyy) + 4.0 * cxy * cxy);
  if (trace <= 0.0 || aniso < 0.05 * trace) {
    o[0] = 1.0f;
    o[1] = 0.0f;
    return;
  }
  double theta = 0.5 * atan2(2.0 * cxy, cxx - cyy);
  o[0] = (float)cos(theta);
  o[1] = (float)sin(theta);
}

__device__ __forceinline__ void atomic_min_float(float *a, float v) {
  int *ai = reinterpret_cast<int *>(a);
  int old = *ai, assumed;
  do {
    assumed = old;
    old = atomicCAS(ai, assumed, __float_as_int(fminf(v, __int_as_float(assumed))));
  } while (assumed != old);
}
__device__ __forceinline__ void atomic_max_float(float *a, float v) {
  int *ai = reinterpret_cast<int *>(a);
  int old = *ai, assumed;
  do {
    assumed = old;
    old = atomicCAS(ai, assumed, __float_as_int(fmaxf(v, __int_as_float(assumed))));
  } while (assumed != old);
}

// Projection of pixel (x, y) on the component basis, written exactly as the
// per-pixel reference does so that the compiler forms the same products.
__device__ __forceinline__ float proj_u(int x, int y, float c, float s) { return x * c + y * s; }
__device__ __forceinline__ float proj_v(int x, int y, float c, float s) { return -x * s + y * c; }

__device__ __forceinline__ void flush_proj(uint32_t l, int xa, int xb, int y, int num_slots,
                                           const unsigned long long *__restrict__ mom,
                                           float *__restrict__ orient) {
  if (l == 0) return;
  const int id = (int)l - 1;
  if (id >= num_slots || mom[(size_t)id * 6] < 3) return;
  float *o = orient + (size_t)id * 6;
  const float c = o[0], s = o[1];
  // Along a row u and v are monotone in x (each rounding step is monotone),
  // so the run's extremes are at its end pixels.
  const float ua = proj_u(xa, y, c, s), ub = proj_u(xb, y, c, s);
  const float va = proj_v(xa, y, c, s), vb = proj_v(xb, y, c, s);
  atomic_min_float(&o[2], fminf(ua, ub));
  atomic_max_float(&o[3], fmaxf(ua, ub));
  atomic_min_float(&o[4], fminf(va, vb));
  atomic_max_float(&o[5], fmaxf(va, vb));
}

__global__ void __launch_bounds__(256)
project_kernel(const uint32_t *__restrict__ labels, int w, int h, int num_slots,
               const unsigned long long *__restrict__ mom, float *__restrict__ orient) {
  const int segs = (w + kSeg - 1) / kSeg;
  const long long total = (long long)segs * h;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(t / segs), x0 = (int)(t % segs) * kSeg;
    const int x1 = min(x0 + kSeg, w);
    const uint32_t *row = labels + (long long)y * w;
    uint32_t cur = row[x0];
    int xa = x0;
    for (int x = x0 + 1; x < x1; ++x) {
      const uint32_t l = row[x];
      if (l != cur) {
        flush_proj(cur, xa, x - 1, y, num_slots, mom, orient);
        cur = l;
        xa = x;
      }
    }
    flush_proj(cur, xa, x1 - 1, y, num_slots, mom, orient);
  }
}

// Rectangle corners from the axis and extents (jfa.cu:381-409); components
// with fewer than 3 pixels or no extent keep their axis-aligned box.
__global__ void emit_kernel(const unsigned long long *__restrict__ mom,
                            const float *__restrict__ orient, int num_slots,
                            DetBox *__restrict__ boxes) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= num_slots) return;
  DetBox &b = boxes[i];
  const float *o = orient + (size_t)i * 6;
  if (mom[(size_t)i * 6] < 3 || o[2] > o[3]) {
    const float x0 = (float)b.xmin, y0 = (float)b.ymin;
    const float x1 = (float)b.xmax, y1 = (float)b.ymax;
    b.ox[0] = x0; b.oy[0] = y0;
    b.ox[1] = x1; b.oy[1] = y0;
    b.ox[2] = x1; b.oy[2] = y1;
    b.ox[3] = x0; b.oy[3] = y1;
    return;
  }
  const float c = o[0], s = o[1];
  const float umin = o[2], umax = o[3], vmin = o[4], vmax = o[5];
  const float uu[4] = {umin, umax, umax, umin};
  const float vv[4] = {vmin, vmin, vmax, vmax};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    b.ox[k] = uu[k] * c - vv[k] * s;
    b.oy[k] = uu[k] * s + vv[k] * c;
  }
}

unsigned grid_for(long long items, int threads) {
  const long long g = (items + threads - 1) / threads;
  const long long cap = (long long)sm_count() * 16;
  return (unsigned)(g < 1 ? 1 : (g < cap ? g : cap));
}

bool map_ok(int w, int h) { return w > 0 && h > 0 && (long long)w * h < (1ll << 31); }

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API int tocr_jfa_crack_perimeter(const int32_t *d_compact_ids, const uint8_t *d_bitmap,
                                      int w, int h, int num_slots, int *d_perim,
                                      void *stream) {
  TOCR_ENTRY();
  if (num_slots <= 0) return TOCR_OK;
  TOCR_REQUIRE(map_ok(w, h), "tocr_jfa_crack_perimeter: bad sizes %dx%d", w, h);
  TOCR_REQUIRE(num_slots <= kMaxComponents, "tocr_jfa_crack_perimeter: num_slots %d > %d",
               num_slots, kMaxComponents);
  TOCR_REQUIRE(d_compact_ids && d_bitmap && d_perim, "tocr_jfa_crack_perimeter: null pointer");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(d_perim, 0, (size_t)num_slots * sizeof(int), st);
  if (e != cudaSuccess)
    return set_error(TOCR_ERR_CUDA, "tocr_jfa_crack_perimeter: %s", cudaGetErrorString(e));
  crack_kernel<<<grid_for((long long)w * h, 256), 256, 0, st>>>(d_compact_ids, d_bitmap, w, h,
                                                                num_slots, d_perim);
  return check_launch("tocr_jfa_crack_perimeter");
}

TOCR_API int tocr_jfa_expand_per_comp(const void *d_bboxes, const int *d_perim, int num_slots,
                                      float unclip_ratio, float min_expand, float max_expand,
                                      float box_thresh, float *d_expand, void *stream) {
  TOCR_ENTRY();
  if (num_slots <= 0) return TOCR_OK;
  TOCR_REQUIRE(num_slots <= kMaxComponents, "tocr_jfa_expand_per_comp: num_slots %d > %d",
               num_slots, kMaxComponents);
  TOCR_REQUIRE(d_bboxes && d_perim && d_expand, "tocr_jfa_expand_per_comp: null pointer");
  expand_kernel<<<(num_slots + 127) / 128, 128, 0, as_stream(stream)>>>(
      static_cast<const DetBox *>(d_bboxes), d_perim, num_slots, unclip_ratio, min_expand,
      max_expand, box_thresh, d_expand);
  return check_launch("tocr_jfa_expand_per_comp");
}

TOCR_API int tocr_jfa_expand_labels(const uint8_t *d_bitmap, const int32_t *d_compact_ids,
                                    const float *d_expand, uint32_t *d_labels, int w, int h,
                                    uint32_t *d_keys, uint32_t *d_seed_list, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(map_ok(w, h), "tocr_jfa_expand_labels: bad sizes %dx%d", w, h);
  TOCR_REQUIRE(d_bitmap && d_compact_ids && d_expand && d_labels && d_keys,
               "tocr_jfa_expand_labels: null pointer");
  cudaStream_t st = as_stream(stream);
  const long long n = (long long)w * h;
  const unsigned g = grid_for(n, 256);
  fill_kernel<<<g, 256, 0, st>>>(d_keys, n, kKeyEmpty);
  if (d_seed_list) {
    cudaError_t e = cudaMemsetAsync(d_seed_list, 0, sizeof(uint32_t), st);
    if (e != cudaSuccess)
      return set_error(TOCR_ERR_CUDA, "tocr_jfa_expand_labels: %s", cudaGetErrorString(e));
    seed_kernel<<<g, 256, 0, st>>>(d_bitmap, d_compact_ids, d_expand, w, h, d_seed_list);
    stamp_list_kernel<<<g, 256, 0, st>>>(d_seed_list, d_compact_ids, d_expand, w, h, d_keys);
  } else {
    stamp_pixels_kernel<<<g, 256, 0, st>>>(d_bitmap, d_compact_ids, d_expand, w, h, d_keys);
  }
  resolve_kernel<<<g, 256, 0, st>>>(d_keys, d_bitmap, d_compact_ids, d_expand, w, h, d_labels);
  return check_launch("tocr_jfa_expand_labels");
}

TOCR_API int tocr_jfa_extract_bboxes(const uint32_t *d_labels, int w, int h, void *d_bboxes,
                                     int num_slots, void *stream) {
  TOCR_ENTRY();
  if (num_slots <= 0) return TOCR_OK;
  TOCR_REQUIRE(map_ok(w, h), "tocr_jfa_extract_bboxes: bad sizes %dx%d", w, h);
  TOCR_REQUIRE(num_slots <= kMaxComponents, "tocr_jfa_extract_bboxes: num_slots %d > %d",
               num_slots, kMaxComponents);
  TOCR_REQUIRE(d_labels && d_bboxes, "tocr_jfa_extract_bboxes: null pointer");
  cudaStream_t st = as_stream(stream);
  DetBox *boxes = static_cast<DetBox *>(d_bboxes);
  box_init_kernel<<<(num_slots + 255) / 256, 256, 0, st>>>(boxes, num_slots);
  const long long segs = (long long)((w + kSeg - 1) / kSeg) * h;
  extract_kernel<false><<<grid_for(segs, 256), 256, 0, st>>>(d_labels, w, h, num_slots, boxes,
                                                             nullptr);
  return check_launch("tocr_jfa_extract_bboxes");
}

TOCR_API int tocr_jfa_extract_oriented(const uint32_t *d_labels, int w, int h, void *d_bboxes,
                                       int num_slots, unsigned long long *d_moments,
                                       float *d_orient, void *stream) {
  TOCR_ENTRY();
  if (num_slots <= 0) return TOCR_OK;
  TOCR_REQUIRE(map_ok(w, h), "tocr_jfa_extract_oriented: bad sizes %dx%d", w, h);
  TOCR_REQUIRE(num_slots <= kMaxComponents, "tocr_jfa_extract_oriented: num_slots %d > %d",
               num_slots, kMaxComponents);
  TOCR_REQUIRE(d_labels && d_bboxes && d_moments && d_orient,
               "tocr_jfa_extract_oriented: null pointer");
  cudaStream_t st = as_stream(stream);
  DetBox *boxes = static_cast<DetBox *>(d_bboxes);
  const unsigned cg = (num_slots + 255) / 256;
  box_init_kernel<<<cg, 256, 0, st>>>(boxes, num_slots);
  cudaError_t e = cudaMemsetAsync(d_moments, 0, (size_t)num_slots * 6 * sizeof(unsigned long long), st);
  if (e != cudaSuccess)
    return set_error(TOCR_ERR_CUDA, "tocr_jfa_extract_oriented: %s", cudaGetErrorString(e));
  const long long segs = (long long)((w + kSeg - 1) / kSeg) * h;
  const unsigned sg = grid_for(segs, 256);
  extract_kernel<true><<<sg, 256, 0, st>>>(d_labels, w, h, num_slots, boxes, d_moments);
  axis_kernel<<<cg, 256, 0, st>>>(d_moments, num_slots, d_orient);
  project_kernel<<<sg, 256, 0, st>>>(d_labels, w, h, num_slots, d_moments, d_orient);
  emit_kernel<<<cg, 256, 0, st>>>(d_moments, d_orient, num_slots, boxes);
  return check_launch("tocr_jfa_extract_oriented");
}

}  // extern "C"
