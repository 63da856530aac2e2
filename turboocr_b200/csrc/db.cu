// Subsystem 3 — DB post-processing on B200: probability maps in, ordered
// text quads and their box scores out, with the boxes of the reference's CPU
// path extract_boxes_from_bitmap (src/detection/det_postprocess.cpp:145-222).
//
// Stages (all on the device, one stream, no host round trip):
//   1. ccl_local_kernel    threshold (pred > thresh, cpu_paddle_det.cpp:115) and
//                          tile-local union-find: foreground 8-connected,
//                          background 4-connected, background on the image
//                          frame joined to a virtual "outside" node 0
//   2. ccl_merge_kernel    union across tile borders (atomicMin linking, so every
//                          root is the smallest node of its component)
//   3. ccl_rows_kernel     full path compression, per-row count of border starts
//   4. starts_*            the starts in cv::findContours(RETR_LIST) order
//                          (descending raster order), capped at 3000 per map
//                          (det_postprocess.cpp:165-167)
//   5. trace_*             border following, CHAIN_APPROX_SIMPLE, count then write
//   6. geom_box1_kernel    size filters and the first min-area box, thread per
//      geom_big_kernel     contour; contours above 96 points take a CTA each
//                          (the lowest and highest point of every x column
//                          gathered with shared-memory atomics, then chain
//                          and rotating calipers over those)
//      score_kernel        polygon-mask mean (box_score_fast,
//                          det_postprocess.cpp:15-55), unclip distance
//   7. unclip_kernel       round-join offset (Clipper's DoOffset), second
//      unclip_big_kernel   min-area box, scale/round/clamp, edge filters;
//                          rings above 96 points again take a CTA each
//                          (vertices offset in parallel)
//   8. compact_kernel      kept boxes in contour order
//
// Node ids: 0 is the outside of map m; pixel p = y*W + x of the map is node
// p+1. A node's parent lives in lab[m*H*W + node-1]. Parents are never larger
// than their node, so every find() walk strictly decreases and ends.
//
// This translation unit is compiled with -fmad=false: the geometry must keep
// the libraries' operation order (explicit fma() only where they contract).
#include <algorithm>
#include <atomic>

#include "tocr_common.cuh"

#include "db_geom.cuh"
#include "clipper_union.cuh"

namespace tocr {
namespace {

using db::HP;
using db::P2;
using db::RRect;

constexpr int kTileW = 32, kTileH = 32, kTilePx = kTileW * kTileH;
constexpr int kMaxCand = 3000;        // det_postprocess.cpp:165
constexpr int kScanThreads = 1024;

// Error bits written to the status word.
constexpr int kErrPointPool = 1;      // traced points exceed the point pool
constexpr int kErrTrace = 2;          // a border walk exceeded its step bound
constexpr int kErrOffsetPool = 4;     // offset points exceed the offset pool
constexpr int kErrBoxes = 8;          // more kept boxes than max_boxes (truncated)
constexpr int kErrUnion = 16;         // a union sweep hit its bounds (raw offset ring used)

struct DbParams {
  int n_maps, H, W;
  float thresh, box_thresh, unclip_ratio, min_box_side, min_unclipped_side;
  long long point_cap, offset_cap;
  int max_boxes;
  int big_cols;                   // widest point set (x columns) the shared-memory path takes
  unsigned long long pool_bytes;  // scratch pool for wider sets
};

// Point sets (contours, unclip rings) above kLocalPts points go to one CTA
// each, reduced to a table of their x columns in shared memory (kBigCols
// columns; the lowest and highest point of each). Wider sets, or hulls above
// kBigHull vertices, fall back to one thread over the global scratch pool.
constexpr int kBigThreads = 512;
constexpr int kBigCols = 6144;
constexpr int kBigHull = 2048;
constexpr size_t kBigTabBytes = sizeof(uint64_t) * 2 * kBigCols;
constexpr size_t kBigStkBytes = sizeof(int) * (2 * kBigCols + 2);
constexpr size_t kBigHullBytes = sizeof(P2) * kBigHull;
constexpr size_t kBigFscBytes = sizeof(float) * 3 * kBigHull;
constexpr size_t kBigSmem = kBigTabBytes + kBigStkBytes + kBigHullBytes + kBigFscBytes;
// the prepared offset path aliases everything after the table
constexpr int kBigQPts = (int)((kBigSmem - kBigTabBytes) / sizeof(P2));
// Scratch pool bytes per point of offset_cap: per unclip the pool holds the
// prepared path, the raw offset ring, the union sweep's arrays (about 200
// bytes per ring point) and the hull work space.
constexpr unsigned long long kPoolBytesPerPoint = 256;
static_assert(kBigSmem <= 227 * 1024, "shared memory of the CTA geometry path");

// Counters of the geometry stages: [0] contour list length, [1] large-ring
// list length, [2..3] pool bytes used (u64), [4] scored-slot list length,
// [5] small-ring list length, [6] next unclip work item.
constexpr int kCounters = 8;

// ---------------------------------------------------------------- union-find --
// Root of v with path halving: each visited node is re-pointed at its
// grandparent. The write only lowers a parent to one of its ancestors (an
// atomicMin, so a smaller link made meanwhile is kept), which leaves every
// node in its set, keeps parents smaller than their nodes and never touches
// a root: "root iff its label is itself" still holds, and union_g re-finds
// roots in its loop.
__device__ __forceinline__ int find_g(int *lab, int v) {
  while (v != 0) {
    const int p = __ldcg(lab + v - 1);
    if (p == v) break;
    if (p == 0) return 0;
    const int g = __ldcg(lab + p - 1);
    if (g != p) atomicMin(lab + v - 1, g);
    v = g;
  }
  return v;
}

__device__ __forceinline__ void union_g(int *lab, int a, int b) {
  for (;;) {
    a = find_g(lab, a);
    b = find_g(lab, b);
    if (a == b) return;
    if (a < b) { const int t = a; a = b; b = t; }
    const int old = atomicMin(lab + a - 1, b);
    if (old == a) return;
    a = old;
  }
}

__device__ __forceinline__ int find_s(volatile int *par, int v) {
  while (v != 0) {
    const int p = par[v - 1];
    if (p == v) break;
    v = p;
  }
  return v;
}

__device__ __forceinline__ void union_s(int *par, int a, int b) {
  for (;;) {
    a = find_s(par, a);
    b = find_s(par, b);
    if (a == b) return;
    if (a < b) { const int t = a; a = b; b = t; }
    const int old = atomicMin(par + a - 1, b);
    if (old == a) return;
    a = old;
  }
}

// 1. threshold (pred non-null; else the bitmap is the input) + tile-local
// labelling, run based: a warp owns a tile row, the
// row's foreground mask is one ballot, and every pixel starts out pointing at
// the first pixel of its same-colour run. Unions are then only made where runs
// of consecutive rows meet: at the first pixel of an overlap (one of the two
// pixels there starts its run), plus the diagonal contacts of foreground runs
// (NW at a run start, NE at a run end). grid (tiles_x, tiles_y, n_maps),
// 256 threads (8 warps x 4 rows).
__global__ void __launch_bounds__(256)
ccl_local_kernel(const float *__restrict__ pred, uint8_t *__restrict__ bitmap, int *__restrict__ lab,
                 uint32_t *__restrict__ bits, uint8_t *__restrict__ root_flag,
                 uint8_t *__restrict__ tile_bg, int H, int W, float thresh) {
  __shared__ unsigned s_fg[kTileH];     // per tile row: foreground bits (bit = lx)
  __shared__ unsigned s_start[kTileH];  // per tile row: run-start bits
  __shared__ int par[kTilePx];
  const int m = blockIdx.z;
  const size_t base = (size_t)m * H * W;
  const int tx0 = blockIdx.x * kTileW, ty0 = blockIdx.y * kTileH;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int x = tx0 + lane;
  const unsigned in_row = (W - tx0 >= 32) ? 0xffffffffu : ((1u << (W - tx0)) - 1u);
  // the warp's four rows of the map are loaded before any is used, so four
  // loads per thread are in flight (one at a time left the kernel far below
  // the memory bandwidth)
  constexpr int kRowsPerWarp = kTileH / 8;
  float pv[kRowsPerWarp];
#pragma unroll
  for (int k = 0; k < kRowsPerWarp; ++k) {
    const int y = ty0 + warp + 8 * k;
    pv[k] = (pred && x < W && y < H) ? pred[base + (size_t)y * W + x] : 0.f;
  }
#pragma unroll
  for (int k = 0; k < kRowsPerWarp; ++k) {
    const int ly = warp + 8 * k;
    const int y = ty0 + ly;
    bool f = false;
    if (x < W && y < H) {
      if (pred) {  // threshold the map; else label the given bitmap
        f = pv[k] > thresh;
        bitmap[base + (size_t)y * W + x] = f ? 255 : 0;
      } else {
        f = bitmap[base + (size_t)y * W + x] != 0;
      }
    }
    const unsigned fg = __ballot_sync(0xffffffffu, f) & in_row;
    // run starts: first pixel of the tile row, or colour differs from the left
    const unsigned diff = (fg ^ (fg << 1)) | 1u;
    const unsigned starts = diff & in_row;
    if (lane == 0) {
      s_fg[ly] = fg;
      s_start[ly] = starts;
      if (bits && y < H) bits[((size_t)m * H + y) * ((W + 31) >> 5) + blockIdx.x] = fg;
    }
    // run start at or left of this lane
    const unsigned upto = starts & (lane == 31 ? 0xffffffffu : ((2u << lane) - 1u));
    const int rs = 31 - __clz(upto);
    par[ly * kTileW + lane] = ly * kTileW + rs + 1;
  }
  // Background-only tile (most of a text page): one 4-connected component,
  // rooted at the outside when the tile touches the image frame, otherwise
  // at the tile's first pixel. No unions needed.
  const bool any_fg = __syncthreads_or(warp < kTileH && lane == 0 &&
                                       (s_fg[warp] | s_fg[warp + 8] | s_fg[warp + 16] |
                                        s_fg[warp + 24]) != 0u);
  if (tile_bg) {
    if (threadIdx.x == 0) tile_bg[((size_t)m * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x] = !any_fg;
  }
  if (!any_fg) {
    const bool frame = tx0 == 0 || ty0 == 0 || tx0 + kTileW >= W || ty0 + kTileH >= H;
    const int g = frame ? 0 : ty0 * W + tx0 + 1;
    for (int ly = warp; ly < kTileH; ly += 8) {
      const int y = ty0 + ly;
      if (x >= W || y >= H) continue;
      lab[base + (size_t)y * W + x] = g;
      if (root_flag) root_flag[base + (size_t)y * W + x] = (!frame && ly == 0 && lane == 0) ? 1 : 0;
    }
    return;
  }
  for (int ly = warp; ly < kTileH; ly += 8) {
    const int y = ty0 + ly;
    if (x >= W || y >= H) continue;
    const unsigned fg = s_fg[ly], st = s_start[ly];
    const bool f = (fg >> lane) & 1u;
    const bool is_start = (st >> lane) & 1u;
    const bool is_end = lane == 31 || x == W - 1 || (((st >> (lane + 1)) & 1u) != 0);
    const int me = ly * kTileW + lane + 1;
    if (ly > 0) {
      const unsigned fu = s_fg[ly - 1], su = s_start[ly - 1];
      const bool fn = (fu >> lane) & 1u;
      if (fn == f && (is_start || ((su >> lane) & 1u))) union_s(par, me, me - kTileW);
      if (f) {
        if (is_start && lane > 0 && ((fu >> (lane - 1)) & 1u)) union_s(par, me, me - kTileW - 1);
        if (is_end && lane < 31 && x + 1 < W && ((fu >> (lane + 1)) & 1u))
          union_s(par, me, me - kTileW + 1);
      }
    }
    if (!f && (((y == 0 || y == H - 1) && is_start) || x == 0 || x == W - 1)) union_s(par, me, 0);
  }
  __syncthreads();
  // pointer jumping until every node points at its root (vertical stacks of
  // runs form chains up to a tile high; at most log2(1024) rounds)
  for (int round = 0; round < 11; ++round) {
    int changed = 0;
    for (int i = threadIdx.x; i < kTilePx; i += blockDim.x) {
      const int p1 = par[i];
      if (p1 != 0) {
        const int p2 = par[p1 - 1];
        if (p2 != p1) { par[i] = p2; changed = 1; }
      }
    }
    if (!__syncthreads_or(changed)) break;
  }
  for (int ly = warp; ly < kTileH; ly += 8) {
    const int y = ty0 + ly;
    if (x >= W || y >= H) continue;
    const int r = find_s(par, ly * kTileW + lane + 1);
    int g = 0;
    if (r != 0) {
      const int rl = r - 1;
      g = (ty0 + rl / kTileW) * W + tx0 + rl % kTileW + 1;
    }
    lab[base + (size_t)y * W + x] = g;
    if (root_flag) root_flag[base + (size_t)y * W + x] = (r == ly * kTileW + lane + 1) ? 1 : 0;
  }
}

// 2. unions across tile borders. One thread per pixel of a tile's first row,
// first column or last column. grid (tiles_x, tiles_y, n_maps), 128 threads.
__global__ void __launch_bounds__(128)
ccl_merge_kernel(const uint8_t *__restrict__ bitmap, int *__restrict__ lab,
                 const uint8_t *__restrict__ tile_bg, int H, int W) {
  const int m = blockIdx.z;
  const size_t base = (size_t)m * H * W;
  const uint8_t *bm = bitmap + base;
  int *lb = lab + base;
  const int tx0 = blockIdx.x * kTileW, ty0 = blockIdx.y * kTileH;
  if (tile_bg) {
    // background-only tile: its single component meets each background-only
    // neighbour along a whole edge, so one union per such neighbour suffices
    const size_t tb = (size_t)m * gridDim.y * gridDim.x;
    const bool me_bg = tile_bg[tb + (size_t)blockIdx.y * gridDim.x + blockIdx.x];
    if (me_bg) {
      // This tile only links upward and leftward (its right neighbour links
      // to it from its own left edge, the tile below from its top row), and a
      // background-only tile has no foreground diagonals to follow.
      const bool has_up = blockIdx.y > 0, has_left = blockIdx.x > 0;
      const bool up_bg = has_up && tile_bg[tb + (size_t)(blockIdx.y - 1) * gridDim.x + blockIdx.x];
      const bool left_bg = has_left && tile_bg[tb + (size_t)blockIdx.y * gridDim.x + blockIdx.x - 1];
      if ((!has_up || up_bg) && (!has_left || left_bg)) {
        if (threadIdx.x == 0) {
          const int me = ty0 * W + tx0 + 1;
          if (has_up) union_g(lb, me, me - W);
          if (has_left) union_g(lb, me, me - 1);
        }
        return;
      }
    }
  }
  // border pixels: top row (kTileW), left column (kTileH), right column (kTileH)
  for (int i = threadIdx.x; i < kTileW + 2 * kTileH; i += blockDim.x) {
    int lx, ly;
    if (i < kTileW) { lx = i; ly = 0; }
    else if (i < kTileW + kTileH) { lx = 0; ly = i - kTileW; }
    else { lx = kTileW - 1; ly = i - kTileW - kTileH; }
    const int x = tx0 + lx, y = ty0 + ly;
    if (x >= W || y >= H) continue;
    const int p = y * W + x, me = p + 1;
    const bool f = bm[p] != 0;
    auto other_tile = [&](int nx, int ny) {
      return nx / kTileW != blockIdx.x || ny / kTileH != blockIdx.y;
    };
    if (f) {
      const int nb[4][2] = {{x - 1, y}, {x - 1, y - 1}, {x, y - 1}, {x + 1, y - 1}};
      for (int k = 0; k < 4; ++k) {
        const int nx = nb[k][0], ny = nb[k][1];
        if (nx < 0 || ny < 0 || nx >= W) continue;
        if (!other_tile(nx, ny)) continue;
        if (bm[ny * W + nx]) union_g(lb, me, ny * W + nx + 1);
      }
    } else {
      const int nb[2][2] = {{x - 1, y}, {x, y - 1}};
      for (int k = 0; k < 2; ++k) {
        const int nx = nb[k][0], ny = nb[k][1];
        if (nx < 0 || ny < 0) continue;
        if (!other_tile(nx, ny)) continue;
        if (!bm[ny * W + nx]) union_g(lb, me, ny * W + nx + 1);
      }
    }
  }
}

// 2b. compression of the tile-local roots (flagged by stage 1), so that
// stage 3 reaches a root in at most two hops. grid (tiles_x, tiles_y,
// n_maps), 256 threads.
__global__ void __launch_bounds__(256)
ccl_roots_kernel(int *__restrict__ lab, const uint8_t *__restrict__ root_flag, int H, int W) {
  const int m = blockIdx.z;
  int *lb = lab + (size_t)m * H * W;
  const uint8_t *rf = root_flag + (size_t)m * H * W;
  const int tx0 = blockIdx.x * kTileW, ty0 = blockIdx.y * kTileH;
  for (int l = threadIdx.x; l < kTilePx; l += blockDim.x) {
    const int x = tx0 + (l % kTileW), y = ty0 + (l / kTileW);
    if (x >= W || y >= H) continue;
    const int p = y * W + x;
    if (!rf[p]) continue;
    const int r = find_g(lb, p + 1);
    if (r != p + 1) atomicMin(lb + p, r);
  }
}

// 3. compression + starts per row. A start is a pixel that is its own root:
// a foreground root starts an outer border at itself, a background root (not
// joined to the outside) starts a hole border at the pixel on its left.
// grid (H, n_maps), 256 threads.
__global__ void __launch_bounds__(256)
ccl_rows_kernel(int *__restrict__ lab, int *__restrict__ row_count, int H, int W, bool compress) {
  const int m = blockIdx.y, y = blockIdx.x;
  int *lb = lab + (size_t)m * H * W;
  __shared__ int s_total;
  if (threadIdx.x == 0) s_total = 0;
  __syncthreads();
  int cnt = 0;
  for (int x = threadIdx.x; x < W; x += blockDim.x) {
    const int p = y * W + x;
    // A pixel starts a border iff it is the root of its component. Without
    // compression that is still exactly "its label is itself": labels only
    // ever point at smaller nodes, and a tile root that a merge relinked holds
    // the smaller node it was linked to.
    int r = lb[p];
    if (compress) {
      r = find_g(lb, r);
      lb[p] = r;
    }
    cnt += (r == p + 1);
  }
  for (int off = 16; off; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
  if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&s_total, cnt);
  __syncthreads();
  if (threadIdx.x == 0 && row_count) row_count[(size_t)m * H + y] = s_total;
}

// 4a. per map: offsets of each row's starts in descending raster order.
// grid n_maps, kScanThreads threads.
__global__ void __launch_bounds__(kScanThreads)
starts_scan_kernel(const int *__restrict__ row_count, int *__restrict__ row_off,
                   int *__restrict__ n_contours, int *__restrict__ n_total, int H,
                   int *__restrict__ ovf_count) {
  const int m = blockIdx.x;
  if (m == 0 && threadIdx.x == 0) *ovf_count = 0;  // overflow chunks of trace_kernel
  const int *rc = row_count + (size_t)m * H;
  int *ro = row_off + (size_t)m * H;
  __shared__ int s_part[kScanThreads];
  __shared__ int s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  // descending rows: row H-1 first
  for (int c0 = 0; c0 < H; c0 += kScanThreads) {
    const int i = c0 + threadIdx.x;
    const int y = H - 1 - i;
    const int v = (i < H) ? rc[y] : 0;
    s_part[threadIdx.x] = v;
    __syncthreads();
    for (int off = 1; off < kScanThreads; off <<= 1) {
      const int t = (threadIdx.x >= off) ? s_part[threadIdx.x - off] : 0;
      __syncthreads();
      s_part[threadIdx.x] += t;
      __syncthreads();
    }
    if (i < H) ro[y] = s_carry + s_part[threadIdx.x] - v;
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) s_carry += s_part[threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    n_total[m] = s_carry;
    n_contours[m] = s_carry < kMaxCand ? s_carry : kMaxCand;
  }
}

// 4b. start records, packed as (pixel index << 1) | hole, at
// starts[m * 3000 + rank]. grid (H, n_maps), 256 threads.
__global__ void __launch_bounds__(256)
starts_write_kernel(const int *__restrict__ lab, const uint8_t *__restrict__ bitmap,
                    const int *__restrict__ row_count, const int *__restrict__ row_off,
                    int *__restrict__ starts, int H, int W) {
  const int m = blockIdx.y, y = blockIdx.x;
  const int rcount = row_count[(size_t)m * H + y];
  if (rcount == 0) return;
  const int roff = row_off[(size_t)m * H + y];
  if (roff >= kMaxCand) return;
  const int *lb = lab + (size_t)m * H * W;
  const uint8_t *bm = bitmap + (size_t)m * H * W;
  __shared__ int s_warp[8];
  __shared__ int s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int x0 = 0; x0 < W; x0 += blockDim.x) {
    const int x = x0 + threadIdx.x;
    const int p = y * W + x;
    const bool st = x < W && lb[p] == p + 1;
    const unsigned bal = __ballot_sync(0xffffffffu, st);
    if (lane == 0) s_warp[warp] = __popc(bal);
    __syncthreads();
    int before = s_carry;
    for (int w = 0; w < warp; ++w) before += s_warp[w];
    const int asc = before + __popc(bal & ((1u << lane) - 1));
    if (st) {
      const int rank = roff + (rcount - 1 - asc);
      if (rank < kMaxCand) {
        const bool hole = bm[p] == 0;
        const int sp = hole ? p - 1 : p;
        starts[(size_t)m * kMaxCand + rank] = (sp << 1) | (hole ? 1 : 0);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_warp[w];
      s_carry += t;
    }
    __syncthreads();
  }
}


// 5. border following. One thread per contour slot (m * 3000 + rank): the
// walk writes its first kSlab points into the slot's slab, the rest into
// chunks of kChunk points taken from a shared overflow pool and linked per
// contour (ovf_first[c], ovf_next[chunk]), and counts them all (npts). After
// the offsets are scanned, gather_kernel copies slab and chunks to the
// contiguous point pool. When the overflow pool runs out, that contour is
// walked a second time straight into the point pool instead.
constexpr int kSlab = 256;
constexpr int kChunk = 1024;
constexpr int kOvfNone = -1, kOvfFailed = -2;

__device__ __forceinline__ int trace_max_steps(int H, int W) {
  const long long ms = 4ll * H * W + 16;
  return ms > 0x7fffffffll ? 0x7fffffff : (int)ms;
}

__global__ void __launch_bounds__(128)
trace_kernel(const uint32_t *__restrict__ bits, const int *__restrict__ starts,
             const int *__restrict__ n_contours, int *__restrict__ npts, P2 *__restrict__ slab,
             int *__restrict__ ovf_first, int *__restrict__ ovf_next, P2 *__restrict__ ovf_pts,
             int *__restrict__ ovf_count, int ovf_chunks, int *__restrict__ status, int n_maps,
             int H, int W) {
  const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (long long)n_maps * kMaxCand) return;
  const int m = (int)(c / kMaxCand), rank = (int)(c % kMaxCand);
  if (rank >= n_contours[m]) {
    npts[c] = 0;
    return;
  }
  const int rec = starts[c];
  const int sp = rec >> 1;
  const int words = (W + 31) >> 5;
  db::NbBits nb{bits + (size_t)m * H * words, H, W, words};
  P2 *sl = slab + c * kSlab;
  int k = 0, first = kOvfNone, chunk = -1, fill = kChunk;
  const int n = db::trace_border_emit(
      nb, sp % W, sp / W, (rec & 1) != 0,
      [&](int x, int y) {
        if (k < kSlab) {
          sl[k] = P2{x, y};
        } else if (first != kOvfFailed) {
          if (fill == kChunk) {
            const int nc = atomicAdd(ovf_count, 1);
            if (nc >= ovf_chunks) {
              first = kOvfFailed;
            } else {
              ovf_next[nc] = -1;
              if (chunk < 0) first = nc;
              else ovf_next[chunk] = nc;
              chunk = nc;
              fill = 0;
            }
          }
          if (first != kOvfFailed) ovf_pts[(size_t)chunk * kChunk + fill++] = P2{x, y};
        }
        ++k;
      },
      trace_max_steps(H, W));
  if (n < 0) atomicOr(status, kErrTrace);
  npts[c] = n < 0 ? 0 : n;
  ovf_first[c] = first;
}

// One warp per contour slot: slab and overflow chunks -> pool (lanes copy),
// or a second walk when the overflow pool ran out.
__global__ void __launch_bounds__(128)
gather_kernel(const uint32_t *__restrict__ bits, const int *__restrict__ starts,
              const int *__restrict__ npts, const long long *__restrict__ pt_off,
              const P2 *__restrict__ slab, const int *__restrict__ ovf_first,
              const int *__restrict__ ovf_next, const P2 *__restrict__ ovf_pts,
              P2 *__restrict__ pts, long long point_cap, int n_maps, int H, int W) {
  const long long c = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (c >= (long long)n_maps * kMaxCand) return;
  const int n = npts[c];
  if (n == 0 || pt_off[c] + n > point_cap) return;
  P2 *dst = pts + pt_off[c];
  const int first = ovf_first[c];
  if (n <= kSlab || first != kOvfFailed) {
    const int ns = n < kSlab ? n : kSlab;
    for (int i = lane; i < ns; i += 32) dst[i] = slab[c * kSlab + i];
    int ch = first;
    for (int done = kSlab; done < n; done += kChunk) {
      const int cnt = n - done < kChunk ? n - done : kChunk;
      for (int i = lane; i < cnt; i += 32) dst[done + i] = ovf_pts[(size_t)ch * kChunk + i];
      ch = ovf_next[ch];
    }
    return;
  }
  if (lane != 0) return;
  const int m = (int)(c / kMaxCand);
  const int rec = starts[c];
  const int sp = rec >> 1;
  const int words = (W + 31) >> 5;
  db::NbBits nb{bits + (size_t)m * H * words, H, W, words};
  db::trace_border_nb(nb, sp % W, sp / W, (rec & 1) != 0, dst, n, trace_max_steps(H, W));
}

// Exclusive scan of the per-slot counts of n_maps x 3000 contour slots into
// int64 offsets (out[n] = total), two passes: a per-map scan (one CTA per
// map, warp shuffles) that leaves the map's total in tot[m], then the map
// bases added in place.
__device__ __forceinline__ long long warp_incl_scan(long long v, int lane) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long t = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += t;
  }
  return v;
}

template <class T>
__global__ void __launch_bounds__(kScanThreads)
scan_map_kernel(const T *__restrict__ in, long long *__restrict__ out, long long *__restrict__ tot) {
  __shared__ long long s_warp[kScanThreads / 32];
  __shared__ long long s_carry;
  const int m = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long base = (long long)m * kMaxCand;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (int c0 = 0; c0 < kMaxCand; c0 += kScanThreads) {
    const int i = c0 + threadIdx.x;
    const long long v = i < kMaxCand ? (long long)in[base + i] : 0;
    const long long incl = warp_incl_scan(v, lane);
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const long long w = lane < kScanThreads / 32 ? s_warp[lane] : 0;
      const long long wi = warp_incl_scan(w, lane);
      if (lane < kScanThreads / 32) s_warp[lane] = wi - w;  // exclusive warp offsets
    }
    __syncthreads();
    if (i < kMaxCand) out[base + i] = s_carry + s_warp[warp] + incl - v;
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) s_carry += s_warp[warp] + incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) tot[m] = s_carry;
}

__global__ void __launch_bounds__(kScanThreads)
scan_base_kernel(long long *__restrict__ out, const long long *__restrict__ tot, int n_maps) {
  __shared__ long long s_base;
  const int m = blockIdx.x;
  if (threadIdx.x == 0) {
    long long b = 0;
    for (int k = 0; k < m; ++k) b += tot[k];
    s_base = b;
    if (m == n_maps - 1) out[(long long)n_maps * kMaxCand] = b + tot[m];
  }
  __syncthreads();
  const long long base = (long long)m * kMaxCand;
  for (int i = threadIdx.x; i < kMaxCand; i += kScanThreads) out[base + i] += s_base;
}

// Point-pool check; also zeroes the CTA geometry path's counters.
__global__ void prep_geom_kernel(const long long *__restrict__ off, long long n, long long cap,
                                 int *__restrict__ status, int *__restrict__ counters) {
  if (off[n] > cap) atomicOr(status, kErrPointPool);
  for (int i = 0; i < kCounters; ++i) counters[i] = 0;
}

// min-area rectangle of a small point set (n <= kLocalPts) in thread-local
// arrays (cached in L1, write-back).
constexpr int kLocalPts = 96;

__device__ RRect rect_local(const P2 *p, int n) {
  HP lw[2 * kLocalPts + 2];
  P2 lh[kLocalPts + 1];
  float lf[3 * kLocalPts + 3];
  const int h = db::convex_hull(p, n, lw, lh);
  return db::min_area_rect(lh, h, lf);
}

__device__ char *pool_alloc(char *pool, int *counters, unsigned long long pool_bytes,
                            unsigned long long bytes, int *status) {
  bytes = (bytes + 15) & ~15ull;
  auto *used = reinterpret_cast<unsigned long long *>(counters + 2);
  const unsigned long long at = atomicAdd(used, bytes);
  if (at + bytes > pool_bytes) {
    atomicOr(status, kErrOffsetPool);
    return nullptr;
  }
  return pool + at;
}

// One thread, global scratch: the min-area rectangle of p[0..n) for sets the
// shared-memory path cannot take. False when the pool is exhausted.
__device__ bool rect_global(const P2 *p, int n, char *pool, int *counters,
                            unsigned long long pool_bytes, int *status, RRect *r) {
  const unsigned long long hp = ((2ull * n + 1) * sizeof(HP) + 15) & ~15ull;
  const unsigned long long hl = ((n + 1ull) * sizeof(P2) + 15) & ~15ull;
  char *w = pool_alloc(pool, counters, pool_bytes, hp + hl + 12ull * (n + 1), status);
  if (!w) return false;
  P2 *hull = reinterpret_cast<P2 *>(w + hp);
  const int h = db::convex_hull(p, n, reinterpret_cast<HP *>(w), hull);
  *r = db::min_area_rect(hull, h, reinterpret_cast<float *>(w + hp + hl));
  return true;
}

// 6a. one thread per contour slot: the filters before the score
// (det_postprocess.cpp:169-186): more than 2 points, boundingRect sides >= 3,
// first min-area box side >= min_box_side. Survivors get their AABB.
// Contours above kLocalPts points are listed for geom_big_kernel.
__global__ void __launch_bounds__(128)
geom_box1_kernel(const int *__restrict__ n_contours, const int *__restrict__ npts,
                 const long long *__restrict__ pt_off, const P2 *__restrict__ pts,
                 int *__restrict__ stage1, int4 *__restrict__ aabb, int *__restrict__ list,
                 int *__restrict__ counters, int *__restrict__ score_done,
                 int *__restrict__ score_list, int *__restrict__ stage2,
                 int *__restrict__ keep2, DbParams P) {
  const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (long long)P.n_maps * kMaxCand) return;
  stage1[c] = 0;
  stage2[c] = 0;
  keep2[c] = 0;
  score_done[c] = 0;
  const int m = (int)(c / kMaxCand), rank = (int)(c % kMaxCand);
  const int n = npts[c];
  if (rank >= n_contours[m] || n <= 2 || pt_off[c] + n > P.point_cap) return;
  const P2 *p = pts + pt_off[c];
  int xmin = p[0].x, xmax = p[0].x, ymin = p[0].y, ymax = p[0].y;
  for (int i = 1; i < n; ++i) {
    xmin = min(xmin, p[i].x); xmax = max(xmax, p[i].x);
    ymin = min(ymin, p[i].y); ymax = max(ymax, p[i].y);
  }
  if (xmax - xmin + 1 < 3 || ymax - ymin + 1 < 3) return;
  aabb[c] = make_int4(xmin, ymin, xmax, ymax);
  if (n > kLocalPts) {
    list[atomicAdd(counters, 1)] = (int)c;
    return;
  }
  const RRect r = rect_local(p, n);
  if ((r.w < r.h ? r.w : r.h) < P.min_box_side) return;
  stage1[c] = 1;
  score_list[atomicAdd(counters + 4, 1)] = (int)c;
}

// ---- CTA geometry: one point set per CTA, all in shared memory ----------
struct BigSmem {
  unsigned long long *lo, *hi;  // column table
  int *stk;
  P2 *hull;
  float *fsc;
  P2 *q;  // aliases stk .. fsc (dead once the ring is in the table)
};

__device__ __forceinline__ BigSmem big_smem(uint8_t *base) {
  BigSmem b;
  b.lo = reinterpret_cast<unsigned long long *>(base);
  b.hi = b.lo + kBigCols;
  b.stk = reinterpret_cast<int *>(base + kBigTabBytes);
  b.hull = reinterpret_cast<P2 *>(base + kBigTabBytes + kBigStkBytes);
  b.fsc = reinterpret_cast<float *>(base + kBigTabBytes + kBigStkBytes + kBigHullBytes);
  b.q = reinterpret_cast<P2 *>(base + kBigTabBytes);
  return b;
}

__device__ __forceinline__ void table_clear(const BigSmem &S, int ncols) {
  for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
    S.lo[c] = db::kColEmpty;
    S.hi[c] = db::kColEmpty;
  }
}

__device__ __forceinline__ void table_add(const BigSmem &S, int c, int y, int idx) {
  atomicMin(S.lo + c, (unsigned long long)db::col_lo_key(y, idx));
  atomicMin(S.hi + c, (unsigned long long)db::col_hi_key(y, idx));
}

// Inclusive sum of v over the CTA (kBigThreads threads); *total gets the sum.
__device__ int cta_inclusive_sum(int v, int *total) {
  __shared__ int s_w[kBigThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_w[wid] = x;
  __syncthreads();
  int base = 0, all = 0;
  for (int w = 0; w < kBigThreads / 32; ++w) {
    if (w < wid) base += s_w[w];
    all += s_w[w];
  }
  __syncthreads();
  *total = all;
  return base + x;
}

// min-area rectangle from the filled table (synchronised) of ncols columns at
// x = base + c. The CTA first finds the extreme candidates of kExtDirs
// directions and drops the candidates strictly inside their polygon; thread
// 0 then chains the rest. False (on every thread) when the hull exceeds
// kBigHull vertices; *r is valid in thread 0.
__device__ bool cta_table_rect(const BigSmem &S, int ncols, int base, RRect *r) {
  __shared__ int s_ok;
  __shared__ unsigned long long s_ext[db::kExtDirs];
  __shared__ HP s_poly[db::kExtDirs];
  __shared__ uint32_t s_keep[(2 * kBigCols + 31) / 32];
  const uint64_t *lo = reinterpret_cast<const uint64_t *>(S.lo);
  const uint64_t *hi = reinterpret_cast<const uint64_t *>(S.hi);
  const int ns = 2 * ncols;
  if (threadIdx.x < db::kExtDirs) s_ext[threadIdx.x] = 0ull;
  __syncthreads();
  {  // extreme candidate of each direction: max of (dot + 2^31) << 32 | entry
    unsigned long long best[db::kExtDirs];
#pragma unroll
    for (int k = 0; k < db::kExtDirs; ++k) best[k] = 0ull;
    HP v;
    for (int e = threadIdx.x; e < ns; e += blockDim.x) {
      if (!db::col_entry(lo, hi, base, e, &v)) continue;
#pragma unroll
      for (int k = 0; k < db::kExtDirs; ++k) {
        const unsigned long long key =
            ((unsigned long long)(db::ext_dot(k, v.x, v.y) + (1ll << 31)) << 32) | (unsigned)e;
        best[k] = key > best[k] ? key : best[k];
      }
    }
#pragma unroll
    for (int k = 0; k < db::kExtDirs; ++k) {
      unsigned long long b = best[k];
      for (int o = 16; o; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
        b = t > b ? t : b;
      }
      if ((threadIdx.x & 31) == 0 && b) atomicMax(s_ext + k, b);
    }
  }
  __syncthreads();
  if (threadIdx.x < db::kExtDirs) {
    HP v{0, 0, 0};
    db::col_entry(lo, hi, base, (int)(s_ext[threadIdx.x] & 0xffffffffu), &v);
    s_poly[threadIdx.x] = v;
  }
  __syncthreads();
  {  // keep mask, one warp per 32 entries
    const int lane = threadIdx.x & 31;
    for (int w = threadIdx.x >> 5; w * 32 < ns; w += blockDim.x >> 5) {
      const int e = w * 32 + lane;
      HP v;
      const bool keep = e < ns && db::col_entry(lo, hi, base, e, &v) &&
                        !db::strictly_inside_extremes(s_poly, db::kExtDirs, v);
      const unsigned bits = __ballot_sync(0xffffffffu, keep);
      if (lane == 0) s_keep[w] = bits;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int m = db::hull_from_table(lo, hi, ncols, base, S.stk, S.hull, kBigHull, s_keep);
    s_ok = m >= 0;
    if (m >= 0) *r = db::min_area_rect(S.hull, m, S.fsc);
  }
  __syncthreads();
  return s_ok != 0;
}

// 6a'. one CTA per listed contour (grid-stride): its first min-area box.
__global__ void __launch_bounds__(kBigThreads)
geom_big_kernel(const int *__restrict__ list, const int *__restrict__ counters,
                const int *__restrict__ npts, const long long *__restrict__ pt_off,
                const P2 *__restrict__ pts, const int4 *__restrict__ aabb,
                int *__restrict__ stage1, int *__restrict__ score_list, char *__restrict__ pool,
                int *__restrict__ pool_counters, int *__restrict__ status, DbParams P) {
  extern __shared__ __align__(16) uint8_t smem[];
  const BigSmem S = big_smem(smem);
  const int count = counters[0];
  for (int li = blockIdx.x; li < count; li += gridDim.x) {
    const int c = list[li];
    const int n = npts[c];
    const P2 *p = pts + pt_off[c];
    const int4 bb = aabb[c];
    const int base = bb.x, ncols = bb.z - bb.x + 1;
    RRect r{};
    bool ok = false;
    if (ncols <= P.big_cols) {
      table_clear(S, ncols);
      __syncthreads();
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const P2 v = p[i];
        table_add(S, v.x - base, v.y, i);
      }
      __syncthreads();
      ok = cta_table_rect(S, ncols, base, &r);
    }
    if (threadIdx.x == 0) {
      if (!ok) ok = rect_global(p, n, pool, pool_counters, P.pool_bytes, status, &r);
      if (ok && (r.w < r.h ? r.w : r.h) >= P.min_box_side) {
        stage1[c] = 1;
        score_list[atomicAdd(pool_counters + 4, 1)] = c;
      }
    }
    __syncthreads();
  }
}

constexpr int kScoreThreads = 256;
constexpr int kBandRows = 32;
constexpr int kMaxWords = 128;  // AABB widths up to 4096 px

__device__ __forceinline__ void fill_bits(unsigned *row, int a, int b) {
  // set bits [a, b] (inclusive, already clipped, a <= b)
  int w0 = a >> 5, w1 = b >> 5;
  for (int w = w0; w <= w1; ++w) {
    const int lo = (w == w0) ? (a & 31) : 0, hi = (w == w1) ? (b & 31) : 31;
    const unsigned mask = (hi == 31 ? 0xffffffffu : ((1u << (hi + 1)) - 1u)) & ~((1u << lo) - 1u);
    atomicOr(row + w, mask);
  }
}

// 6b. box_score_fast: the mean of pred over the filled contour (edge pixels
// plus odd-parity interior) inside its AABB, accumulated in double; then the
// unclip distance area * ratio / perimeter (det_postprocess.cpp:59-66).
// grid (x, kScoreGroups): the x CTAs stride over the list of slots that
// passed the first filters (score_list) and CTA group g takes the slot's
// 32-row bands g, g + G, ... so
// that a large contour is summed by G CTAs at once. Each group leaves its
// partial sum (only groups that own a band take part); the last group to
// finish a slot (counter done[c]) adds the partials in group order
// (deterministic) and writes the score.
constexpr int kScoreGroups = 8;

__global__ void __launch_bounds__(kScoreThreads)
score_kernel(const float *__restrict__ pred, const int *__restrict__ score_list,
             int *__restrict__ counters, const int4 *__restrict__ aabb, const int *__restrict__ npts,
             const long long *__restrict__ pt_off, const P2 *__restrict__ pts,
             int *__restrict__ stage2, float *__restrict__ score, double *__restrict__ dist,
             double *__restrict__ part_sum, long long *__restrict__ part_cnt,
             int *__restrict__ done, int *__restrict__ ring_list, DbParams P) {
  __shared__ unsigned s_edge[kBandRows][kMaxWords];
  __shared__ unsigned s_tog[kBandRows][kMaxWords];
  __shared__ double s_sum[kScoreThreads / 32];
  __shared__ long long s_cnt[kScoreThreads / 32];
  __shared__ int s_last;
  const int g = blockIdx.y;
  const int count = counters[4];
  for (int li = blockIdx.x; li < count; li += gridDim.x) {
  const long long c = score_list[li];
  const int m = (int)(c / kMaxCand);
  const int H = P.H, W = P.W;
  const int n = npts[c];
  const P2 *p = pts + pt_off[c];
  const int4 bb = aabb[c];
  const int bx0 = max(0, bb.x), by0 = max(0, bb.y), bx1 = min(W - 1, bb.z), by1 = min(H - 1, bb.w);
  double sum = 0.;
  long long cnt = 0;
  const bool nonempty = bx1 > bx0 && by1 > by0;
  // groups that own a band take part (at least group 0)
  const int bands = nonempty ? (by1 - by0) / kBandRows + 1 : 1;
  const int groups = bands < kScoreGroups ? bands : kScoreGroups;
  if (g >= groups) continue;
  if (nonempty) {
    const int width = bx1 - bx0 + 1, words = (width + 31) >> 5;
    const float *pm = pred + (size_t)m * H * W;
    for (int band = by0 + g * kBandRows; band <= by1; band += kScoreGroups * kBandRows) {
      const int rows = min(kBandRows, by1 - band + 1);
      for (int i = threadIdx.x; i < kBandRows * words; i += kScoreThreads) {
        s_edge[i / words][i % words] = 0u;
        s_tog[i / words][i % words] = 0u;
      }
      __syncthreads();
      // edge-major: every thread takes edges and marks the rows of this band
      // they cover (contour edges are horizontal, vertical or diagonal)
      for (int i = threadIdx.x; i < n; i += kScoreThreads)
        db::poly_edge_marks(p[i], p[(i + 1 < n) ? i + 1 : 0], band, band + rows - 1,
            [&](int y, int a, int b) {
              if (a > b) { const int t = a; a = b; b = t; }
              a = max(a, bx0); b = min(b, bx1);
              if (a <= b) fill_bits(s_edge[y - band], a - bx0, b - bx0);
            },
            [&](int y, int x) {
              if (x >= bx0 && x <= bx1)
                atomicXor(&s_tog[y - band][(x - bx0) >> 5], 1u << ((x - bx0) & 31));
            });
      __syncthreads();
      if (threadIdx.x < rows) {
        const int r = threadIdx.x;
        unsigned carry = 0u;
        for (int k = 0; k < words; ++k) {
          unsigned t = s_tog[r][k];
          t ^= t << 1; t ^= t << 2; t ^= t << 4; t ^= t << 8; t ^= t << 16;  // inclusive prefix parity
          const unsigned par = carry ? ~t : t;
          carry = par >> 31;
          s_edge[r][k] |= par;
        }
        const int tail = width & 31;
        if (tail) s_edge[r][words - 1] &= (1u << tail) - 1u;
      }
      __syncthreads();
      // a warp per (row, 32-pixel word) of the mask, four words in flight
      // per warp: coalesced row reads, empty words skipped
      {
        const int lane = threadIdx.x & 31;
        constexpr int kWarps = kScoreThreads / 32, kUnroll = 4;
        const int total = rows * words;
        for (int k0 = threadIdx.x >> 5; k0 < total; k0 += kWarps * kUnroll) {
          float v[kUnroll];
          bool on[kUnroll];
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int k = k0 + u * kWarps;
            on[u] = false;
            v[u] = 0.f;
            if (k < total) {
              const int r = k / words, wd = k - r * words;
              on[u] = (s_edge[r][wd] >> lane) & 1u;
              if (on[u]) v[u] = pm[(size_t)(band + r) * W + bx0 + (wd << 5) + lane];
            }
          }
#pragma unroll
          for (int u = 0; u < kUnroll; ++u)
            if (on[u]) { sum += (double)v[u]; ++cnt; }
        }
      }
      __syncthreads();
    }
  }
  for (int off = 16; off; off >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, off);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
  }
  if ((threadIdx.x & 31) == 0) {
    s_sum[threadIdx.x >> 5] = sum;
    s_cnt[threadIdx.x >> 5] = cnt;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double tsum = 0.;
    long long tcnt = 0;
    for (int w = 0; w < kScoreThreads / 32; ++w) { tsum += s_sum[w]; tcnt += s_cnt[w]; }
    part_sum[c * kScoreGroups + g] = tsum;
    part_cnt[c * kScoreGroups + g] = tcnt;
    __threadfence();
    s_last = atomicAdd(done + c, 1) == groups - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    double tsum = 0.;
    long long tcnt = 0;
    for (int k = 0; k < groups; ++k) {
      tsum += __ldcg(part_sum + c * kScoreGroups + k);
      tcnt += __ldcg(part_cnt + c * kScoreGroups + k);
    }
    const float sc = (nonempty && tcnt > 0) ? (float)(tsum / (double)tcnt) : 0.f;
    score[c] = sc;
    stage2[c] = 0;
    if (sc >= P.box_thresh) {
      const double per = db::arc_length(p, n);
      // unclip returns the contour itself when the perimeter is 0 (distance 0 here)
      dist[c] = per != 0. ? db::contour_area(p, n) * (double)P.unclip_ratio / per : 0.;
      stage2[c] = 1;
      // unclip work list: large contours from the front, small ones from the back
      if (n > kLocalPts) ring_list[atomicAdd(counters + 1, 1)] = (int)c;
      else ring_list[(long long)P.n_maps * kMaxCand - 1 - atomicAdd(counters + 5, 1)] = (int)c;
    }
  }
  __syncthreads();
  }
}

// Second min-area box -> quad in the original image, filters
// (det_postprocess.cpp:200-219).
__device__ void finish_box(const RRect &rr, long long c, const int *geo, int *keep2, int *boxes,
                           const DbParams &P) {
  if ((rr.w < rr.h ? rr.w : rr.h) < P.min_unclipped_side) return;
  int box[8];
  db::mini_box(rr, box);
  const int m = (int)(c / kMaxCand);
  int orig_h = P.H, orig_w = P.W, res_h = P.H, res_w = P.W;
  if (geo) {
    orig_h = geo[4 * m]; orig_w = geo[4 * m + 1]; res_h = geo[4 * m + 2]; res_w = geo[4 * m + 3];
  }
  const float ratio_h = (float)res_h / (float)orig_h;
  const float ratio_w = (float)res_w / (float)orig_w;
  for (int k = 0; k < 4; ++k) {
    const int bx = db::round_half_away((float)box[2 * k] / ratio_w);
    const int by = db::round_half_away((float)box[2 * k + 1] / ratio_h);
    box[2 * k] = bx < 0 ? 0 : (bx > orig_w - 1 ? orig_w - 1 : bx);
    box[2 * k + 1] = by < 0 ? 0 : (by > orig_h - 1 ? orig_h - 1 : by);
  }
  const int dx01 = box[0] - box[2], dy01 = box[1] - box[3];
  const int dx03 = box[0] - box[6], dy03 = box[1] - box[7];
  const int rw = (int)sqrt((double)(dx01 * dx01 + dy01 * dy01));
  const int rh = (int)sqrt((double)(dx03 * dx03 + dy03 * dy03));
  if (rw <= 3 || rh <= 3) return;
  for (int k = 0; k < 8; ++k) boxes[c * 8 + k] = box[k];
  keep2[c] = 1;
}

// True when the prepared path is an axis-aligned rectangle (4 points, edges
// alternately horizontal and vertical): text-line contours.
__device__ __forceinline__ bool axis_rect(const P2 *q, int m) {
  if (m != 4) return false;
  const bool h0 = q[0].y == q[1].y && q[2].y == q[3].y && q[1].x == q[2].x && q[3].x == q[0].x;
  const bool v0 = q[0].x == q[1].x && q[2].x == q[3].x && q[1].y == q[2].y && q[3].y == q[0].y;
  return h0 || v0;
}

// 7. unclip of one contour slot (det_postprocess.cpp:57-102) as the reference
// computes it: Clipper's raw round-join offset (DoOffset), the union of that
// path with positive fill (ClipperOffset::Execute, clipper_union.cuh), the
// output ring of largest area; then the second min-area box and finish_box.
// Runs on lane 0 of a warp whose other lanes serve the sweep's list-wide
// steps (bk). The offset ring, the sweep's arrays and the hull work space
// come from the scratch pool. When the pool or the sweep's bounds run out,
// the box comes from the raw offset ring instead and status bit kErrUnion is
// set.
__device__ void unclip_one(long long c, const int *__restrict__ npts,
                           const long long *__restrict__ pt_off, const P2 *__restrict__ pts,
                           const double *__restrict__ dist, const int *__restrict__ geo,
                           int *__restrict__ keep2, int *__restrict__ boxes,
                           char *__restrict__ pool, int *__restrict__ pool_counters,
                           int *__restrict__ status, const DbParams &P, db::cu::BulkArgs *bk) {
  const int n = npts[c];
  const P2 *p = pts + pt_off[c];
  const double d = dist[c];
  const P2 *ring = p;  // unclip returns the contour itself when there is no offset
  int rn = n;
  if (d != 0.) {
    P2 *q = reinterpret_cast<P2 *>(
        pool_alloc(pool, pool_counters, P.pool_bytes, (n + 1ull) * sizeof(P2), status));
    if (!q) return;
    const int m = db::offset_prepare(p, n, q);
    if (m > 0) {
      const int raw_n = db::offset_raw(q, m, d, nullptr, 0);
      const int out_cap = 2 * raw_n + 64;
      const unsigned long long raw_b = ((unsigned long long)raw_n * sizeof(P2) + 15) & ~15ull;
      const unsigned long long out_b = ((unsigned long long)out_cap * sizeof(P2) + 15) & ~15ull;
      char *w = pool_alloc(pool, pool_counters, P.pool_bytes,
                           raw_b + out_b + db::cu::arena_bytes(raw_n), status);
      if (!w) return;
      P2 *raw = reinterpret_cast<P2 *>(w);
      P2 *out = reinterpret_cast<P2 *>(w + raw_b);
      db::offset_raw(q, m, d, raw, raw_n);
      if (axis_rect(q, m)) {
        // an axis-aligned rectangle's offset is a convex rounded rectangle:
        // the union only drops collinear points, which moves no box corner
        ring = raw;
        rn = raw_n;
      } else {
        db::cu::Sweep sw;
        sw.init(w + raw_b + out_b, raw_n);
        sw.set_bulk(bk, 32);
        int k = -1;
        if (sw.execute(raw, raw_n)) k = sw.best_ring(out, out_cap);
        if (k < 0) {  // sweep out of bounds: the raw ring stands in, flagged
          atomicOr(status, kErrUnion);
          ring = raw;
          rn = raw_n;
        } else if (k > 0) {
          ring = out;
          rn = k;
        }
      }
    }
  }
  if (rn < 3) return;
  RRect r;
  if (rn <= kLocalPts) {
    r = rect_local(ring, rn);
  } else if (!rect_global(ring, rn, pool, pool_counters, P.pool_bytes, status, &r)) {
    return;
  }
  finish_box(r, c, geo, keep2, boxes, P);
}


// One warp per unclip work item (large contours first, from the list that
// score_kernel filled): the sweeps of different rings take different
// branches, so they do not share a warp.
__global__ void __launch_bounds__(128)
union_kernel(const int *__restrict__ ring_list, int *__restrict__ counters,
             const int *__restrict__ npts, const long long *__restrict__ pt_off,
             const P2 *__restrict__ pts, const double *__restrict__ dist,
             const int *__restrict__ geo, int *__restrict__ keep2, int *__restrict__ boxes,
             char *__restrict__ pool, int *__restrict__ status, DbParams P) {
  __shared__ db::cu::BulkArgs s_bulk[4];
  const int lane = threadIdx.x & 31;
  db::cu::BulkArgs *bk = &s_bulk[threadIdx.x >> 5];
  const long long C = (long long)P.n_maps * kMaxCand;
  const int n_big = counters[1];
  const int n_all = n_big + counters[5];
  for (;;) {
    int k = 0;
    if (lane == 0) k = atomicAdd(counters + 6, 1);
    k = __shfl_sync(0xffffffffu, k, 0);
    if (k >= n_all) return;
    const long long c = k < n_big ? ring_list[k] : ring_list[C - 1 - (k - n_big)];
    if (lane == 0) {
      unclip_one(c, npts, pt_off, pts, dist, geo, keep2, boxes, pool, counters, status, P, bk);
      bk->op = db::cu::kOpStop;
      db::cu::bulk_step(bk, 0);
    } else {
      while (db::cu::bulk_step(bk, lane)) {
      }
    }
  }
}

// 8. kept boxes of map m in contour order. grid n_maps, kScanThreads threads.
__global__ void __launch_bounds__(kScanThreads)
compact_kernel(const int *__restrict__ keep2, const int *__restrict__ boxes,
               const float *__restrict__ score, int *__restrict__ out_boxes,
               float *__restrict__ out_scores, int *__restrict__ out_counts,
               int *__restrict__ status, int max_boxes) {
  const int m = blockIdx.x;
  __shared__ int s_part[kScanThreads];
  __shared__ int s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (int c0 = 0; c0 < kMaxCand; c0 += kScanThreads) {
    const int i = c0 + threadIdx.x;
    const long long c = (long long)m * kMaxCand + i;
    const int v = (i < kMaxCand) ? keep2[c] : 0;
    s_part[threadIdx.x] = v;
    __syncthreads();
    for (int off = 1; off < kScanThreads; off <<= 1) {
      const int t = (threadIdx.x >= off) ? s_part[threadIdx.x - off] : 0;
      __syncthreads();
      s_part[threadIdx.x] += t;
      __syncthreads();
    }
    if (v) {
      const int pos = s_carry + s_part[threadIdx.x] - 1;
      if (pos < max_boxes) {
        for (int k = 0; k < 8; ++k) out_boxes[((size_t)m * max_boxes + pos) * 8 + k] = boxes[c * 8 + k];
        out_scores[(size_t)m * max_boxes + pos] = score[c];
      }
    }
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) s_carry += s_part[threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out_counts[m] = s_carry < max_boxes ? s_carry : max_boxes;
    if (s_carry > max_boxes) atomicOr(status, kErrBoxes);
  }
}

// ---- cuda_gpu_ccl_detect (ccl_kernels.cu:241-493): per-component boxes ------
// GpuDetBox of include/turbo_ocr/kernels/kernels.h:118-126.
struct CclBox {
  int xmin, ymin, xmax, ymax;
  float score;
  int pixel_count;
  float ox[4], oy[4];
};
constexpr int kMaxGpuComponents = 3000;

// Foreground roots per row (a root is a pixel labelled with itself).
__global__ void __launch_bounds__(256)
ccl_root_count_kernel(const uint8_t *__restrict__ bitmap, const int *__restrict__ lab, int H, int W,
                      int *__restrict__ row_count) {
  __shared__ int s;
  if (threadIdx.x == 0) s = 0;
  __syncthreads();
  const int y = blockIdx.x;
  int c = 0;
  for (int x = threadIdx.x; x < W; x += blockDim.x) {
    const int p = y * W + x;
    c += bitmap[p] != 0 && lab[p] == p + 1;
  }
  for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(&s, c);
  __syncthreads();
  if (threadIdx.x == 0) row_count[y] = s;
}

// Exclusive scan of the row counts (one CTA), total into *total.
__global__ void __launch_bounds__(1024)
ccl_root_scan_kernel(int *__restrict__ row, int H, int *__restrict__ total) {
  __shared__ int s_w[32];
  __shared__ int s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int y0 = 0; y0 < H; y0 += 1024) {
    const int y = y0 + threadIdx.x;
    const int v = y < H ? row[y] : 0;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += t;
    }
    if (lane == 31) s_w[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int w = s_w[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += t;
      }
      s_w[lane] = w;
    }
    __syncthreads();
    const int incl = x + (wid > 0 ? s_w[wid - 1] : 0) + s_carry;
    if (y < H) row[y] = incl - v;
    __syncthreads();
    if (threadIdx.x == 1023) s_carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = s_carry;
}

// Compact id of every root in raster order (ids >= 3000 become -1), written
// at the root pixel. One CTA per row, 256-pixel chunks.
__global__ void __launch_bounds__(256)
ccl_root_ids_kernel(const uint8_t *__restrict__ bitmap, const int *__restrict__ lab, int H, int W,
                    const int *__restrict__ row_off, int *__restrict__ cid) {
  __shared__ int s_w[8];
  __shared__ int s_carry;
  const int y = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_carry = row_off[y];
  __syncthreads();
  for (int x0 = 0; x0 < W; x0 += 256) {
    const int x = x0 + threadIdx.x, p = y * W + x;
    const bool root = x < W && bitmap[p] != 0 && lab[p] == p + 1;
    const unsigned b = __ballot_sync(0xffffffffu, root);
    if (lane == 0) s_w[wid] = __popc(b);
    __syncthreads();
    int before = s_carry;
    for (int k = 0; k < wid; ++k) before += s_w[k];
    if (root) {
      const int id = before + __popc(b & ((1u << lane) - 1u));
      cid[p] = id < kMaxGpuComponents ? id : -1;
    }
    __syncthreads();
    if (threadIdx.x == 0)
      for (int k = 0; k < 8; ++k) s_carry += s_w[k];
    __syncthreads();
  }
}

// Every pixel: its root's compact id (-1 for background); and the per-id
// box / pixel count / prediction sum.
__global__ void __launch_bounds__(256)
ccl_extract_kernel(const uint8_t *__restrict__ bitmap, const int *__restrict__ lab,
                   const float *__restrict__ pred, int H, int W, int *__restrict__ cid,
                   CclBox *__restrict__ boxes) {
  const long long n = (long long)H * W;
  for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < n;
       p += (long long)gridDim.x * blockDim.x) {
    if (bitmap[p] == 0) { cid[p] = -1; continue; }
    const int r = lab[p] - 1;
    const int id = cid[r];  // the root's entry (roots write only their own value)
    if (r != p) cid[p] = id;
    if (id < 0) continue;
    const int x = (int)(p % W), y = (int)(p / W);
    CclBox &b = boxes[id];
    atomicMin(&b.xmin, x);
    atomicMax(&b.xmax, x);
    atomicMin(&b.ymin, y);
    atomicMax(&b.ymax, y);
    atomicAdd(&b.pixel_count, 1);
    atomicAdd(&b.score, pred[p]);
  }
}

__global__ void ccl_box_init_kernel(CclBox *__restrict__ boxes) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= kMaxGpuComponents) return;
  CclBox b{};
  b.xmin = b.ymin = INT_MAX;
  boxes[i] = b;
}

// The reference filter (ccl_kernels.cu:346-368): pixel_count >= 3, box sides
// >= 3, mean >= box_thresh; kept boxes in compact-id order (one CTA).
__global__ void __launch_bounds__(1024)
ccl_box_filter_kernel(const CclBox *__restrict__ in, float box_thresh, CclBox *__restrict__ out,
                      int *__restrict__ count) {
  __shared__ int s_w[32];
  __shared__ int s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int i0 = 0; i0 < kMaxGpuComponents; i0 += 1024) {
    const int i = i0 + threadIdx.x;
    CclBox b{};
    bool keep = false;
    if (i < kMaxGpuComponents) {
      b = in[i];
      if (b.pixel_count >= 3 && b.xmax - b.xmin + 1 >= 3 && b.ymax - b.ymin + 1 >= 3) {
        b.score = b.score / (float)b.pixel_count;
        keep = !(b.score < box_thresh);
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) s_w[wid] = __popc(bal);
    __syncthreads();
    int before = s_carry;
    for (int k = 0; k < wid; ++k) before += s_w[k];
    if (keep) out[before + __popc(bal & ((1u << lane) - 1u))] = b;
    __syncthreads();
    if (threadIdx.x == 0)
      for (int k = 0; k < 32; ++k) s_carry += s_w[k];
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = s_carry;
}

}  // namespace
}  // namespace tocr

// ------------------------------------------------------------------ host -----
namespace tocr {
namespace {

struct DbLayout {
  size_t bitmap, tile_bg, bits, slab, lab, scan_tot, row_count, row_off, n_contours, n_total,
      starts, npts, pt_off, pts, stage1, aabb, stage2, score, dist, keep2, boxes, list1, list3,
      counters, pool, ovf_first, ovf_next, ovf_pts, ovf_count, part_sum, part_cnt, score_done,
      total;
  int ovf_chunks;
  unsigned long long pool_bytes;
};

size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

DbLayout db_layout(int n_maps, int h, int w, long long point_cap, long long offset_cap) {
  DbLayout L{};
  const size_t px = (size_t)n_maps * h * w;
  const size_t C = (size_t)n_maps * kMaxCand;
  size_t o = 0;
  auto take = [&](size_t bytes) { const size_t at = o; o = align_up(o + bytes); return at; };
  L.bitmap = take(px);
  L.tile_bg = take((size_t)n_maps * ((h + kTileH - 1) / kTileH) * ((w + kTileW - 1) / kTileW));
  L.slab = take(C * kSlab * sizeof(P2));
  L.bits = take((size_t)n_maps * h * ((w + 31) / 32) * 4);
  L.lab = take(px * 4);
  L.scan_tot = take((size_t)n_maps * 8);
  L.row_count = take((size_t)n_maps * h * 4);
  L.row_off = take((size_t)n_maps * h * 4);
  L.n_contours = take((size_t)n_maps * 4);
  L.n_total = take((size_t)n_maps * 4);
  L.starts = take(C * 4);
  L.npts = take(C * 4);
  L.pt_off = take((C + 1) * 8);
  L.pts = take((size_t)point_cap * sizeof(P2));
  L.stage1 = take(C * 4);
  L.aabb = take(C * 16);
  L.stage2 = take(C * 4);
  L.score = take(C * 4);
  L.dist = take(C * 8);
  L.keep2 = take(C * 4);
  L.boxes = take(C * 8 * 4);
  L.list1 = take(C * 4);
  L.list3 = take(C * 4);
  L.counters = take(kCounters * 4);
  L.pool_bytes = (unsigned long long)offset_cap * kPoolBytesPerPoint;
  L.pool = take(L.pool_bytes);
  // trace overflow: the points beyond each contour's slab, in kChunk chunks
  L.ovf_chunks = (int)std::min<long long>(point_cap / kChunk + 256, 1ll << 30);
  L.ovf_first = take(C * 4);
  L.ovf_next = take((size_t)L.ovf_chunks * 4);
  L.ovf_pts = take((size_t)L.ovf_chunks * kChunk * sizeof(P2));
  L.ovf_count = take(4);
  L.part_sum = take(C * kScoreGroups * 8);
  L.part_cnt = take(C * kScoreGroups * 8);
  L.score_done = take(C * 4);
  L.total = o;
  return L;
}

void default_caps(int n_maps, int h, int w, long long *point_cap, long long *offset_cap) {
  if (*point_cap <= 0) *point_cap = (long long)n_maps * ((long long)h * w / 4 + 4096);
  if (*offset_cap <= 0) *offset_cap = *point_cap;
}

// Test hook: the widest point set (x columns) the shared-memory geometry path takes.
std::atomic<int> g_big_cols{kBigCols};

}  // namespace
}  // namespace tocr

using namespace tocr;

extern "C" {

TOCR_API size_t tocr_db_workspace_bytes(int n_maps, int h, int w, long long point_cap,
                                        long long offset_cap) {
  if (n_maps <= 0 || h <= 0 || w <= 0) return 0;
  default_caps(n_maps, h, w, &point_cap, &offset_cap);
  return db_layout(n_maps, h, w, point_cap, offset_cap).total;
}

TOCR_API int tocr_db_postprocess(const float *d_pred, int n_maps, int h, int w,
                                 const int *d_geometry, float thresh, float box_thresh,
                                 float unclip_ratio, float min_box_side,
                                 float min_unclipped_side, long long point_cap,
                                 long long offset_cap, void *d_workspace,
                                 size_t workspace_bytes, int *d_boxes, float *d_scores,
                                 int *d_counts, int max_boxes, int *d_status, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n_maps >= 0 && h > 0 && w > 0 && max_boxes > 0,
               "tocr_db_postprocess: bad sizes n_maps=%d h=%d w=%d max_boxes=%d", n_maps, h, w,
               max_boxes);
  TOCR_REQUIRE((long long)h * w < (1ll << 30) && h < (1 << 19),
               "tocr_db_postprocess: map of %dx%d too large", h, w);
  TOCR_REQUIRE(w <= 32 * kMaxWords, "tocr_db_postprocess: map width %d exceeds %d", w,
               32 * kMaxWords);
  if (n_maps == 0) return TOCR_OK;
  TOCR_REQUIRE(d_pred && d_workspace && d_boxes && d_scores && d_counts && d_status,
               "tocr_db_postprocess: null pointer");
  default_caps(n_maps, h, w, &point_cap, &offset_cap);
  const DbLayout L = db_layout(n_maps, h, w, point_cap, offset_cap);
  TOCR_REQUIRE(workspace_bytes >= L.total,
               "tocr_db_postprocess: workspace of %zu bytes, %zu needed", workspace_bytes, L.total);
  TOCR_REQUIRE(aligned(d_workspace, 256), "tocr_db_postprocess: workspace must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  char *ws = static_cast<char *>(d_workspace);
  auto at = [&](size_t off) { return ws + off; };
  uint8_t *bitmap = (uint8_t *)at(L.bitmap);
  uint8_t *tile_bg = (uint8_t *)at(L.tile_bg);
  P2 *slab = (P2 *)at(L.slab);
  uint32_t *bits = (uint32_t *)at(L.bits);
  int *lab = (int *)at(L.lab);
  long long *scan_tot = (long long *)at(L.scan_tot);
  int *row_count = (int *)at(L.row_count), *row_off = (int *)at(L.row_off);
  int *n_contours = (int *)at(L.n_contours), *n_total = (int *)at(L.n_total);
  int *starts = (int *)at(L.starts), *npts = (int *)at(L.npts);
  long long *pt_off = (long long *)at(L.pt_off);
  P2 *pts = (P2 *)at(L.pts);
  float *score = (float *)at(L.score);
  int *stage1 = (int *)at(L.stage1), *stage2 = (int *)at(L.stage2), *keep2 = (int *)at(L.keep2),
      *boxes = (int *)at(L.boxes), *list1 = (int *)at(L.list1),
      *list3 = (int *)at(L.list3),
      *counters = (int *)at(L.counters);
  char *pool = at(L.pool);
  int *ovf_first = (int *)at(L.ovf_first), *ovf_next = (int *)at(L.ovf_next),
      *ovf_count = (int *)at(L.ovf_count);
  P2 *ovf_pts = (P2 *)at(L.ovf_pts);
  double *part_sum = (double *)at(L.part_sum);
  long long *part_cnt = (long long *)at(L.part_cnt);
  int *score_done = (int *)at(L.score_done);
  int4 *aabb = (int4 *)at(L.aabb);
  double *dist = (double *)at(L.dist);

  DbParams P{n_maps, h, w, thresh, box_thresh, unclip_ratio, min_box_side, min_unclipped_side,
             point_cap, offset_cap, max_boxes, g_big_cols.load(), L.pool_bytes};
  const long long C = (long long)n_maps * kMaxCand;
  const unsigned cgrid = (unsigned)((C + 127) / 128);
  const dim3 tiles((w + kTileW - 1) / kTileW, (h + kTileH - 1) / kTileH, n_maps);

  cudaError_t e = cudaFuncSetAttribute(geom_big_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kBigSmem);
  if (e != cudaSuccess) return set_error(TOCR_ERR_CUDA, "db smem attribute: %s", cudaGetErrorString(e));
  e = cudaMemsetAsync(d_status, 0, sizeof(int), st);
  if (e != cudaSuccess) return set_error(TOCR_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  ccl_local_kernel<<<tiles, 256, 0, st>>>(d_pred, bitmap, lab, bits, nullptr, tile_bg, h, w,
                                          thresh);
  ccl_merge_kernel<<<tiles, 128, 0, st>>>(bitmap, lab, tile_bg, h, w);
  ccl_rows_kernel<<<dim3(h, n_maps), 256, 0, st>>>(lab, row_count, h, w, false);
  starts_scan_kernel<<<n_maps, kScanThreads, 0, st>>>(row_count, row_off, n_contours, n_total, h,
                                                      ovf_count);
  starts_write_kernel<<<dim3(h, n_maps), 256, 0, st>>>(lab, bitmap, row_count, row_off, starts, h, w);
  trace_kernel<<<cgrid, 128, 0, st>>>(bits, starts, n_contours, npts, slab, ovf_first, ovf_next,
                                      ovf_pts, ovf_count, L.ovf_chunks, d_status, n_maps, h, w);
  scan_map_kernel<int><<<n_maps, kScanThreads, 0, st>>>(npts, pt_off, scan_tot);
  scan_base_kernel<<<n_maps, kScanThreads, 0, st>>>(pt_off, scan_tot, n_maps);
  prep_geom_kernel<<<1, 1, 0, st>>>(pt_off, C, point_cap, d_status, counters);
  gather_kernel<<<(unsigned)((C * 32 + 127) / 128), 128, 0, st>>>(
      bits, starts, npts, pt_off, slab, ovf_first, ovf_next, ovf_pts, pts, point_cap, n_maps, h, w);
  geom_box1_kernel<<<cgrid, 128, 0, st>>>(n_contours, npts, pt_off, pts, stage1, aabb, list1,
                                          counters, score_done, list3, stage2, keep2, P);
  const unsigned bgrid = (unsigned)(C < sm_count() ? C : sm_count());
  geom_big_kernel<<<bgrid, kBigThreads, kBigSmem, st>>>(list1, counters, npts, pt_off, pts, aabb,
                                                        stage1, list3, pool, counters, d_status, P);
  score_kernel<<<dim3((unsigned)(C < 148 * 8 ? C : 148 * 8), kScoreGroups), kScoreThreads, 0, st>>>(
      d_pred, list3, counters, aabb, npts, pt_off, pts, stage2, score, dist, part_sum, part_cnt,
      score_done, list1, P);
  // list1 (geom_big_kernel's large-contour list) is reused for the unclip work list
  const unsigned ugrid = (unsigned)std::min<long long>((C + 3) / 4, (long long)sm_count() * 16);
  union_kernel<<<ugrid, 128, 0, st>>>(list1, counters, npts, pt_off, pts, dist, d_geometry, keep2,
                                      boxes, pool, d_status, P);
  compact_kernel<<<n_maps, kScanThreads, 0, st>>>(keep2, boxes, score, d_boxes, d_scores, d_counts,
                                                  d_status, max_boxes);
  return check_launch("tocr_db_postprocess");
}

// Test hook (tocr_capi.h): sets the widest point set (x columns) the
// shared-memory geometry path takes (0: every set above the thread-local
// size uses the global pool; < 0 or above the compiled capacity: the
// compiled capacity).
TOCR_API void tocr_debug_db_shared_columns(int columns) {
  g_big_cols.store(columns < 0 || columns > kBigCols ? kBigCols : columns);
}

// Labels of the first three stages, for tests and tools: labels[m][y][x] =
// 0 for background joined to the image frame, else 1 + the raster index of
// the smallest pixel of the pixel's component (foreground 8-connected,
// background 4-connected). d_bitmap receives the 0/255 threshold bitmap.
TOCR_API size_t tocr_db_components_scratch_bytes(int n_maps, int h, int w) {
  if (n_maps <= 0 || h <= 0 || w <= 0) return 0;
  const size_t tiles = (size_t)n_maps * ((h + kTileH - 1) / kTileH) * ((w + kTileW - 1) / kTileW);
  return (size_t)n_maps * h * w + tiles;
}

TOCR_API int tocr_db_components(const float *d_pred, int n_maps, int h, int w, float thresh,
                                int *d_labels, uint8_t *d_bitmap, void *d_scratch, void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(n_maps >= 0 && h > 0 && w > 0 && (long long)h * w < (1ll << 30),
               "tocr_db_components: bad sizes n_maps=%d h=%d w=%d", n_maps, h, w);
  if (n_maps == 0) return TOCR_OK;
  TOCR_REQUIRE(d_pred && d_labels && d_bitmap, "tocr_db_components: null pointer");
  cudaStream_t st = as_stream(stream);
  const dim3 tiles((w + kTileW - 1) / kTileW, (h + kTileH - 1) / kTileH, n_maps);
  uint8_t *root_flag = static_cast<uint8_t *>(d_scratch);
  uint8_t *tile_bg = root_flag ? root_flag + (size_t)n_maps * h * w : nullptr;
  ccl_local_kernel<<<tiles, 256, 0, st>>>(d_pred, d_bitmap, d_labels, nullptr, root_flag, tile_bg,
                                          h, w, thresh);
  ccl_merge_kernel<<<tiles, 128, 0, st>>>(d_bitmap, d_labels, tile_bg, h, w);
  if (root_flag) ccl_roots_kernel<<<tiles, 256, 0, st>>>(d_labels, root_flag, h, w);
  ccl_rows_kernel<<<dim3(h, n_maps), 256, 0, st>>>(d_labels, nullptr, h, w, true);
  return check_launch("tocr_db_components");
}

// cuda_gpu_ccl_detect (include/turbo_ocr/kernels/kernels.h:131-145): labels
// (8-connected) of the 255/0 bitmap, compact ids in raster order of each
// component's first pixel (at most 3000), per-id box / pixel count / mean
// prediction, the reference's filter, kept boxes in id order; one
// synchronisation, then *h_num_boxes boxes in h_boxes.
TOCR_API int tocr_gpu_ccl_detect(const uint8_t *d_bitmap, const float *d_pred, int w, int h,
                                 float box_thresh, int *d_labels, int *d_compact_ids,
                                 int *d_id_counter, void *d_bboxes, int *d_num_boxes,
                                 void *h_boxes, int *h_num_boxes, int *h_num_total,
                                 void *stream) {
  TOCR_ENTRY();
  TOCR_REQUIRE(w > 0 && h > 0 && (long long)w * h < (1ll << 30) && h <= (int)(
                   (2 * kMaxGpuComponents * sizeof(CclBox)) / (2 * sizeof(int))),
               "tocr_gpu_ccl_detect: bad sizes %dx%d", w, h);
  TOCR_REQUIRE(d_bitmap && d_pred && d_labels && d_compact_ids && d_id_counter && d_bboxes &&
                   d_num_boxes && h_boxes && h_num_boxes,
               "tocr_gpu_ccl_detect: null pointer");
  cudaStream_t st = as_stream(stream);
  const dim3 tiles((w + kTileW - 1) / kTileW, (h + kTileH - 1) / kTileH, 1);
  CclBox *boxes = static_cast<CclBox *>(d_bboxes);
  int *row = reinterpret_cast<int *>(boxes);  // row offsets, before the boxes are used
  ccl_local_kernel<<<tiles, 256, 0, st>>>(nullptr, const_cast<uint8_t *>(d_bitmap), d_labels,
                                          nullptr, nullptr, nullptr, h, w, 0.f);
  ccl_merge_kernel<<<tiles, 128, 0, st>>>(d_bitmap, d_labels, nullptr, h, w);
  ccl_rows_kernel<<<dim3(h, 1), 256, 0, st>>>(d_labels, nullptr, h, w, true);
  ccl_root_count_kernel<<<h, 256, 0, st>>>(d_bitmap, d_labels, h, w, row);
  ccl_root_scan_kernel<<<1, 1024, 0, st>>>(row, h, d_id_counter);
  ccl_root_ids_kernel<<<h, 256, 0, st>>>(d_bitmap, d_labels, h, w, row, d_compact_ids);
  ccl_box_init_kernel<<<(kMaxGpuComponents + 255) / 256, 256, 0, st>>>(boxes);
  const long long n = (long long)w * h;
  const unsigned grid = (unsigned)std::min<long long>((n + 255) / 256, (long long)sm_count() * 16);
  ccl_extract_kernel<<<grid, 256, 0, st>>>(d_bitmap, d_labels, d_pred, h, w, d_compact_ids, boxes);
  ccl_box_filter_kernel<<<1, 1024, 0, st>>>(boxes, box_thresh, boxes + kMaxGpuComponents,
                                            d_num_boxes);
  int rc = check_launch("tocr_gpu_ccl_detect");
  if (rc != TOCR_OK) return rc;
  cudaError_t e = cudaMemcpyAsync(h_num_boxes, d_num_boxes, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && h_num_total)
    e = cudaMemcpyAsync(h_num_total, d_id_counter, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h_boxes, boxes + kMaxGpuComponents, kMaxGpuComponents * sizeof(CclBox),
                        cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess)
    return set_error(TOCR_ERR_CUDA, "tocr_gpu_ccl_detect: %s", cudaGetErrorString(e));
  if (*h_num_boxes > kMaxGpuComponents) *h_num_boxes = kMaxGpuComponents;
  return TOCR_OK;
}

}  // extern "C"
