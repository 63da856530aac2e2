// DB post-processing geometry, written once for the device kernels (db.cu)
// and for a host build used by the CPU tests. Every routine reproduces the
// arithmetic of the reference's CPU path operation for operation:
//
//   border following (CHAIN_APPROX_SIMPLE) ... cv::findContours(RETR_LIST), called at
//                                              src/detection/det_postprocess.cpp:162-163
//   convex hull + rotating calipers ......... cv::minAreaRect, det_postprocess.cpp:129
//   rectangle corners + corner order ........ RotatedRect::points, order_quad_tl_tr_br_bl,
//                                              det_postprocess.cpp:104-143
//   polygon mask mean ........................ box_score_fast, det_postprocess.cpp:15-55
//   area / perimeter / offset distance ....... unclip, det_postprocess.cpp:57-66
//   round-join polygon offset ............... ClipperOffset (Clipper 6.4.2, jtRound,
//                                              etClosedPolygon), det_postprocess.cpp:72-101
//
// The algorithms are the published ones (Suzuki & Abe 1985 border following;
// Andrew's monotone chain; Toussaint's rotating calipers; Vatti-style
// positive-fill offset cleanup). The floating-point operation order was
// fixed by testing against the libraries' outputs: OpenCV's float/double code
// is uncontracted, while the reference builds Clipper with -O3
// -march=x86-64-v3 (CMakeLists.txt:97-100,259-268), so its multiply-adds are
// FMAs — written here as explicit fma() calls. Device code that includes this
// header is compiled with -fmad=false so nothing else is contracted.
#pragma once

#include <cmath>
#include <cstdint>

#if defined(__CUDACC__)
#define TG __host__ __device__ __forceinline__
#else
#define TG inline
#endif

namespace tocr {
namespace db {

struct P2 {
  int x, y;
};
struct F2 {
  float x, y;
};

// ------------------------------------------------------------------ tracing --
#if defined(__CUDA_ARCH__)
TG int __builtin_ctz_tg(uint32_t v) { return __ffs((int)v) - 1; }
TG int __builtin_clz_tg(uint32_t v) { return __clz((int)v); }
#else
TG int __builtin_ctz_tg(uint32_t v) { return __builtin_ctz(v); }
TG int __builtin_clz_tg(uint32_t v) { return __builtin_clz(v); }
#endif

// Freeman chain codes, image coordinates (y down): 0 E, 1 NE, 2 N, 3 NW,
// 4 W, 5 SW, 6 S, 7 SE. Increasing code = counter-clockwise on screen.
TG int code_dx(int d) { return (d == 0 || d == 1 || d == 7) ? 1 : (d >= 3 && d <= 5) ? -1 : 0; }
TG int code_dy(int d) { return (d >= 1 && d <= 3) ? -1 : (d >= 5) ? 1 : 0; }

// Follows the border that starts at pixel (x0, y0): the raster-first pixel
// of an 8-connected foreground component (outer border, previous pixel on
// the W side) or the foreground pixel left of the raster-first pixel of a
// hole (hole border, previous pixel on the E side). Points are emitted where
// the chain code changes (CHAIN_APPROX_SIMPLE); the start pixel is always
// emitted. nb(x, y) returns the 8-neighbourhood of (x, y) as a bit mask
// (bit d set when the neighbour in chain-code direction d is foreground;
// outside the image counts as background). Calls emit(x, y) for each point
// and returns their count, or -1 if max_steps was exceeded.
template <class NB, class EMIT>
TG int trace_border_emit(NB &nb, int x0, int y0, bool hole, EMIT &&emit, int max_steps) {
  const int dstart = hole ? 0 : 4;
  int d1 = -1;
  {
    const unsigned m0 = nb(x0, y0);
    for (int k = 1; k <= 8; ++k) {  // clockwise from the previous pixel
      const int d = (dstart - k) & 7;
      if ((m0 >> d) & 1u) {
        d1 = d;
        break;
      }
    }
  }
  // first foreground direction counter-clockwise after `from` (the mask is
  // rotated so that direction from+1 is bit 0); `from` itself when none
  auto ccw_after = [](unsigned mask, int from) {
    const unsigned r = ((mask | (mask << 8)) >> (from + 1)) & 0xFFu;
    return r ? (from + 1 + __builtin_ctz_tg(r)) & 7 : from;
  };
  int n = 0;
  if (d1 < 0) {  // isolated pixel
    emit(x0, y0);
    return 1;
  }
  const int x1 = x0 + code_dx(d1), y1 = y0 + code_dy(d1);
  int last_code = d1 ^ 4;
  int x3 = x0, y3 = y0, dback = d1;
  for (int step = 0; step < max_steps; ++step) {
    const int d4 = ccw_after(nb(x3, y3), dback);  // counter-clockwise after the previous pixel
    if (d4 != last_code) {
      emit(x3, y3);
      ++n;
      last_code = d4;
    }
    const int x4 = x3 + code_dx(d4), y4 = y3 + code_dy(d4);
    if (x4 == x0 && y4 == y0 && x3 == x1 && y3 == y1) return n;
    dback = (d4 + 4) & 7;
    x3 = x4;
    y3 = y4;
    // Straight horizontal stretches: from (x3, y3), after an E move the walk
    // keeps moving E while SW, S, SE are background and E is foreground (W
    // mirrored with NE, N, NW); such moves repeat the chain code, so no point
    // is emitted. Jump over them; on the start row stop two pixels short of
    // the start pixel, so the closing test above still sees the last moves.
    if (d4 == 0 || d4 == 4) {
      int L = nb.run(x3, y3, d4);
      if (y3 == y0) {
        const int room = d4 == 0 ? x0 - x3 - 2 : x3 - x0 - 2;
        if ((d4 == 0 ? x3 < x0 : x3 > x0) && L > room) L = room;
      }
      if (L > max_steps - step - 1) L = max_steps - step - 1;
      if (L > 0) {
        x3 += d4 == 0 ? L : -L;
        step += L;
      }
    }
  }
  return -1;
}

// trace_border_emit into out: writes at most cap points, returns the full
// count (or -1).
template <class NB>
TG int trace_border_nb(NB &nb, int x0, int y0, bool hole, P2 *out, int cap, int max_steps) {
  int k = 0;
  return trace_border_emit(
      nb, x0, y0, hole,
      [&](int x, int y) {
        if (k < cap) out[k] = P2{x, y};
        ++k;
      },
      max_steps);
}

// Neighbourhood mask from a per-pixel predicate fg(x, y).
template <class FG>
struct NbFromFg {
  const FG &fg;
  TG unsigned operator()(int x, int y) const {
    unsigned m = 0;
    for (int d = 0; d < 8; ++d) m |= (fg(x + code_dx(d), y + code_dy(d)) ? 1u : 0u) << d;
    return m;
  }
  // Number of further moves in direction dir (0 E or 4 W) that repeat it.
  TG int run(int x, int y, int dir) const {
    const int s = dir == 0 ? 1 : -1, side = dir == 0 ? 1 : -1;  // S row for E, N row for W
    int L = 0;
    for (;;) {
      const int cx = x + s * L;
      if (fg(cx - 1, y + side) || fg(cx, y + side) || fg(cx + 1, y + side) || !fg(cx + s, y))
        return L;
      ++L;
    }
  }
};

template <class FG>
TG int trace_border(const FG &fg, int x0, int y0, bool hole, P2 *out, int cap, int max_steps) {
  NbFromFg<FG> nb{fg};
  return trace_border_nb(nb, x0, y0, hole, out, cap, max_steps);
}

// Neighbourhood masks from a bit-packed bitmap (bit x & 31 of word
// y * words + (x >> 5)), caching the 3 x 2 words around the last centre so
// that a walk along a row reloads once per 32 pixels.
// Low 32 bits of (hi:lo) >> sh, sh in [0, 31].
TG uint32_t funnel_r(uint32_t lo, uint32_t hi, int sh) {
#ifdef __CUDA_ARCH__
  return __funnelshift_r(lo, hi, sh);
#else
  return (uint32_t)((((uint64_t)hi << 32) | lo) >> sh);
#endif
}

// Read of the packed bitmap: written by an earlier kernel, read-only while
// borders are traced, so the device reads it through the non-coherent cache.
TG uint32_t ld_bits(const uint32_t *p) {
#ifdef __CUDA_ARCH__
  return __ldg(p);
#else
  return *p;
#endif
}

struct NbBits {
  const uint32_t *bits;
  int H, W, words;
  int cy = -1000000, cw = -1000000;
  uint32_t r[3][2];
  TG unsigned operator()(int x, int y) {
    const int w0 = (x - 1) >> 5;  // arithmetic shift: x - 1 = -1 gives -1
    if (y != cy || w0 != cw) {
      cy = y;
      cw = w0;
      for (int i = 0; i < 3; ++i) {
        const int yy = y - 1 + i;
        const bool row_ok = yy >= 0 && yy < H;
        r[i][0] = (row_ok && w0 >= 0 && w0 < words) ? ld_bits(bits + (long long)yy * words + w0) : 0u;
        r[i][1] = (row_ok && w0 + 1 < words) ? ld_bits(bits + (long long)yy * words + w0 + 1) : 0u;
      }
    }
    const int sh = (x - 1) - (w0 << 5);  // bit of column x - 1 inside word w0, 0..31
    // columns x-1, x, x+1 of rows y-1, y, y+1 (columns beyond the image width
    // read 0: the bitmap is zero-padded per row)
    const uint32_t t0 = funnel_r(r[0][0], r[0][1], sh) & 7u;
    const uint32_t t1 = funnel_r(r[1][0], r[1][1], sh) & 7u;
    const uint32_t t2 = funnel_r(r[2][0], r[2][1], sh) & 7u;
    // directions: 0 E (x+1,y) 1 NE (x+1,y-1) 2 N 3 NW 4 W 5 SW 6 S 7 SE:
    // NE N NW are row y-1 right to left, SW S SE row y+1 left to right
    const uint32_t rev0 = ((t0 & 1u) << 2) | (t0 & 2u) | (t0 >> 2);
    return (t1 >> 2) | (rev0 << 1) | ((t1 & 1u) << 4) | (t2 << 5);
  }
  TG uint32_t word(int y, int w) const {
    return (y >= 0 && y < H && w >= 0 && w < words) ? ld_bits(bits + (long long)y * words + w) : 0u;
  }
  // First column >= x0 whose bit in row y equals v (W if none before the end).
  TG int find_fwd(int y, int x0, bool v) const {
    if (x0 < 0) {
      if (!v) return x0;  // columns left of the image are background
      x0 = 0;
    }
    for (int w = x0 >> 5; w < words; ++w) {
      uint32_t b = word(y, w);
      if (!v) b = ~b;
      if (w == (x0 >> 5)) b &= ~0u << (x0 & 31);
      if (b) {
        const int c = (w << 5) + __builtin_ctz_tg(b);
        return c < W ? c : W;
      }
    }
    return v ? W + 64 : W;  // no set bit: never; no clear bit: columns >= W are background
  }
  // Last column <= x0 whose bit in row y equals v (-1 if none).
  TG int find_bwd(int y, int x0, bool v) const {
    if (x0 >= W) {
      if (!v) return x0;  // columns right of the image are background
      x0 = W - 1;
    }
    for (int w = x0 >> 5; w >= 0; --w) {
      uint32_t b = word(y, w);
      if (!v) b = ~b;
      if (w == (x0 >> 5)) b &= (x0 & 31) == 31 ? ~0u : ((2u << (x0 & 31)) - 1u);
      if (b) return (w << 5) + 31 - __builtin_clz_tg(b);
    }
    return v ? -64 : -1;
  }
  TG int run(int x, int y, int dir) const {
    if (dir == 0) {
      const int a = find_fwd(y + 1, x - 1, true);   // first foreground below, from x-1
      const int b = find_fwd(y, x + 1, false);      // first background on the row, from x+1
      const int L = (a < b ? a : b) - x - 1;
      return L > 0 ? L : 0;
    }
    const int a = find_bwd(y - 1, x + 1, true);     // last foreground above, up to x+1
    const int b = find_bwd(y, x - 1, false);        // last background on the row, up to x-1
    const int L = x - 1 - (a > b ? a : b);
    return L > 0 ? L : 0;
  }
};

// --------------------------------------------------------------- sorting ----
struct HP {  // hull candidate: point + index in the input sequence
  int x, y, idx;
};
TG bool hp_less(const HP &a, const HP &b) {
  return a.x < b.x || (a.x == b.x && (a.y < b.y || (a.y == b.y && a.idx < b.idx)));
}
TG void hp_sift(HP *a, int start, int end) {
  int root = start;
  while (2 * root + 1 <= end) {
    int child = 2 * root + 1;
    if (child + 1 <= end && hp_less(a[child], a[child + 1])) ++child;
    if (hp_less(a[root], a[child])) {
      HP t = a[root];
      a[root] = a[child];
      a[child] = t;
      root = child;
    } else {
      return;
    }
  }
}
TG void hp_sort(HP *a, int n) {  // in-place heapsort (no recursion, no allocation)
  for (int s = (n - 2) / 2; s >= 0; --s) hp_sift(a, s, n - 1);
  for (int e = n - 1; e > 0; --e) {
    HP t = a[0];
    a[0] = a[e];
    a[e] = t;
    hp_sift(a, 0, e - 1);
  }
}

// ------------------------------------------------------------------ hull -----
TG long long cross3(const HP &o, const HP &a, const HP &b) {
  return (long long)(a.x - o.x) * (b.y - o.y) - (long long)(a.y - o.y) * (b.x - o.x);
}

// Writes the chain (accessor at(i) -> HP, i < m, in the order of Andrew's
// monotone chain) to hull, rotated to cv::convexHull's starting vertex: when
// the input indices of the hull vertices are cyclically increasing the hull
// starts at the smallest index, when cyclically decreasing at the largest,
// otherwise at the vertex with the largest (x, y).
template <class AT>
TG void hull_start_copy(int m, const AT &at, P2 *hull) {
  int start = 0;
  if (m >= 3) {
    int inc = 0;
    for (int i = 0; i < m; ++i) inc += at((i + 1) % m).idx > at(i).idx;
    if (inc == m - 1 || inc == 1) {
      const bool increasing = (inc == m - 1);
      for (int i = 1; i < m; ++i)
        if (increasing ? at(i).idx < at(start).idx : at(i).idx > at(start).idx) start = i;
    } else {
      for (int i = 1; i < m; ++i)
        if (at(i).x > at(start).x || (at(i).x == at(start).x && at(i).y > at(start).y)) start = i;
    }
  } else {
    for (int i = 1; i < m; ++i)
      if (at(i).x > at(start).x || (at(i).x == at(start).x && at(i).y > at(start).y)) start = i;
  }
  for (int i = 0; i < m; ++i) {
    const HP q = at((start + i) % m);
    hull[i] = P2{q.x, q.y};
  }
}

// Strict convex hull (no collinear or repeated points) of pts[0..n), in the
// orientation and with the starting vertex of cv::convexHull(clockwise=false)
// (a repeated point counts with its first index; start rule as
// hull_start_copy). `work` needs 2n+1 entries and is clobbered. Returns the
// hull size.
TG int convex_hull(const P2 *pts, int n, HP *work, P2 *hull) {
  if (n <= 0) return 0;
  HP *s = work;            // sorted points [0, n)
  HP *h = work + n;        // hull chain, up to n+1 entries
  for (int i = 0; i < n; ++i) s[i] = HP{pts[i].x, pts[i].y, i};
  hp_sort(s, n);
  {  // repeated points: keep the first occurrence (smallest input index)
    int u = 1;
    for (int i = 1; i < n; ++i)
      if (s[i].x != s[u - 1].x || s[i].y != s[u - 1].y) s[u++] = s[i];
    n = u;
  }
  int k = 0;
  for (int i = 0; i < n; ++i) {  // lower chain
    while (k >= 2 && cross3(h[k - 2], h[k - 1], s[i]) <= 0) --k;
    h[k++] = s[i];
  }
  for (int i = n - 2, t = k + 1; i >= 0; --i) {  // upper chain
    while (k >= t && cross3(h[k - 2], h[k - 1], s[i]) <= 0) --k;
    h[k++] = s[i];
  }
  int m = k > 1 ? k - 1 : k;  // last point repeats the first
  if (m == 2 && h[0].x == h[1].x && h[0].y == h[1].y) m = 1;
  hull_start_copy(m, [&](int i) { return h[i]; }, hull);
  return m;
}

// ----------------------------------------------------- column hull (CTA) ----
// Only the lowest and the highest point of an x column can be strict hull
// vertices (every other point lies between them), and a repeated point
// counts with its first index. So a point set reduces to a table over its x
// columns: lo[c] = min of (y, index) and hi[c] = max y with min index, each
// packed into one u64 so that a plain (or atomic) minimum keeps it:
// (y + 2^20) or (2^20 - 1 - y) in the top 21 bits, the index below.
// kColEmpty marks a column without points. Requires |y| < 2^20.
constexpr uint64_t kColEmpty = ~0ull;
constexpr int kColYBias = 1 << 20;
TG bool col_y_fits(long long y) { return y > -kColYBias && y < kColYBias; }
TG uint64_t col_lo_key(int y, int idx) {
  return ((uint64_t)(uint32_t)(y + kColYBias) << 43) | (uint64_t)(uint32_t)idx;
}
TG uint64_t col_hi_key(int y, int idx) {
  return ((uint64_t)(uint32_t)(kColYBias - 1 - y) << 43) | (uint64_t)(uint32_t)idx;
}
TG int col_lo_y(uint64_t k) { return (int)(k >> 43) - kColYBias; }
TG int col_hi_y(uint64_t k) { return kColYBias - 1 - (int)(k >> 43); }
TG int col_idx(uint64_t k) { return (int)(k & 0x7FFFFFFFull); }
TG void col_add(uint64_t *lo, uint64_t *hi, int c, int y, int idx) {  // serial form
  const uint64_t a = col_lo_key(y, idx), b = col_hi_key(y, idx);
  if (a < lo[c]) lo[c] = a;
  if (b < hi[c]) hi[c] = b;
}

// Entry e of the candidate sequence (in (x, y, index) order): column e/2,
// its lowest point (e even) or its highest (e odd; absent when the column
// holds a single y). False when absent.
TG bool col_entry(const uint64_t *lo, const uint64_t *hi, int base, int e, HP *out) {
  const int c = e >> 1;
  const uint64_t l = lo[c];
  if (l == kColEmpty) return false;
  if (e & 1) {
    const uint64_t h = hi[c];
    const int yh = col_hi_y(h);
    if (yh == col_lo_y(l)) return false;
    *out = HP{base + c, yh, col_idx(h)};
  } else {
    *out = HP{base + c, col_lo_y(l), col_idx(l)};
  }
  return true;
}

// Interior filter (Akl-Toussaint): the points extreme in kExtDirs integer
// directions of increasing angle lie on the hull boundary and, in that
// order, form a convex polygon inside the hull; a point strictly inside it
// is no hull vertex and can be dropped before the chain. Directions are
// 512 * (cos, sin) of k * 22.5 degrees, rounded.
constexpr int kExtDirs = 16;
TG int ext_cos(int k) {
  const int c[16] = {512, 473, 362, 196, 0, -196, -362, -473, -512, -473, -362, -196, 0, 196, 362, 473};
  return c[k & 15];
}
TG long long ext_dot(int k, int x, int y) {
  return (long long)ext_cos(k) * x + (long long)ext_cos(k + 12) * y;
}
// True when v is strictly inside the polygon poly[0..k) of extreme points
// (at least three non-degenerate edges needed; a degenerate polygon has no
// inside).
TG bool strictly_inside_extremes(const HP *poly, int k, const HP &v) {
  int edges = 0;
  for (int i = 0; i < k; ++i) {
    const HP &a = poly[i], &b = poly[(i + 1) % k];
    if (a.x == b.x && a.y == b.y) continue;
    if (cross3(a, b, v) <= 0) return false;
    ++edges;
  }
  return edges >= 3;
}

// Andrew's monotone chain over the candidates of the table of ncols columns
// (x = base + c): the same hull, orientation and starting vertex as
// convex_hull on the original points. keep (optional): bit e set for the
// entries that may be hull vertices (every hull vertex must be kept). stk
// (entries) needs 2*ncols+1 ints. Returns the hull size, or -1 when it
// exceeds hull_cap.
TG int hull_from_table(const uint64_t *lo, const uint64_t *hi, int ncols, int base, int *stk,
                       P2 *hull, int hull_cap, const uint32_t *keep = nullptr) {
  const int ns = 2 * ncols;
  HP a, b, v;
  auto at = [&](int e) {
    HP r{0, 0, 0};
    col_entry(lo, hi, base, e, &r);
    return r;
  };
  // next kept entry at or after e (ns if none) / at or before e (-1 if none)
  const int nw = (ns + 31) >> 5;
  auto next_kept = [&](int e) {
    if (!keep) return e;
    for (int w = e >> 5; w < nw; ++w) {
      uint32_t b = keep[w];
      if (w == (e >> 5)) b &= ~0u << (e & 31);
      if (b) return (w << 5) + __builtin_ctz_tg(b);
    }
    return ns;
  };
  auto prev_kept = [&](int e) {
    if (!keep) return e;
    for (int w = e >> 5; w >= 0; --w) {
      uint32_t b = keep[w];
      if (w == (e >> 5)) b &= (e & 31) == 31 ? ~0u : ((2u << (e & 31)) - 1u);
      if (b) return (w << 5) + 31 - __builtin_clz_tg(b);
    }
    return -1;
  };
  int top = 0, last = -1;
  for (int e = next_kept(0); e < ns; e = next_kept(e + 1)) {  // lower chain
    if (!col_entry(lo, hi, base, e, &v)) continue;
    last = e;
    while (top >= 2) {
      a = at(stk[top - 2]);
      b = at(stk[top - 1]);
      if (cross3(a, b, v) > 0) break;
      --top;
    }
    stk[top++] = e;
  }
  if (last < 0) return 0;
  const int t = top + 1;
  for (int e = last > 0 ? prev_kept(last - 1) : -1; e >= 0; e = e > 0 ? prev_kept(e - 1) : -1) {
    if (!col_entry(lo, hi, base, e, &v)) continue;  // upper chain
    while (top >= t) {
      a = at(stk[top - 2]);
      b = at(stk[top - 1]);
      if (cross3(a, b, v) > 0) break;
      --top;
    }
    stk[top++] = e;
  }
  int m = top > 1 ? top - 1 : top;
  if (m == 2) {
    a = at(stk[0]);
    b = at(stk[1]);
    if (a.x == b.x && a.y == b.y) m = 1;
  }
  if (m > hull_cap) return -1;
  hull_start_copy(m, [&](int i) { return at(stk[i]); }, hull);
  return m;
}

// ------------------------------------------------------------ min-area rect --
struct RRect {
  float cx, cy, w, h, angle;  // angle in degrees, as cv::RotatedRect
};

// The angle convention of the OpenCV used by the reference's CPU path: the
// side vector is expressed with an angle in [-90, 0) degrees (computed in
// double, one rounding to float), swapping width and height when the
// perpendicular side is chosen.
TG RRect normalize_rect(RRect r, double deg) {
  for (int it = 0; it < 4 && deg >= 0; ++it) {
    if (deg >= 90) {
      deg -= 180;
    } else {
      deg -= 90;
      const float t = r.w; r.w = r.h; r.h = t;
    }
  }
  if (deg < -90) {
    deg += 90;
    const float t = r.w; r.w = r.h; r.h = t;
  }
  r.angle = (float)deg;
  return r;
}

// d1 / sqrt(l1) > d2 / sqrt(l2), exactly (l1, l2 > 0; |d| <= 2^31 * 2^31).
TG bool cos_greater(long long d1, long long l1, long long d2, long long l2) {
  if ((d1 >= 0) != (d2 >= 0)) return d1 >= 0 && !(d1 == 0 && d2 == 0);
  const unsigned long long a1 = (unsigned long long)(d1 < 0 ? -d1 : d1);
  const unsigned long long a2 = (unsigned long long)(d2 < 0 ? -d2 : d2);
  // compare a1^2 * l2 against a2^2 * l1 in 192-bit-safe steps via 128-bit parts
  const unsigned __int128 s1 = (unsigned __int128)a1 * a1, s2 = (unsigned __int128)a2 * a2;
  // s * l can exceed 128 bits only for coordinates beyond 2^20; split l
  const unsigned long long L2 = (unsigned long long)l2, L1 = (unsigned long long)l1;
  const unsigned __int128 lo1 = (s1 & 0xffffffffffffffffull) * L2, hi1 = (s1 >> 64) * L2;
  const unsigned __int128 lo2 = (s2 & 0xffffffffffffffffull) * L1, hi2 = (s2 >> 64) * L1;
  const unsigned __int128 t1 = hi1 + (lo1 >> 64), t2 = hi2 + (lo2 >> 64);
  const unsigned long long b1 = (unsigned long long)lo1, b2 = (unsigned long long)lo2;
  const bool gt = t1 > t2 || (t1 == t2 && b1 > b2);
  const bool lt = t1 < t2 || (t1 == t2 && b1 < b2);
  return d1 >= 0 ? gt : lt;  // both non-negative: larger magnitude wins
}

// cv::minAreaRect on a hull produced by convex_hull (rotating calipers in
// float; edge lengths and orientation tests in double).
TG RRect min_area_rect(const P2 *hull, int n, float *scratch /* 3n floats */,
                       float *raw6 = nullptr) {
  RRect r{0.f, 0.f, 0.f, 0.f, 0.f};
  if (n <= 0) return r;
  if (n == 1) {
    r.cx = (float)hull[0].x;
    r.cy = (float)hull[0].y;
    return normalize_rect(r, 0.0);
  }
  if (n == 2) {
    const float x0 = (float)hull[0].x, y0 = (float)hull[0].y;
    const float x1 = (float)hull[1].x, y1 = (float)hull[1].y;
    r.cx = (x0 + x1) * 0.5f;
    r.cy = (y0 + y1) * 0.5f;
    const double dx = (double)x1 - x0, dy = (double)y1 - y0;
    r.w = (float)sqrt(dx * dx + dy * dy);
    r.h = 0.f;
    return normalize_rect(r, atan2(dy, dx) * 180 / 3.141592653589793238);
  }
  float *ilen = scratch;       // 1 / |edge|
  float *vx = scratch + n;     // edge vectors
  float *vy = scratch + 2 * n;
  int left = 0, bottom = 0, right = 0, top = 0;
  float left_x = (float)hull[0].x, right_x = left_x;
  float top_y = (float)hull[0].y, bottom_y = top_y;
  for (int i = 0; i < n; ++i) {
    const float px = (float)hull[i].x, py = (float)hull[i].y;
    if (px < left_x) { left_x = px; left = i; }
    if (px > right_x) { right_x = px; right = i; }
    if (py > top_y) { top_y = py; top = i; }
    if (py < bottom_y) { bottom_y = py; bottom = i; }
    const int j = (i + 1 < n) ? i + 1 : 0;
    const double dx = (double)((float)hull[j].x - px);
    const double dy = (double)((float)hull[j].y - py);
    vx[i] = (float)dx;
    vy[i] = (float)dy;
    ilen[i] = (float)(1. / sqrt(dx * dx + dy * dy));
  }
  float orientation = 0.f;
  {
    double ax = vx[n - 1], ay = vy[n - 1];
    for (int i = 0; i < n; ++i) {
      const double bx = vx[i], by = vy[i];
      const double c = ax * by - ay * bx;
      if (c != 0) {
        orientation = (c > 0) ? 1.f : -1.f;
        break;
      }
      ax = bx;
      ay = by;
    }
  }
  float ba = orientation, bb = 0.f;  // current caliper direction (a, b)
  // The same direction as an exact integer vector: the edge that set it.
  long long Bx = orientation > 0 ? 1 : -1, By = 0;
  int seq[4] = {bottom, right, top, left};
  float minarea = 3.402823466e+38f;
  int best_left = 0, best_bottom = 0;
  float best_a = 0.f, best_b = 0.f, best_w = 0.f, best_h = 0.f;
  for (int k = 0; k < n; ++k) {
    // The caliper whose next edge makes the smallest angle with it advances
    // (first caliper on exact ties). OpenCV 4.13 makes this choice as exact
    // geometry, not with the rounded float cosines: compare
    // dot(caliper_i, e_i) / |e_i| across the four calipers in integers.
    long long dot[4], len2[4];
    for (int i = 0; i < 4; ++i) {
      const int j = seq[i];
      const int jn = (j + 1 < n) ? j + 1 : 0;
      const long long ex = (long long)hull[jn].x - hull[j].x, ey = (long long)hull[jn].y - hull[j].y;
      long long d;
      if (i == 0) d = Bx * ex + By * ey;
      else if (i == 1) d = -By * ex + Bx * ey;
      else if (i == 2) d = -Bx * ex - By * ey;
      else d = By * ex - Bx * ey;
      dot[i] = d;
      len2[i] = ex * ex + ey * ey;
    }
    int main = 0;
    for (int i = 1; i < 4; ++i)
      if (cos_greater(dot[i], len2[i], dot[main], len2[main])) main = i;
    const int pi = seq[main];
    const float lx = vx[pi] * ilen[pi], ly = vy[pi] * ilen[pi];
    {
      const int jn = (pi + 1 < n) ? pi + 1 : 0;
      const long long ex = (long long)hull[jn].x - hull[pi].x, ey = (long long)hull[jn].y - hull[pi].y;
      if (main == 0) { ba = lx; bb = ly; Bx = ex; By = ey; }
      else if (main == 1) { ba = ly; bb = -lx; Bx = ey; By = -ex; }
      else if (main == 2) { ba = -lx; bb = -ly; Bx = -ex; By = -ey; }
      else { ba = -ly; bb = lx; Bx = -ey; By = ex; }
    }
    seq[main] = (seq[main] + 1 == n) ? 0 : seq[main] + 1;
    float dx = (float)hull[seq[1]].x - (float)hull[seq[3]].x;
    float dy = (float)hull[seq[1]].y - (float)hull[seq[3]].y;
    const float width = dx * ba + dy * bb;
    dx = (float)hull[seq[2]].x - (float)hull[seq[0]].x;
    dy = (float)hull[seq[2]].y - (float)hull[seq[0]].y;
    const float height = -dx * bb + dy * ba;
    const float area = width * height;
    if (area <= minarea) {
      minarea = area;
      best_left = seq[3];
      best_a = ba;
      best_w = width;
      best_b = bb;
      best_h = height;
      best_bottom = seq[0];
    }
  }
  const float A1 = best_a, B1 = best_b, A2 = -best_b, B2 = best_a;
  const float C1 = A1 * (float)hull[best_left].x + (float)hull[best_left].y * B1;
  const float C2 = A2 * (float)hull[best_bottom].x + (float)hull[best_bottom].y * B2;
  const float idet = 1.f / (A1 * B2 - A2 * B1);
  const float px = (C1 * B2 - C2 * B1) * idet;
  const float py = (A1 * C2 - A2 * C1) * idet;
  const float o1x = A1 * best_w, o1y = B1 * best_w;
  const float o2x = A2 * best_h, o2y = B2 * best_h;
  if (raw6) {
    raw6[0] = px; raw6[1] = py; raw6[2] = o1x; raw6[3] = o1y; raw6[4] = o2x; raw6[5] = o2y;
  }
  r.cx = px + (o1x + o2x) * 0.5f;
  r.cy = py + (o1y + o2y) * 0.5f;
  r.w = (float)sqrt((double)o1x * o1x + (double)o1y * o1y);
  r.h = (float)sqrt((double)o2x * o2x + (double)o2y * o2y);
  return normalize_rect(r, atan2((double)o1y, (double)o1x) * 180 / 3.141592653589793238);
}

// cv::RotatedRect::points corner order.
TG void rect_points(const RRect &r, float xs[4], float ys[4]) {
  const double ang = r.angle * 3.141592653589793238 / 180.;
  const float b = (float)cos(ang) * 0.5f;
  const float a = (float)sin(ang) * 0.5f;
  xs[0] = r.cx - a * r.h - b * r.w;
  ys[0] = r.cy + b * r.h - a * r.w;
  xs[1] = r.cx + a * r.h - b * r.w;
  ys[1] = r.cy - b * r.h - a * r.w;
  xs[2] = 2 * r.cx - xs[0];
  ys[2] = 2 * r.cy - ys[0];
  xs[3] = 2 * r.cx - xs[1];
  ys[3] = 2 * r.cy - ys[1];
}

// order_quad_tl_tr_br_bl (det_postprocess.cpp:104-126): stable insertion sort
// by x, then the left pair splits into tl/bl and the right pair into tr/br by y.
TG void order_quad(float xs[4], float ys[4]) {
  for (int i = 1; i < 4; ++i) {
    const float kx = xs[i], ky = ys[i];
    int j = i - 1;
    while (j >= 0 && xs[j] > kx) {
      xs[j + 1] = xs[j];
      ys[j + 1] = ys[j];
      --j;
    }
    xs[j + 1] = kx;
    ys[j + 1] = ky;
  }
  const int tl = (ys[0] < ys[1]) ? 0 : 1, bl = 1 - tl;
  const int tr = (ys[2] < ys[3]) ? 2 : 3, br = 5 - tr;
  const float ox[4] = {xs[tl], xs[tr], xs[br], xs[bl]};
  const float oy[4] = {ys[tl], ys[tr], ys[br], ys[bl]};
  for (int k = 0; k < 4; ++k) {
    xs[k] = ox[k];
    ys[k] = oy[k];
  }
}

// std::round on float: half away from zero.
TG int round_half_away(float v) { return (int)roundf(v); }

// get_mini_boxes (det_postprocess.cpp:128-143): ordered, rounded corners.
TG void mini_box(const RRect &r, int box[8]) {
  float xs[4], ys[4];
  rect_points(r, xs, ys);
  order_quad(xs, ys);
  for (int k = 0; k < 4; ++k) {
    box[2 * k] = round_half_away(xs[k]);
    box[2 * k + 1] = round_half_away(ys[k]);
  }
}

// ------------------------------------------------------------ polygon mask --
// The pixels cv::fillPoly(LINE_8) sets for a closed contour whose edges are
// horizontal, vertical or diagonal (every CHAIN_APPROX_SIMPLE contour): the
// edge pixels plus the pixels strictly inside by the even-odd rule. For row
// y, calls span(x0, x1) (inclusive, unordered, possibly overlapping) for
// every inside run and every edge run. `xs` is scratch for up to n crossings.
template <class SPAN>
TG void poly_row_spans(const P2 *p, int n, int y, int *xs, const SPAN &span) {
  int nc = 0;
  for (int i = 0; i < n; ++i) {
    const P2 a = p[i], b = p[(i + 1 < n) ? i + 1 : 0];
    // edge pixels on this row
    if (a.y == b.y) {
      if (a.y == y) span(a.x < b.x ? a.x : b.x, a.x < b.x ? b.x : a.x);
      continue;
    }
    const int ylo = a.y < b.y ? a.y : b.y, yhi = a.y < b.y ? b.y : a.y;
    if (y < ylo || y > yhi) continue;
    // lattice point of the (vertical or diagonal) edge on row y
    const int dx = b.x - a.x, dy = b.y - a.y;
    const int x = a.x + (y - a.y) * (dx == 0 ? 0 : (dx > 0 ? 1 : -1)) * (dy > 0 ? 1 : -1);
    span(x, x);
    if (y < yhi) xs[nc++] = x;  // half-open crossing rule [ylo, yhi)
  }
  for (int i = 1; i < nc; ++i) {  // crossings in increasing x
    const int v = xs[i];
    int j = i - 1;
    while (j >= 0 && xs[j] > v) {
      xs[j + 1] = xs[j];
      --j;
    }
    xs[j + 1] = v;
  }
  for (int i = 0; i + 1 < nc; i += 2) span(xs[i], xs[i + 1]);
}

// The marks of one contour edge a -> b (horizontal, vertical or diagonal, as
// CHAIN_APPROX_SIMPLE makes them) on the rows [ya, yb]: edge(y, x0, x1) for
// its pixels on row y (inclusive, unordered) and cross(y, x) for its crossing
// of row y under the half-open rule [ylo, yhi).
template <class EDGE, class CROSS>
TG void poly_edge_marks(P2 a, P2 b, int ya, int yb, const EDGE &edge, const CROSS &cross) {
  if (a.y == b.y) {
    if (a.y >= ya && a.y <= yb) edge(a.y, a.x, b.x);
    return;
  }
  const int ylo = a.y < b.y ? a.y : b.y, yhi = a.y < b.y ? b.y : a.y;
  const int y0 = ylo > ya ? ylo : ya, y1 = yhi < yb ? yhi : yb;
  const int dx = b.x - a.x, dy = b.y - a.y;
  const int sx = (dx == 0 ? 0 : (dx > 0 ? 1 : -1)) * (dy > 0 ? 1 : -1);
  for (int y = y0; y <= y1; ++y) {
    const int x = a.x + (y - a.y) * sx;  // lattice point of the edge on row y
    edge(y, x, x);
    if (y < yhi) cross(y, x);
  }
}

// The same pixel set as poly_row_spans without sorting, for bitmask fills:
// edge(x0, x1) for every edge run (inclusive, unordered) and cross(x) for
// every crossing of the half-open rule, over edges [i0, i1) on row y. The
// row's mask is the edge runs plus the pixels where the count of crossings at
// or left of them is odd (the closing crossing of each inside run is itself
// an edge pixel).
template <class EDGE, class CROSS>
TG void poly_row_marks(const P2 *p, int n, int y, int i0, int i1, const EDGE &edge,
                       const CROSS &cross) {
  for (int i = i0; i < i1; ++i)
    poly_edge_marks(p[i], p[(i + 1 < n) ? i + 1 : 0], y, y,
                    [&](int, int x0, int x1) { edge(x0, x1); }, [&](int, int x) { cross(x); });
}

// ------------------------------------------------- area / arc length -----------
// cv::contourArea (unoriented) of an int polygon: exact in double.
TG double contour_area(const P2 *p, int n) {
  if (n < 3) return 0.;
  double a = 0.;
  P2 prev = p[n - 1];
  for (int i = 0; i < n; ++i) {
    a += (double)prev.x * p[i].y - (double)prev.y * p[i].x;
    prev = p[i];
  }
  a *= 0.5;
  return a < 0 ? -a : a;
}

// cv::arcLength(closed) of an int polygon: float segment lengths summed in double.
TG double arc_length(const P2 *p, int n) {
  if (n <= 1) return 0.;
  double per = 0.;
  float px = (float)p[n - 1].x, py = (float)p[n - 1].y;
  for (int i = 0; i < n; ++i) {
    const float x = (float)p[i].x, y = (float)p[i].y;
    const float dx = x - px, dy = y - py;
    per += sqrtf(dx * dx + dy * dy);
    px = x;
    py = y;
  }
  return per;
}

// ------------------------------------------------------------- offsetting ----
// Clipper's Round(): half away from zero on a double, to int64.
TG long long clip_round(double v) { return v < 0 ? (long long)(v - 0.5) : (long long)(v + 0.5); }

struct DP {
  double x, y;
};

// Unit normal of the edge p1 -> p2 (Clipper GetUnitNormal), FMA-contracted.
TG DP unit_normal(P2 p1, P2 p2) {
  if (p1.x == p2.x && p1.y == p2.y) return DP{0., 0.};
  double dx = (double)(p2.x - p1.x);
  double dy = (double)(p2.y - p1.y);
  const double f = 1 * 1.0 / sqrt(fma(dx, dx, dy * dy));
  dx *= f;
  dy *= f;
  return DP{dy, -dx};
}

// Prepares the offset path like ClipperOffset::AddPath + FixOrientations:
// drops trailing copies of the first point and consecutive duplicates, then
// reverses to positive orientation (Clipper's Area >= 0). Writes to q and
// returns its length (0 when fewer than 3 distinct points remain).
TG int offset_prepare(const P2 *p, int n, P2 *q) {
  if (n <= 0) return 0;
  int hi = n - 1;
  while (hi > 0 && p[0].x == p[hi].x && p[0].y == p[hi].y) --hi;
  int m = 0;
  q[m++] = p[0];
  for (int i = 1; i <= hi; ++i)
    if (q[m - 1].x != p[i].x || q[m - 1].y != p[i].y) q[m++] = p[i];
  if (m < 3) return 0;
  double a = 0.;
  for (int i = 0, j = m - 1; i < m; ++i) {
    a = fma((double)q[j].x + q[i].x, (double)q[j].y - q[i].y, a);
    j = i;
  }
  if (!(-a * 0.5 >= 0)) {
    for (int i = 0, j = m - 1; i < j; ++i, --j) {
      const P2 t = q[i];
      q[i] = q[j];
      q[j] = t;
    }
  }
  return m;
}

// offset_prepare in the form one CTA computes it: the path runs to the
// last point that differs from p[0]; a point is kept when it differs from
// its predecessor (the predecessor is always the last point kept); the
// orientation test sums the integer shoelace terms in int64, which equals
// the sequential double sum (every term is an integer, partial sums stay
// far below 2^53). Host tests compare it with offset_prepare.
TG bool prep_kept(const P2 *p, int i) {
  return i == 0 || p[i].x != p[i - 1].x || p[i].y != p[i - 1].y;
}
TG long long shoelace_term(const P2 *q, int m, int i) {
  const P2 a = q[i == 0 ? m - 1 : i - 1], b = q[i];
  return (long long)(a.x + b.x) * (long long)(a.y - b.y);
}
TG int offset_prepare_rule(const P2 *p, int n, P2 *q) {
  if (n <= 0) return 0;
  int hi = 0;
  for (int i = 0; i < n; ++i)
    if (p[i].x != p[0].x || p[i].y != p[0].y) hi = i;
  int m = 0;
  for (int i = 0; i <= hi; ++i)
    if (prep_kept(p, i)) q[m++] = p[i];
  if (m < 3) return 0;
  long long a = 0;
  for (int i = 0; i < m; ++i) a += shoelace_term(q, m, i);
  if (a > 0)
    for (int i = 0, j = m - 1; i < j; ++i, --j) {
      const P2 t = q[i];
      q[i] = q[j];
      q[j] = t;
    }
  return m;
}

// Per-call constants of the round joins (ClipperOffset::DoOffset).
struct OffsetConsts {
  double m_sin, m_cos, steps_per_rad;
};
TG OffsetConsts offset_consts(double delta) {
  const double ad = delta < 0 ? -delta : delta;
  const double y = (0.25 > ad * 0.25) ? ad * 0.25 : 0.25;
  const double pi = 3.141592653589793238, two_pi = pi * 2;
  double steps = pi / acos(1 - y / ad);
  if (steps > ad * pi) steps = ad * pi;
  OffsetConsts oc;
  oc.m_sin = sin(two_pi / steps);
  oc.m_cos = cos(two_pi / steps);
  oc.steps_per_rad = steps / two_pi;
  if (delta < 0.0) oc.m_sin = -oc.m_sin;
  return oc;
}

// One vertex j of the offset (ClipperOffset::OffsetPoint + DoRound) with
// previous vertex k: calls emit(x, y) for its points. Returns true when
// Clipper keeps k for the next vertex (the early return for a nearly
// straight joint), false when k becomes j.
template <class EMIT>
TG bool offset_vertex(const P2 *q, int m, int j, int k, double delta, const OffsetConsts &oc,
                      EMIT &&emit) {
  const DP nk = unit_normal(q[k], q[(k + 1) % m]);
  const DP nj = unit_normal(q[j], q[(j + 1) % m]);
  double sinA = fma(nk.x, nj.y, -(nj.x * nk.y));
  if (fabs(sinA * delta) < 1.0) {
    const double cosA = fma(nk.x, nj.x, nj.y * nk.y);
    if (cosA > 0) {
      emit(clip_round(fma(nk.x, delta, (double)q[j].x)), clip_round(fma(nk.y, delta, (double)q[j].y)));
      return true;
    }
  } else if (sinA > 1.0) {
    sinA = 1.0;
  } else if (sinA < -1.0) {
    sinA = -1.0;
  }
  if (sinA * delta < 0) {
    emit(clip_round(fma(nk.x, delta, (double)q[j].x)), clip_round(fma(nk.y, delta, (double)q[j].y)));
    emit(q[j].x, q[j].y);
    emit(clip_round(fma(nj.x, delta, (double)q[j].x)), clip_round(fma(nj.y, delta, (double)q[j].y)));
  } else {
    const double a = atan2(sinA, fma(nk.x, nj.x, nk.y * nj.y));
    long long st = clip_round(oc.steps_per_rad * fabs(a));
    const int steps_i = st > 1 ? (int)st : 1;
    double X = nk.x, Y = nk.y;
    for (int i = 0; i < steps_i; ++i) {
      emit(clip_round(fma(X, delta, (double)q[j].x)), clip_round(fma(Y, delta, (double)q[j].y)));
      const double X2 = X;
      X = fma(X, oc.m_cos, -(oc.m_sin * Y));
      Y = fma(X2, oc.m_sin, Y * oc.m_cos);
    }
    emit(clip_round(fma(nj.x, delta, (double)q[j].x)), clip_round(fma(nj.y, delta, (double)q[j].y)));
  }
  return false;
}

TG bool offset_is_identity(double delta) { return delta > -1.0E-20 && delta < 1.0E-20; }

// Raw round-join offset of the prepared closed path q[0..m) by delta
// (ClipperOffset::DoOffset, before the union): calls emit(x, y) for each ring
// point in order and returns their count.
template <class EMIT>
TG int offset_emit(const P2 *q, int m, double delta, EMIT &&emit_out) {
  int n = 0;
  auto emit = [&](long long x, long long y) {
    emit_out(x, y);
    ++n;
  };
  if (offset_is_identity(delta)) {
    for (int i = 0; i < m; ++i) emit(q[i].x, q[i].y);
    return n;
  }
  const OffsetConsts oc = offset_consts(delta);
  int k = m - 1;
  for (int j = 0; j < m; ++j)
    if (!offset_vertex(q, m, j, k, delta, oc, emit)) k = j;
  return n;
}

// offset_emit into out: writes at most cap points, returns the full count.
TG int offset_raw(const P2 *q, int m, double delta, P2 *out, int cap) {
  int n = 0;
  return offset_emit(q, m, delta, [&](long long x, long long y) {
    if (n < cap) out[n] = P2{(int)x, (int)y};
    ++n;
  });
}

// Winding number (crossing rule) of the point (x, y) w.r.t. the closed path r[0..n).
TG int winding_number(const P2 *r, int n, double x, double y) {
  int wn = 0;
  for (int i = 0; i < n; ++i) {
    const double x1 = r[i].x, y1 = r[i].y;
    const int j = (i + 1 < n) ? i + 1 : 0;
    const double x2 = r[j].x, y2 = r[j].y;
    const double c = (x2 - x1) * (y - y1) - (x - x1) * (y2 - y1);
    if (y1 <= y) {
      if (y2 > y && c > 0) ++wn;
    } else {
      if (y2 <= y && c < 0) --wn;
    }
  }
  return wn;
}

// True when some point arbitrarily close to (x, y) has positive winding,
// i.e. (x, y) lies in the closure of the union's positive-fill region.
TG bool in_positive_closure(const P2 *r, int n, int x, int y) {
  const double off[8][2] = {{0.3125, 0.0625}, {-0.3125, -0.0625}, {0.0625, -0.3125},
                            {-0.0625, 0.3125}, {0.1875, 0.1875}, {-0.1875, -0.1875},
                            {0.1875, -0.1875}, {-0.1875, 0.1875}};
  for (int k = 0; k < 8; ++k)
    if (winding_number(r, n, x + off[k][0], y + off[k][1]) > 0) return true;
  return false;
}

// Exact intersection of segments ab and cd rounded half away from zero.
TG bool seg_intersect_round(P2 a, P2 b, P2 c, P2 d, P2 &out) {
  const long long x1 = a.x, y1 = a.y, x2 = b.x, y2 = b.y;
  const long long x3 = c.x, y3 = c.y, x4 = d.x, y4 = d.y;
  long long den = (x1 - x2) * (y3 - y4) - (y1 - y2) * (x3 - x4);
  if (den == 0) return false;
  long long tn = (x1 - x3) * (y3 - y4) - (y1 - y3) * (x3 - x4);
  long long un = (x1 - x3) * (y1 - y2) - (y1 - y3) * (x1 - x2);
  if (den < 0) { den = -den; tn = -tn; un = -un; }
  if (tn < 0 || tn > den || un < 0 || un > den) return false;
  // x = x1 + tn (x2 - x1) / den, rounded half away from zero
  auto rdiv = [](long long num, long long dd) -> long long {  // dd > 0
    const long long q = num >= 0 ? (2 * num + dd) / (2 * dd) : -((-2 * num + dd) / (2 * dd));
    return q;
  };
  const long long nx = x1 * den + tn * (x2 - x1);
  const long long ny = y1 * den + tn * (y2 - y1);
  out = P2{(int)rdiv(nx, den), (int)rdiv(ny, den)};
  return true;
}

}  // namespace db
}  // namespace tocr
