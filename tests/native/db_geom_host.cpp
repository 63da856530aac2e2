// Test-only host build of turboocr_b200/csrc/db_geom.cuh: exposes the DB
// geometry routines over a C ABI so the CPU tests can compare them, routine
// by routine, with OpenCV and with the reference's Clipper. Built by the
// tests themselves (tests/db_native.py); never linked into the product.
#include <algorithm>
#include <cstring>
#include <vector>

#include "clipper_union.cuh"
#include "db_geom.cuh"

using namespace tocr::db;

extern "C" {

// Border following from one start pixel; returns the point count.
int dbh_trace(const unsigned char *bm, int H, int W, int x0, int y0, int hole, int *out, int cap) {
  auto fg = [&](int x, int y) { return x >= 0 && y >= 0 && x < W && y < H && bm[y * W + x] != 0; };
  return trace_border(fg, x0, y0, hole != 0, reinterpret_cast<P2 *>(out), cap, 64 * W * H + 64);
}

// Same walk through the bit-packed neighbourhood provider used on the device.
int dbh_trace_bits(const unsigned char *bm, int H, int W, int x0, int y0, int hole, int *out,
                   int cap) {
  const int words = (W + 31) / 32;
  std::vector<uint32_t> bits((size_t)H * words, 0u);
  for (int y = 0; y < H; ++y)
    for (int x = 0; x < W; ++x)
      if (bm[y * W + x]) bits[(size_t)y * words + (x >> 5)] |= 1u << (x & 31);
  NbBits nb{bits.data(), H, W, words};
  return trace_border_nb(nb, x0, y0, hole != 0, reinterpret_cast<P2 *>(out), cap, 64 * W * H + 64);
}

int dbh_hull(const int *pts, int n, int *out) {
  std::vector<HP> work(2 * n + 2);
  return convex_hull(reinterpret_cast<const P2 *>(pts), n, work.data(), reinterpret_cast<P2 *>(out));
}

// The device's shared-memory hull: the column table (lowest / highest point
// of every x column, first index), chain over its candidates. Returns the
// hull size (-1: more than hull_cap vertices, -2: more than col_cap columns).
// filter != 0: candidates strictly inside the polygon of the extreme points
// of kExtDirs directions are dropped first (the device's interior filter).
int dbh_hull_table(const int *pts, int n, int *out, int col_cap, int hull_cap, int filter) {
  if (n <= 0) return 0;
  int x0 = pts[0], x1 = pts[0];
  for (int i = 1; i < n; ++i) {
    x0 = std::min(x0, pts[2 * i]);
    x1 = std::max(x1, pts[2 * i]);
  }
  const int ncols = x1 - x0 + 1;
  if (ncols > col_cap) return -2;
  std::vector<uint64_t> lo(ncols, kColEmpty), hi(ncols, kColEmpty);
  for (int i = 0; i < n; ++i) col_add(lo.data(), hi.data(), pts[2 * i] - x0, pts[2 * i + 1], i);
  std::vector<int> stk(2 * (size_t)ncols + 2);
  std::vector<uint32_t> keep((2 * (size_t)ncols + 31) / 32, 0u);
  if (filter) {
    HP ext[kExtDirs];
    long long best[kExtDirs];
    bool any = false;
    HP v;
    for (int e = 0; e < 2 * ncols; ++e) {
      if (!col_entry(lo.data(), hi.data(), x0, e, &v)) continue;
      for (int k = 0; k < kExtDirs; ++k) {
        const long long d = ext_dot(k, v.x, v.y);
        if (!any || d > best[k]) { best[k] = d; ext[k] = v; }
      }
      any = true;
    }
    for (int e = 0; e < 2 * ncols; ++e)
      if (col_entry(lo.data(), hi.data(), x0, e, &v) && !strictly_inside_extremes(ext, kExtDirs, v))
        keep[e >> 5] |= 1u << (e & 31);
  }
  return hull_from_table(lo.data(), hi.data(), ncols, x0, stk.data(), reinterpret_cast<P2 *>(out),
                         hull_cap, filter ? keep.data() : nullptr);
}

// offset_prepare (rule != 0: in the CTA form, offset_prepare_rule); returns
// the prepared length, out holds it.
int dbh_offset_prepare(const int *pts, int n, int *out, int rule) {
  const P2 *p = reinterpret_cast<const P2 *>(pts);
  P2 *q = reinterpret_cast<P2 *>(out);
  return rule ? offset_prepare_rule(p, n, q) : offset_prepare(p, n, q);
}

// Offset ring through the per-vertex form with k = j - 1 for every vertex
// (the device's parallel emission): returns the count, or -1 when some vertex
// before the last keeps k (the device then emits serially).
int dbh_offset_parallel(const int *pts, int n, double delta, int *out, int cap) {
  std::vector<P2> q(n + 1);
  const int m = offset_prepare(reinterpret_cast<const P2 *>(pts), n, q.data());
  if (m == 0 || offset_is_identity(delta)) return -1;
  const OffsetConsts oc = offset_consts(delta);
  int cnt = 0;
  for (int j = 0; j < m; ++j) {
    const bool keep = offset_vertex(q.data(), m, j, j == 0 ? m - 1 : j - 1, delta, oc,
                                    [&](long long x, long long y) {
                                      if (cnt < cap) { out[2 * cnt] = (int)x; out[2 * cnt + 1] = (int)y; }
                                      ++cnt;
                                    });
    if (keep && j < m - 1) return -1;
  }
  return cnt;
}

// minAreaRect of a point sequence: writes cx, cy, w, h, angle.
void dbh_min_area_rect(const int *pts, int n, float *out5) {
  std::vector<HP> work(2 * n + 2);
  std::vector<P2> hull(n + 1);
  const int m = convex_hull(reinterpret_cast<const P2 *>(pts), n, work.data(), hull.data());
  std::vector<float> scratch(3 * m + 3);
  RRect r = min_area_rect(hull.data(), m, scratch.data());
  out5[0] = r.cx; out5[1] = r.cy; out5[2] = r.w; out5[3] = r.h; out5[4] = r.angle;
}

void dbh_mini_box(const int *pts, int n, int *box8, float *min_side) {
  std::vector<HP> work(2 * n + 2);
  std::vector<P2> hull(n + 1);
  const int m = convex_hull(reinterpret_cast<const P2 *>(pts), n, work.data(), hull.data());
  std::vector<float> scratch(3 * m + 3);
  RRect r = min_area_rect(hull.data(), m, scratch.data());
  *min_side = r.w < r.h ? r.w : r.h;
  mini_box(r, box8);
}

void dbh_mar_raw(const int *pts, int n, float *raw6) {
  std::vector<HP> work(2 * n + 2);
  std::vector<P2> hull(n + 1);
  const int m = convex_hull(reinterpret_cast<const P2 *>(pts), n, work.data(), hull.data());
  std::vector<float> scratch(3 * m + 3);
  (void)min_area_rect(hull.data(), m, scratch.data(), raw6);
}

// Polygon mask of a contour over its bounding box [x0, x0+w) x [y0, y0+h).
void dbh_poly_mask(const int *pts, int n, int x0, int y0, int w, int h, unsigned char *mask) {
  std::vector<int> xs(n + 1);
  memset(mask, 0, (size_t)w * h);
  for (int y = y0; y < y0 + h; ++y)
    poly_row_spans(reinterpret_cast<const P2 *>(pts), n, y, xs.data(), [&](int a, int b) {
      if (a > b) { int t = a; a = b; b = t; }
      for (int x = a; x <= b; ++x)
        if (x >= x0 && x < x0 + w) mask[(size_t)(y - y0) * w + (x - x0)] = 1;
    });
}

// Same mask through poly_row_marks: edge runs | odd crossing parity.
void dbh_poly_mask_parity(const int *pts, int n, int x0, int y0, int w, int h, unsigned char *mask) {
  memset(mask, 0, (size_t)w * h);
  std::vector<unsigned char> tog(w + 1);
  for (int y = y0; y < y0 + h; ++y) {
    std::fill(tog.begin(), tog.end(), 0);
    unsigned char *row = mask + (size_t)(y - y0) * w;
    poly_row_marks(reinterpret_cast<const P2 *>(pts), n, y, 0, n,
        [&](int a, int b) {
          if (a > b) { int t = a; a = b; b = t; }
          for (int x = a; x <= b; ++x)
            if (x >= x0 && x < x0 + w) row[x - x0] = 1;
        },
        [&](int x) { if (x >= x0 && x < x0 + w) tog[x - x0] ^= 1; });
    int par = 0;
    for (int x = 0; x < w; ++x) {
      par ^= tog[x];
      if (par) row[x] = 1;
    }
  }
}

double dbh_area(const int *pts, int n) { return contour_area(reinterpret_cast<const P2 *>(pts), n); }
double dbh_arclen(const int *pts, int n) { return arc_length(reinterpret_cast<const P2 *>(pts), n); }

int dbh_offset_raw(const int *pts, int n, double delta, int *out, int cap) {
  std::vector<P2> q(n + 1);
  const int m = offset_prepare(reinterpret_cast<const P2 *>(pts), n, q.data());
  if (m == 0) return 0;
  return offset_raw(q.data(), m, delta, reinterpret_cast<P2 *>(out), cap);
}

}  // extern "C"

// unclip() with Clipper's union (clipper_union.cuh) on the raw offset: the
// largest output ring in path order. Returns its length, 0 for an empty
// solution, -1 when the sweep failed, -2 when out is too small.
extern "C" int dbh_unclip_union(const int *pts, int n, double delta, int *out, int cap) {
  std::vector<P2> q(n + 1);
  const int m = offset_prepare(reinterpret_cast<const P2 *>(pts), n, q.data());
  if (m == 0) return 0;
  const int rn = offset_raw(q.data(), m, delta, nullptr, 0);
  if (rn <= 0) return 0;
  std::vector<P2> ring(rn);
  offset_raw(q.data(), m, delta, ring.data(), rn);
  std::vector<char> arena(cu::arena_bytes(rn) + 64);
  cu::Sweep s;
  s.init(arena.data(), rn);
  if (!s.execute(ring.data(), rn)) return -1;
  const int k = s.best_ring(reinterpret_cast<P2 *>(out), cap);
  return k < 0 ? (s.fail ? -1 : -2) : k;
}

// Peak use of the sweep's arrays for one unclip (test of the capacities).
extern "C" int dbh_union_usage(const int *pts, int n, double delta, int *use) {
  std::vector<P2> q(n + 1);
  const int m = offset_prepare(reinterpret_cast<const P2 *>(pts), n, q.data());
  if (m == 0) return 0;
  std::vector<P2> ring(1 << 20);
  const int rn = offset_raw(q.data(), m, delta, ring.data(), 1 << 20);
  if (rn <= 0) return 0;
  std::vector<char> arena(cu::arena_bytes(rn) + 64);
  cu::Sweep s;
  s.init(arena.data(), rn);
  const bool ok = s.execute(ring.data(), rn);
  use[0] = rn; use[1] = s.n_lm; use[2] = s.n_op; use[3] = s.n_or; use[4] = s.n_jn;
  use[5] = (int)s.guard;
  return ok ? 1 : -1;
}

// std_sort (libstdc++'s introsort restated in clipper_union.cuh) against the
// host's std::sort on the same keys: both permutations of 0..n-1, keys
// compared by descending value as Clipper's sorts do.
#include <algorithm>
extern "C" int dbh_sort_check(const int *keys, int n, int *perm_std, int *perm_own) {
  struct K { int key, id; };
  std::vector<K> a(n), b(n);
  for (int i = 0; i < n; ++i) a[i] = b[i] = K{keys[i], i};
  auto less = [](const K &x, const K &y) { return y.key < x.key; };
  std::sort(a.begin(), a.end(), less);
  std::vector<int> stk(3 * 64);
  bool fail = false;
  cu::std_sort(b.data(), n, less, stk.data(), 64, &fail);
  for (int i = 0; i < n; ++i) { perm_std[i] = a[i].id; perm_own[i] = b[i].id; }
  return fail ? -1 : 0;
}

// ---- warp emulation for the union sweep's list-wide steps -------------------
// dbh_set_union_lanes(n): with n > 1, every list-wide step of the sweep runs
// on n threads (this one is lane 0) that meet at a std::barrier wherever the
// device's lanes meet at __syncwarp, so the CPU tests cover the split of each
// step over the 32 lanes of a warp. n <= 1 restores the single-thread steps.
#include <barrier>
#include <memory>
#include <thread>

namespace {
struct LanePool {
  int n = 0;
  std::unique_ptr<std::barrier<>> bar;
  std::vector<std::thread> th;
  cu::BulkArgs *job = nullptr;
  bool stop = false;
  void start(int lanes) {
    n = lanes;
    bar = std::make_unique<std::barrier<>>(lanes);
    for (int l = 1; l < lanes; ++l)
      th.emplace_back([this, l] {
        for (;;) {
          bar->arrive_and_wait();  // job posted
          if (stop) return;
          cu::bulk_exec(*job, l, n);
          bar->arrive_and_wait();  // job done
        }
      });
  }
  void run(cu::BulkArgs *a) {
    job = a;
    bar->arrive_and_wait();
    cu::bulk_exec(*a, 0, n);
    bar->arrive_and_wait();
  }
  void shutdown() {
    if (!bar) return;
    stop = true;
    bar->arrive_and_wait();
    for (auto &t : th) t.join();
    th.clear();
    bar.reset();
    stop = false;
    n = 0;
  }
};
LanePool g_pool;
}  // namespace

extern "C" void dbh_set_union_lanes(int n) {
  g_pool.shutdown();
  if (n <= 1) {
    cu::g_host_lanes = 1;
    cu::g_host_runner = nullptr;
    cu::g_host_barrier = nullptr;
    return;
  }
  g_pool.start(n);
  cu::g_host_lanes = n;
  cu::g_host_runner = [](cu::BulkArgs *a, int) { g_pool.run(a); };
  cu::g_host_barrier = [] { g_pool.bar->arrive_and_wait(); };
}
