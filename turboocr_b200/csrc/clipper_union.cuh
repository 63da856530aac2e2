// The union step of the reference's unclip(): ClipperOffset::Execute
// (Clipper 6.4.2, third_party/clipper/clipper.cpp:3887-3915) passes the raw
// round-join offset path through Clipper::Execute(ctUnion, pftPositive,
// pftPositive) (clipper.cpp:1508-1622), and unclip keeps the output ring of
// largest signed area (src/detection/det_postprocess.cpp:86-93).
//
// Bit-exact box vertices need the same output ring, so this is a restatement
// of that sweep (Vatti's algorithm as Clipper implements it) for exactly the
// case unclip uses: one closed subject path, positive fill on both sides, no
// clip paths, collinear points not preserved, not strictly simple, Paths
// output, coordinates below 2^30 (Clipper's 64-bit slope products). The steps
// and tie-breaks are Clipper's, because its integer rounding of intersection
// points, its scanbeam clamps and its polygon building decide which vertices
// the ring has: edge construction and local minima (AddPath, ProcessBound,
// FindNextLocMin), the scanbeam loop (ExecuteInternal), AEL insertion
// (E2InsertsBeforeE1), winding counts and contribution (SetWindingCount,
// IsContributing for this fill), IntersectEdges, horizontals
// (ProcessHorizontal), the per-scanbeam intersection list (bubble sort,
// libstdc++ std::sort by y, adjacency fixup), maxima and intermediate
// vertices, output polygon linking (AddOutPt, AddLocalMin/MaxPoly,
// AppendPolygon), joins (JoinCommonEdges, JoinPoints, JoinHorz) and the final
// FixupOutPolygon. The data layout is this file's own: every object lives in
// caller-provided arrays and is named by an int index (-1 = none), so one GPU
// thread can run the sweep in a slab of global memory.
//
// std::sort is not stable; which of two equal keys comes first is fixed by
// libstdc++'s introsort (median-of-three quicksort above 16 elements, heap
// sort past depth 2*log2(n), then insertion sort), restated in std_sort().
//
// Robustness: every allocation is bounded by the arena's capacities and
// every list walk by the number of objects in existence. When a bound is hit
// the sweep stops with fail set; the caller then discards the result.
#pragma once

#include <cmath>
#include <cstdint>

#include "db_geom.cuh"

#if defined(__CUDACC__)
#define CU_HD __host__ __device__
#else
#define CU_HD
#endif

namespace tocr {
namespace db {
namespace cu {

constexpr int kNil = -1;
constexpr int kUnassigned = -1;
constexpr double kHorizontal = -1.0E+40;
constexpr int kSideLeft = 1, kSideRight = 2;
constexpr long long kCoordLimit = 0x3FFFFFFFLL;

// Coordinates are stored as int (the caller checks |v| <= 2^30); every
// product and sum that Clipper forms on them is taken in 64 bits.
struct Edge {
  int bx, by, cx, cy, tx, ty;  // Bot, Curr, Top
  double dx;
  int wdelta, wcnt, wcnt2, out_idx, side;
  int next, prev, next_lml, ael_pos, next_sel, prev_sel;
};
struct OutPt {
  int idx;
  int next, prev;
  int x, y;
};
struct OutRec {
  int idx, is_hole, first_left, pts, bottom_pt;
};
struct LocMin {
  long long y;
  int left, right;
};
struct Join {
  int op1, op2;
  int offx, offy;
};
struct INode {
  int e1, e2;
  int x, y;
};

// Capacities of one sweep's arrays, from the path length n.
struct Caps {
  int edges, minima, scan, outpts, outrecs, joins, ghosts, inodes, stack;
};
// per-scanbeam work arrays of the intersection list: 3 x edges + 1 x inodes
// ints and a second INode array
TG Caps caps_for(int n) {
  Caps c;
  // Peak use measured over ~50k contours (noise, rotated shapes, text maps,
  // rings up to 22k points): out points 1.11 n, out records 0.22 n, joins
  // 0.14 n, local minima 0.22 n. Overflow is detected, never silent.
  c.edges = n;
  c.minima = n / 2 + 2;
  c.scan = 2 * n + 8;
  c.outpts = 2 * n + 16;
  c.outrecs = n / 2 + 8;
  c.joins = n / 2 + 8;
  c.ghosts = n / 4 + 8;
  c.inodes = n + 16;
  c.stack = 64;  // introsort depth <= 2 log2(n) + 1
  return c;
}
// Bytes of the arena for a path of n points (16-byte aligned sections).
TG unsigned long long arena_bytes(int n) {
  const Caps c = caps_for(n);
  auto al = [](unsigned long long b) { return (b + 15ull) & ~15ull; };
  return al(sizeof(Edge) * (unsigned long long)c.edges) +
         al(sizeof(LocMin) * (unsigned long long)c.minima) +
         al(sizeof(long long) * (unsigned long long)c.scan) +
         al(sizeof(OutPt) * (unsigned long long)(c.outpts + 1)) +
         al(sizeof(OutRec) * (unsigned long long)(c.outrecs + 1)) +
         al(sizeof(Join) * (unsigned long long)c.joins) +
         al(sizeof(Join) * (unsigned long long)c.ghosts) +
         al(sizeof(INode) * (unsigned long long)c.inodes) +
         al(sizeof(int) * 3ull * (unsigned long long)c.stack) +
         al(sizeof(int) * 4ull * (unsigned long long)(c.edges + 2)) +
         al(sizeof(int) * (unsigned long long)c.inodes) +
         al(sizeof(INode) * (unsigned long long)c.inodes) +
         al(sizeof(int) * 3ull * (unsigned long long)(c.edges + 2));
}

// ------------------------------------------------------------ std::sort -------
// libstdc++'s std::sort (introsort) on a[0..n), with `less` the comparator.
template <class T, class Less>
CU_HD void std_sort(T *a, int n, Less less, int *stk, int stk_cap, bool *fail) {
  if (n <= 1) return;
  auto lg = [](int v) { int r = 0; while (v >>= 1) ++r; return r; };
  auto sw = [&](int i, int j) { T t = a[i]; a[i] = a[j]; a[j] = t; };
  auto adjust_heap = [&](int first, int hole, int len, T value) {
    const int top = hole;
    int child = hole;
    while (child < (len - 1) / 2) {
      child = 2 * (child + 1);
      if (less(a[first + child], a[first + child - 1])) --child;
      a[first + hole] = a[first + child];
      hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
      child = 2 * (child + 1);
      a[first + hole] = a[first + child - 1];
      hole = child - 1;
    }
    int parent = (hole - 1) / 2;
    while (hole > top && less(a[first + parent], value)) {
      a[first + hole] = a[first + parent];
      hole = parent;
      parent = (hole - 1) / 2;
    }
    a[first + hole] = value;
  };
  auto heap_sort = [&](int first, int last) {
    const int len = last - first;
    if (len >= 2) {
      for (int parent = (len - 2) / 2;; --parent) {
        adjust_heap(first, parent, len, a[first + parent]);
        if (parent == 0) break;
      }
    }
    for (int l = last; l - first > 1;) {
      --l;
      T value = a[l];
      a[l] = a[first];
      adjust_heap(first, 0, l - first, value);
    }
  };
  // introsort loop with an explicit stack of (first, last, depth)
  int sp = 0;
  stk[0] = 0; stk[1] = n; stk[2] = lg(n) * 2;
  sp = 1;
  while (sp > 0) {
    --sp;
    int first = stk[3 * sp], last = stk[3 * sp + 1], depth = stk[3 * sp + 2];
    while (last - first > 16) {
      if (depth == 0) {
        heap_sort(first, last);
        break;
      }
      --depth;
      const int mid = first + (last - first) / 2;
      // move the median of (first+1, mid, last-1) to first
      const int x = first + 1, y = mid, z = last - 1;
      if (less(a[x], a[y])) {
        if (less(a[y], a[z])) sw(first, y);
        else if (less(a[x], a[z])) sw(first, z);
        else sw(first, x);
      } else if (less(a[x], a[z])) sw(first, x);
      else if (less(a[y], a[z])) sw(first, z);
      else sw(first, y);
      // unguarded partition of (first+1, last) around a[first]
      int lo = first + 1, hi = last;
      for (;;) {
        while (less(a[lo], a[first])) ++lo;
        --hi;
        while (less(a[first], a[hi])) --hi;
        if (!(lo < hi)) break;
        sw(lo, hi);
        ++lo;
      }
      const int cut = lo;
      if (sp >= stk_cap) { *fail = true; return; }
      stk[3 * sp] = cut; stk[3 * sp + 1] = last; stk[3 * sp + 2] = depth;
      ++sp;
      last = cut;
    }
  }
  // final insertion sort
  auto linear_insert = [&](int i) {
    T val = a[i];
    int j = i - 1;
    while (less(val, a[j])) { a[j + 1] = a[j]; --j; }
    a[j + 1] = val;
  };
  auto insertion_sort = [&](int first, int last) {
    for (int i = first + 1; i < last; ++i) {
      if (less(a[i], a[first])) {
        T val = a[i];
        for (int j = i; j > first; --j) a[j] = a[j - 1];
        a[first] = val;
      } else {
        linear_insert(i);
      }
    }
  };
  if (n > 16) {
    insertion_sort(0, 16);
    for (int i = 16; i < n; ++i) linear_insert(i);
  } else {
    insertion_sort(0, n);
  }
}

// ------------------------------------------------------- list-wide steps -------
// The sweep's per-scanbeam passes over the whole active edge list (AEL): the
// edges' x at the scanbeam top, the clusters of the intersection sort, the
// update of every edge at the top, the list of edges that end there, the
// SEL copy, the array shifts of insertions and deletions and the linear
// searches. Each is a pure data-parallel step with a fixed result, written
// once for nl lanes: the host runs it with one lane; on the device the
// warp that owns a ring runs it with 32 lanes while lane 0 keeps Clipper's
// sequential logic (bulk_step). Chunks are contiguous, lane order is list
// order, and partial results meet in the per-lane arrays, so the outcome
// does not depend on nl.
enum BulkOp : int {
  kOpStop = 0, kOpKeys, kOpTop, kOpPromote, kOpSel, kOpInsert, kOpDelete, kOpFindIns, kOpFindOut
};
constexpr int kMaxLanes = 32;
struct BulkArgs {
  int op, a, b, n, result;
  long long y;
  Edge *E;
  int *AEL, *ARR, *KEY, *SUF, *SPL, *CLS;
  int p0[kMaxLanes], p1[kMaxLanes], p2[kMaxLanes], p3[kMaxLanes];
};

TG long long round_half_away_ll(double v) { return v < 0 ? (long long)(v - 0.5) : (long long)(v + 0.5); }
TG long long edge_top_x(const Edge &e, long long y) {
  return y == e.ty ? (long long)e.tx : (long long)e.bx + round_half_away_ll(e.dx * (double)(y - e.by));
}
// Clipper's E2InsertsBeforeE1
TG bool inserts_before(const Edge *E, int e1, int e2) {
  if (E[e2].cx == E[e1].cx) {
    if (E[e2].ty > E[e1].ty) return E[e2].tx < edge_top_x(E[e1], E[e2].ty);
    return E[e1].tx > edge_top_x(E[e2], E[e1].ty);
  }
  return E[e2].cx < E[e1].cx;
}

#if !defined(__CUDA_ARCH__)
// Host emulation of the warp (tests): g_host_lanes lanes run each step as
// threads through g_host_runner and meet at g_host_barrier.
inline int g_host_lanes = 1;
inline void (*g_host_runner)(BulkArgs *, int) = nullptr;
inline void (*g_host_barrier)() = nullptr;
#endif

TG void bulk_sync(int nl) {
#if defined(__CUDA_ARCH__)
  if (nl > 1) __syncwarp();
#else
  if (nl > 1 && g_host_barrier) g_host_barrier();
#endif
}

// First list position p >= p0 (p < n) where pred(p) holds, else n; rounds of
// nl positions.
template <class PRED>
TG int bulk_find(BulkArgs &A, int lane, int nl, int p0, int n, PRED pred) {
  for (int base = p0; base < n; base += nl) {
    const int p = base + lane;
    A.p0[lane] = (p < n && pred(p)) ? 1 : 0;
    bulk_sync(nl);
    int hit = -1;
    for (int j = 0; j < nl; ++j)
      if (A.p0[j]) { hit = base + j; break; }
    bulk_sync(nl);
    if (hit >= 0) return hit;
  }
  return n;
}

// Exclusive sum of v over the lanes (all lanes get their offset; *total the sum).
TG int bulk_offset(BulkArgs &A, int lane, int nl, int v, int *total) {
  A.p2[lane] = v;
  bulk_sync(nl);
  int off = 0, all = 0;
  for (int j = 0; j < nl; ++j) {
    if (j < lane) off += A.p2[j];
    all += A.p2[j];
  }
  bulk_sync(nl);
  *total = all;
  return off;
}

TG void bulk_exec(BulkArgs &A, int lane, int nl) {
  Edge *E = A.E;
  int *AEL = A.AEL;
  const int n = A.n;
  const int ch = (n + nl - 1) / nl;
  const int lo = lane * ch < n ? lane * ch : n;
  const int hi = lo + ch < n ? lo + ch : n;
  switch (A.op) {
    case kOpKeys: {
      // x at the top of every edge (Curr.X), the sort copy (ARR, KEY); then
      // the clusters of the bubble sort: cut after position i when every key
      // up to i is <= every key after i; clusters of two or more positions
      // (they hold an inversion) go to CLS as (first, last) in list order.
      const long long y = A.y;
      int cmin = 0x7fffffff, cmax = (int)0x80000000;
      for (int k = lo; k < hi; ++k) {
        const int e = AEL[k];
        const int x = (int)edge_top_x(E[e], y);
        E[e].cx = x;
        A.ARR[k] = e;
        A.KEY[k] = x;
        cmin = x < cmin ? x : cmin;
        cmax = x > cmax ? x : cmax;
      }
      A.p0[lane] = cmin;
      A.p1[lane] = cmax;
      bulk_sync(nl);
      int desc = 0;
      for (int k = lo; k < hi; ++k)
        if (k + 1 < n && A.KEY[k] > A.KEY[k + 1]) { desc = 1; break; }
      int any = 0;
      bulk_offset(A, lane, nl, desc, &any);
      if (any == 0) {
        if (lane == 0) A.result = 0;
        return;
      }
      int pm_in = (int)0x80000000, sm_in = 0x7fffffff;
      for (int j = 0; j < nl; ++j) {
        if (j < lane) pm_in = A.p1[j] > pm_in ? A.p1[j] : pm_in;
        if (j > lane) sm_in = A.p0[j] < sm_in ? A.p0[j] : sm_in;
      }
      {  // suffix minima of the chunk, seeded with the later chunks' minimum
        int sm = sm_in;
        for (int k = hi - 1; k >= lo; --k) {
          sm = A.KEY[k] < sm ? A.KEY[k] : sm;
          A.SUF[k] = sm;
        }
      }
      // cut flags (i is a cut when max KEY[0..i] <= min KEY[i+1..n)); the
      // last cut of each chunk, for the cluster starts of the next chunks
      auto suf_after = [&](int i) { return i + 1 < hi ? A.SUF[i + 1] : sm_in; };
      int last_cut = -1, pm = pm_in;
      for (int i = lo; i < hi; ++i) {
        pm = A.KEY[i] > pm ? A.KEY[i] : pm;
        if (i == n - 1 || pm <= suf_after(i)) last_cut = i;
      }
      A.p3[lane] = last_cut;
      bulk_sync(nl);
      int prev = -1;
      for (int j = 0; j < lane; ++j) prev = A.p3[j] > prev ? A.p3[j] : prev;
      int cnt = 0;
      {
        int pv = prev, p2 = pm_in;
        for (int i = lo; i < hi; ++i) {
          p2 = A.KEY[i] > p2 ? A.KEY[i] : p2;
          if (i == n - 1 || p2 <= suf_after(i)) {
            if (i > pv + 1) ++cnt;
            pv = i;
          }
        }
      }
      int total = 0;
      int off = bulk_offset(A, lane, nl, cnt, &total);
      {
        int pv = prev, p2 = pm_in;
        for (int i = lo; i < hi; ++i) {
          p2 = A.KEY[i] > p2 ? A.KEY[i] : p2;
          if (i == n - 1 || p2 <= suf_after(i)) {
            if (i > pv + 1) {
              A.CLS[2 * off] = pv + 1;
              A.CLS[2 * off + 1] = i;
              ++off;
            }
            pv = i;
          }
        }
      }
      if (lane == 0) A.result = total;
      return;
    }
    case kOpTop:
    case kOpPromote: {
      // kOpTop: every edge that does not end at y gets its x and y at y
      // (Curr); the edges that end at y are listed in SPL in list order.
      // kOpPromote: the edges that end at y and go on (NextInLML) are listed.
      const long long y = A.y;
      int cnt = 0;
      for (int k = lo; k < hi; ++k) {
        const int e = AEL[k];
        const bool ends = E[e].ty == y;
        if (A.op == kOpTop) {
          if (!ends) {
            E[e].cx = (int)edge_top_x(E[e], y);
            E[e].cy = (int)y;
          } else {
            ++cnt;
          }
        } else if (ends && E[e].next_lml != kNil) {
          ++cnt;
        }
      }
      int total = 0;
      int off = bulk_offset(A, lane, nl, cnt, &total);
      for (int k = lo; k < hi; ++k) {
        const int e = AEL[k];
        if (E[e].ty == y && (A.op == kOpTop || E[e].next_lml != kNil)) A.SPL[off++] = e;
      }
      if (lane == 0) A.result = total;
      return;
    }
    case kOpSel:
      for (int k = lo; k < hi; ++k) {
        const int e = AEL[k];
        E[e].prev_sel = k > 0 ? AEL[k - 1] : kNil;
        E[e].next_sel = k + 1 < n ? AEL[k + 1] : kNil;
      }
      return;
    case kOpInsert: {  // positions [a, n) move up by one (from the top down)
      const int pos = A.a;
      for (int base = n - 1; base >= pos; base -= nl) {
        const int k = base - lane;
        const int m = k >= pos ? AEL[k] : kNil;
        bulk_sync(nl);
        if (k >= pos) {
          AEL[k + 1] = m;
          E[m].ael_pos = k + 1;
        }
        bulk_sync(nl);
      }
      return;
    }
    case kOpDelete: {  // positions (a, n) move down by one (from the bottom up)
      const int pos = A.a;
      for (int base = pos; base + 1 < n; base += nl) {
        const int k = base + lane;
        const int m = k + 1 < n ? AEL[k + 1] : kNil;
        bulk_sync(nl);
        if (k + 1 < n) {
          AEL[k] = m;
          E[m].ael_pos = k;
        }
        bulk_sync(nl);
      }
      return;
    }
    case kOpFindIns: {  // first p >= a where edge b inserts before AEL[p]
      const int e = A.b;
      const int r = bulk_find(A, lane, nl, A.a, n, [&](int p) { return inserts_before(E, AEL[p], e); });
      if (lane == 0) A.result = r;
      return;
    }
    case kOpFindOut: {  // first p with OutIdx == a
      const int o = A.a;
      const int r = bulk_find(A, lane, nl, 0, n, [&](int p) { return E[AEL[p]].out_idx == o; });
      if (lane == 0) A.result = r;
      return;
    }
    default:
      return;
  }
}

#if defined(__CUDACC__)
// One step of the warp that owns a ring: lane 0 has written the command;
// every lane runs its share. False once the command is kOpStop. Not inlined,
// so that every lane meets the same barrier instructions.
__device__ __noinline__ bool bulk_step(BulkArgs *A, int lane) {
  __syncwarp();
  if (*(volatile int *)&A->op == kOpStop) return false;
  bulk_exec(*A, lane, 32);
  __syncwarp();
  return true;
}
#endif

// ------------------------------------------------------------ the sweep -------
struct Sweep {
  Edge *E;
  LocMin *LM;
  long long *SB;
  OutPt *OP;
  OutRec *OR;
  Join *JN;
  Join *GJ;
  INode *IN;
  int *STK;
  int *ARR, *KEY, *SUF, *PASS;
  INode *IN2;
  int *SPL, *CLS;       // list-wide step outputs: edge lists, bubble-sort clusters
  BulkArgs *bk;         // list-wide step arguments (per warp on the device)
  int bk_lanes;
  Caps cap;
  int n_edges, n_lm, cur_lm, n_sb, n_op, n_or, n_jn, n_gj, n_in;
  // The active edge list (AEL) is kept as an array in x order, AEL[0..
  // ael_n), with each member's index in Edge::ael_pos (-1 when not in it):
  // Clipper's NextInAEL / PrevInAEL are the neighbours in that array, and its
  // walks become loops over it. Clipper only reads the links of an edge that
  // is not in the AEL to learn that it is not there.
  int *AEL;
  int ael_n;
  int sorted;  // SEL head
  long long guard, guard_limit;
  bool fail;

  CU_HD void init(char *arena, int n) {
    cap = caps_for(n);
    auto al = [](unsigned long long b) { return (b + 15ull) & ~15ull; };
    char *p = arena;
    E = reinterpret_cast<Edge *>(p); p += al(sizeof(Edge) * (unsigned long long)cap.edges);
    LM = reinterpret_cast<LocMin *>(p); p += al(sizeof(LocMin) * (unsigned long long)cap.minima);
    SB = reinterpret_cast<long long *>(p); p += al(sizeof(long long) * (unsigned long long)cap.scan);
    OP = reinterpret_cast<OutPt *>(p); p += al(sizeof(OutPt) * (unsigned long long)(cap.outpts + 1));
    OR = reinterpret_cast<OutRec *>(p); p += al(sizeof(OutRec) * (unsigned long long)(cap.outrecs + 1));
    JN = reinterpret_cast<Join *>(p); p += al(sizeof(Join) * (unsigned long long)cap.joins);
    GJ = reinterpret_cast<Join *>(p); p += al(sizeof(Join) * (unsigned long long)cap.ghosts);
    IN = reinterpret_cast<INode *>(p); p += al(sizeof(INode) * (unsigned long long)cap.inodes);
    STK = reinterpret_cast<int *>(p); p += al(sizeof(int) * 3ull * (unsigned long long)cap.stack);
    ARR = reinterpret_cast<int *>(p);
    KEY = ARR + (cap.edges + 2);
    SUF = KEY + (cap.edges + 2);
    AEL = SUF + (cap.edges + 2);
    p += al(sizeof(int) * 4ull * (unsigned long long)(cap.edges + 2));
    PASS = reinterpret_cast<int *>(p); p += al(sizeof(int) * (unsigned long long)cap.inodes);
    IN2 = reinterpret_cast<INode *>(p); p += al(sizeof(INode) * (unsigned long long)cap.inodes);
    SPL = reinterpret_cast<int *>(p);
    CLS = SPL + (cap.edges + 2);
    bk = nullptr;
    bk_lanes = 1;
    n_edges = n_lm = cur_lm = n_sb = n_op = n_or = n_jn = n_gj = n_in = 0;
    ael_n = 0;
    sorted = kNil;
    fail = false;
    guard = 0;
    // Bound on the total number of loop steps of one sweep: about ten times
    // the most measured (240 steps per path point on 13k-point rings); a
    // sweep that reaches it stops with fail set instead of running on.
    guard_limit = 2048ll * (long long)(n + 64) + (1ll << 22);
  }
  CU_HD bool tick() {
    if (++guard > guard_limit) fail = true;
    return !fail;
  }
  // The list-wide steps: arguments to bk, then every lane of the owning warp
  // (device, bk_lanes 32) or this thread alone runs bulk_exec.
  CU_HD void set_bulk(BulkArgs *a, int lanes) {
    bk = a;
    bk_lanes = lanes;
  }
  CU_HD int bulk(int op, int a = 0, int b = 0, long long y = 0) {
    BulkArgs &A = *bk;
    A.op = op; A.a = a; A.b = b; A.y = y; A.n = ael_n; A.result = 0;
    A.E = E; A.AEL = AEL; A.ARR = ARR; A.KEY = KEY; A.SUF = SUF; A.SPL = SPL; A.CLS = CLS;
#if defined(__CUDA_ARCH__)
    if (bk_lanes > 1) {
      bulk_step(bk, 0);
      return A.result;
    }
#else
    if (bk_lanes > 1 && g_host_runner) {
      g_host_runner(bk, bk_lanes);
      return A.result;
    }
#endif
    bulk_exec(A, 0, 1);
    return A.result;
  }

  // ---- small helpers -----------------------------------------------------
  static CU_HD long long round_c(double v) {
    return v < 0 ? (long long)(v - 0.5) : (long long)(v + 0.5);
  }
  CU_HD bool is_horz(int e) const { return E[e].dx == kHorizontal; }
  CU_HD void set_dx(Edge &e) {
    const long long dy = (long long)e.ty - e.by;
    e.dx = dy == 0 ? kHorizontal : (double)((long long)e.tx - e.bx) / (double)dy;
  }
  CU_HD long long top_x(int ei, long long y) const {
    const Edge &e = E[ei];
    return y == e.ty ? (long long)e.tx : (long long)e.bx + round_c(e.dx * (double)(y - e.by));
  }
  static CU_HD bool slopes3(long long x1, long long y1, long long x2, long long y2, long long x3,
                            long long y3) {
    return (y1 - y2) * (x2 - x3) == (x1 - x2) * (y2 - y3);
  }
  static CU_HD bool slopes4(long long x1, long long y1, long long x2, long long y2, long long x3,
                            long long y3, long long x4, long long y4) {
    return (y1 - y2) * (x3 - x4) == (x1 - x2) * (y3 - y4);
  }
  CU_HD bool slopes_edges(int a, int b) const {
    return ((long long)E[a].ty - E[a].by) * ((long long)E[b].tx - E[b].bx) ==
           ((long long)E[a].tx - E[a].bx) * ((long long)E[b].ty - E[b].by);
  }
  static CU_HD double get_dx(long long x1, long long y1, long long x2, long long y2) {
    return y1 == y2 ? kHorizontal : (double)(x2 - x1) / (double)(y2 - y1);
  }

  // ---- scanbeam max-heap ----------------------------------------------------
  CU_HD void sb_push(long long y) {
    if (n_sb >= cap.scan) { fail = true; return; }
    int i = n_sb++;
    while (i > 0) {
      const int p = (i - 1) / 2;
      if (SB[p] >= y) break;
      SB[i] = SB[p];
      i = p;
    }
    SB[i] = y;
  }
  CU_HD long long sb_pop_one() {
    const long long top = SB[0];
    const long long last = SB[--n_sb];
    int i = 0;
    for (;;) {
      int c = 2 * i + 1;
      if (c >= n_sb) break;
      if (c + 1 < n_sb && SB[c + 1] > SB[c]) ++c;
      if (SB[c] <= last) break;
      SB[i] = SB[c];
      i = c;
    }
    if (n_sb > 0) SB[i] = last;
    return top;
  }
  CU_HD bool pop_scanbeam(long long *y) {
    if (n_sb == 0) return false;
    *y = sb_pop_one();
    while (n_sb > 0 && SB[0] == *y) sb_pop_one();
    return true;
  }

  // ---- out points / records ------------------------------------------------
  CU_HD int new_outpt() {
    if (n_op >= cap.outpts) { fail = true; OP[cap.outpts] = OutPt{0, cap.outpts, cap.outpts, 0, 0}; return cap.outpts; }
    return n_op++;
  }
  CU_HD int create_outrec() {
    int r;
    if (n_or >= cap.outrecs) { fail = true; r = cap.outrecs; }
    else r = n_or++;
    OutRec &o = OR[r];
    o.is_hole = 0;
    o.first_left = kNil;
    o.pts = kNil;
    o.bottom_pt = kNil;
    o.idx = r;
    return r;
  }
  CU_HD void add_join(int op1, int op2, long long x, long long y) {
    if (n_jn >= cap.joins) { fail = true; return; }
    JN[n_jn++] = Join{op1, op2, (int)x, (int)y};
  }
  CU_HD void add_ghost(int op, long long x, long long y) {
    if (n_gj >= cap.ghosts) { fail = true; return; }
    GJ[n_gj++] = Join{op, kNil, (int)x, (int)y};
  }

  // ---- path -> edges and local minima (AddPath, closed, subject) ------------
  CU_HD int remove_edge(int e) {
    E[E[e].prev].next = E[e].next;
    E[E[e].next].prev = E[e].prev;
    const int r = E[e].next;
    E[e].prev = kNil;
    return r;
  }
  CU_HD void reverse_horz(int e) {
    const int t = E[e].tx;
    E[e].tx = E[e].bx;
    E[e].bx = t;
  }
  CU_HD int find_next_locmin(int e) {
    for (;;) {
      while ((E[e].bx != E[E[e].prev].bx || E[e].by != E[E[e].prev].by) ||
             (E[e].cx == E[e].tx && E[e].cy == E[e].ty)) {
        if (!tick()) return e;
        e = E[e].next;
      }
      if (!is_horz(e) && !is_horz(E[e].prev)) break;
      while (is_horz(E[e].prev)) { if (!tick()) return e; e = E[e].prev; }
      const int e2 = e;
      while (is_horz(e)) { if (!tick()) return e; e = E[e].next; }
      if (E[e].ty == E[E[e].prev].by) continue;  // an intermediate horizontal
      if (E[E[e2].prev].bx < E[e].bx) e = e2;
      break;
    }
    return e;
  }
  // ProcessBound for closed paths (no Skip edges exist)
  CU_HD int process_bound(int e, bool forward) {
    int result = e;
    if (is_horz(e)) {
      const int es = forward ? E[e].prev : E[e].next;
      if (is_horz(es)) {
        if (E[es].bx != E[e].bx && E[es].tx != E[e].bx) reverse_horz(e);
      } else if (E[es].bx != E[e].bx) {
        reverse_horz(e);
      }
    }
    const int estart = e;
    if (forward) {
      while (E[result].ty == E[E[result].next].by) { if (!tick()) return result; result = E[result].next; }
      if (is_horz(result)) {
        int h = result;
        while (is_horz(E[h].prev)) { if (!tick()) return result; h = E[h].prev; }
        if (E[E[h].prev].tx > E[E[result].next].tx) result = E[h].prev;
      }
      while (e != result) {
        if (!tick()) return result;
        E[e].next_lml = E[e].next;
        if (is_horz(e) && e != estart && E[e].bx != E[E[e].prev].tx) reverse_horz(e);
        e = E[e].next;
      }
      if (is_horz(e) && e != estart && E[e].bx != E[E[e].prev].tx) reverse_horz(e);
      result = E[result].next;
    } else {
      while (E[result].ty == E[E[result].prev].by) { if (!tick()) return result; result = E[result].prev; }
      if (is_horz(result)) {
        int h = result;
        while (is_horz(E[h].next)) { if (!tick()) return result; h = E[h].next; }
        if (E[E[h].next].tx == E[E[result].prev].tx || E[E[h].next].tx > E[E[result].prev].tx)
          result = E[h].next;
      }
      while (e != result) {
        if (!tick()) return result;
        E[e].next_lml = E[e].prev;
        if (is_horz(e) && e != estart && E[e].bx != E[E[e].next].tx) reverse_horz(e);
        e = E[e].prev;
      }
      if (is_horz(e) && e != estart && E[e].bx != E[E[e].next].tx) reverse_horz(e);
      result = E[result].prev;
    }
    return result;
  }
  // Returns false when the path adds nothing (fewer than 3 distinct
  // non-collinear vertices, or flat).
  CU_HD bool add_path(const P2 *pg, int count) {
    int hi = count - 1;
    while (hi > 0 && pg[hi].x == pg[0].x && pg[hi].y == pg[0].y) --hi;
    while (hi > 0 && pg[hi].x == pg[hi - 1].x && pg[hi].y == pg[hi - 1].y) --hi;
    if (hi < 2) return false;
    for (int i = 0; i <= hi; ++i) {
      if (pg[i].x > kCoordLimit || pg[i].y > kCoordLimit || -(long long)pg[i].x > kCoordLimit ||
          -(long long)pg[i].y > kCoordLimit) {
        fail = true;
        return false;
      }
      Edge &e = E[i];
      e.bx = e.by = e.tx = e.ty = 0;
      e.cx = pg[i].x;
      e.cy = pg[i].y;
      e.dx = 0.0;
      e.wdelta = e.wcnt = e.wcnt2 = 0;
      e.side = 0;
      e.out_idx = kUnassigned;
      e.next = i == hi ? 0 : i + 1;
      e.prev = i == 0 ? hi : i - 1;
      e.next_lml = e.next_sel = e.prev_sel = kNil;
      e.ael_pos = -1;
    }
    n_edges = hi + 1;
    int start = 0, e = 0, stop = 0;
    for (;;) {
      if (!tick()) return false;
      if (E[e].cx == E[E[e].next].cx && E[e].cy == E[E[e].next].cy) {
        if (e == E[e].next) break;
        if (e == start) start = E[e].next;
        e = remove_edge(e);
        stop = e;
        continue;
      }
      if (E[e].prev == E[e].next) break;
      if (slopes3(E[E[e].prev].cx, E[E[e].prev].cy, E[e].cx, E[e].cy, E[E[e].next].cx,
                  E[E[e].next].cy)) {
        if (e == start) start = E[e].next;
        e = remove_edge(e);
        e = E[e].prev;
        stop = e;
        continue;
      }
      e = E[e].next;
      if (e == stop) break;
    }
    if (E[e].prev == E[e].next) return false;
    // second stage of edge initialisation
    bool flat = true;
    e = start;
    do {
      Edge &d = E[e];
      const Edge &nx = E[d.next];
      if (d.cy >= nx.cy) {
        d.bx = d.cx; d.by = d.cy; d.tx = nx.cx; d.ty = nx.cy;
      } else {
        d.tx = d.cx; d.ty = d.cy; d.bx = nx.cx; d.by = nx.cy;
      }
      set_dx(d);
      e = d.next;
      if (flat && E[e].cy != E[start].cy) flat = false;
      if (!tick()) return false;
    } while (e != start);
    if (flat) return false;
    int emin = kNil;
    if (E[E[e].prev].bx == E[E[e].prev].tx && E[E[e].prev].by == E[E[e].prev].ty) e = E[e].next;
    for (;;) {
      e = find_next_locmin(e);
      if (fail) return false;
      if (e == emin) break;
      if (emin == kNil) emin = e;
      if (n_lm >= cap.minima) { fail = true; return false; }
      LocMin lm;
      lm.y = E[e].by;
      bool left_forward;
      if (E[e].dx < E[E[e].prev].dx) {
        lm.left = E[e].prev;
        lm.right = e;
        left_forward = false;
      } else {
        lm.left = e;
        lm.right = E[e].prev;
        left_forward = true;
      }
      E[lm.left].wdelta = (E[lm.left].next == lm.right) ? -1 : 1;
      E[lm.right].wdelta = -E[lm.left].wdelta;
      e = process_bound(lm.left, left_forward);
      const int e2 = process_bound(lm.right, !left_forward);
      if (fail) return false;
      LM[n_lm++] = lm;
      if (!left_forward) e = e2;
    }
    return true;
  }

  // ---- AEL / SEL -----------------------------------------------------------
  CU_HD bool e2_inserts_before_e1(int e1, int e2) const {
    if (E[e2].cx == E[e1].cx) {
      if (E[e2].ty > E[e1].ty) return E[e2].tx < top_x(e1, E[e2].ty);
      return E[e1].tx > top_x(e2, E[e1].ty);
    }
    return E[e2].cx < E[e1].cx;
  }
  CU_HD int head() const { return ael_n > 0 ? AEL[0] : kNil; }
  CU_HD int nxt(int e) const {
    const int p = E[e].ael_pos;
    return (p >= 0 && p + 1 < ael_n) ? AEL[p + 1] : kNil;
  }
  CU_HD int prv(int e) const {
    const int p = E[e].ael_pos;
    return p > 0 ? AEL[p - 1] : kNil;
  }
  CU_HD void ael_insert_at(int e, int pos) {
    if (ael_n >= n_edges) { fail = true; return; }
    if (pos < ael_n) bulk(kOpInsert, pos);
    AEL[pos] = e;
    E[e].ael_pos = pos;
    ++ael_n;
  }
  CU_HD void insert_into_ael(int e, int start) {
    if (ael_n == 0) {
      ael_insert_at(e, 0);
    } else if (start == kNil && e2_inserts_before_e1(AEL[0], e)) {
      ael_insert_at(e, 0);
    } else {
      // first position after start where e inserts before the edge there
      const int k = start == kNil ? 0 : E[start].ael_pos;
      ael_insert_at(e, bulk(kOpFindIns, k + 1, e));
    }
  }
  CU_HD void delete_from_ael(int e) {
    const int p = E[e].ael_pos;
    if (p < 0) return;
    if (p + 1 < ael_n) bulk(kOpDelete, p);
    --ael_n;
    E[e].ael_pos = -1;
  }
  CU_HD void delete_from_sel(int e) {
    const int p = E[e].prev_sel, n = E[e].next_sel;
    if (p == kNil && n == kNil && e != sorted) return;
    if (p != kNil) E[p].next_sel = n; else sorted = n;
    if (n != kNil) E[n].prev_sel = p;
    E[e].next_sel = E[e].prev_sel = kNil;
  }
  CU_HD void add_to_sel(int e) {
    if (sorted == kNil) {
      sorted = e;
      E[e].prev_sel = E[e].next_sel = kNil;
    } else {
      E[e].next_sel = sorted;
      E[e].prev_sel = kNil;
      E[sorted].prev_sel = e;
      sorted = e;
    }
  }
  CU_HD void copy_ael_to_sel() {
    sorted = head();
    if (ael_n > 0) bulk(kOpSel);
  }
  // SwapPositionsInAEL: both edges must be in the AEL (Clipper's test
  // NextInAEL == PrevInAEL is true only for an edge outside it, or alone).
  CU_HD void swap_in_ael(int a, int b) {
    if (nxt(a) == prv(a) || nxt(b) == prv(b)) return;
    const int pa = E[a].ael_pos, pb = E[b].ael_pos;
    AEL[pa] = b; E[b].ael_pos = pa;
    AEL[pb] = a; E[a].ael_pos = pb;
  }
  CU_HD void swap_in_sel(int a, int b) {
    if (E[a].next_sel == kNil && E[a].prev_sel == kNil) return;
    if (E[b].next_sel == kNil && E[b].prev_sel == kNil) return;
    if (E[a].next_sel == b) {
      const int nx = E[b].next_sel, pv = E[a].prev_sel;
      if (nx != kNil) E[nx].prev_sel = a;
      if (pv != kNil) E[pv].next_sel = b;
      E[b].prev_sel = pv; E[b].next_sel = a;
      E[a].prev_sel = b; E[a].next_sel = nx;
    } else if (E[b].next_sel == a) {
      const int nx = E[a].next_sel, pv = E[b].prev_sel;
      if (nx != kNil) E[nx].prev_sel = b;
      if (pv != kNil) E[pv].next_sel = a;
      E[a].prev_sel = pv; E[a].next_sel = b;
      E[b].prev_sel = a; E[b].next_sel = nx;
    } else {
      const int nx = E[a].next_sel, pv = E[a].prev_sel;
      E[a].next_sel = E[b].next_sel;
      if (E[a].next_sel != kNil) E[E[a].next_sel].prev_sel = a;
      E[a].prev_sel = E[b].prev_sel;
      if (E[a].prev_sel != kNil) E[E[a].prev_sel].next_sel = a;
      E[b].next_sel = nx;
      if (E[b].next_sel != kNil) E[E[b].next_sel].prev_sel = b;
      E[b].prev_sel = pv;
      if (E[b].prev_sel != kNil) E[E[b].prev_sel].next_sel = b;
    }
    if (E[a].prev_sel == kNil) sorted = a;
    else if (E[b].prev_sel == kNil) sorted = b;
  }
  CU_HD void update_edge_into_ael(int &e) {
    const int nl = E[e].next_lml;
    if (nl == kNil) { fail = true; return; }
    E[nl].out_idx = E[e].out_idx;
    const int pos = E[e].ael_pos;
    if (pos < 0) { fail = true; return; }
    AEL[pos] = nl;
    E[nl].ael_pos = pos;
    E[e].ael_pos = -1;
    E[nl].side = E[e].side;
    E[nl].wdelta = E[e].wdelta;
    E[nl].wcnt = E[e].wcnt;
    E[nl].wcnt2 = E[e].wcnt2;
    e = nl;
    E[e].cx = E[e].bx;
    E[e].cy = E[e].by;
    if (!is_horz(e)) sb_push(E[e].ty);
  }

  // ---- winding (positive fill, subject only) --------------------------------
  CU_HD void set_winding_count(int ei) {
    Edge &edge = E[ei];
    int e = prv(ei), g = 0;
    while (e != kNil && E[e].wdelta == 0) {
      if (++g > n_edges) { fail = true; return; }
      e = prv(e);
    }
    if (e == kNil) {
      edge.wcnt = edge.wdelta == 0 ? 1 : edge.wdelta;
      edge.wcnt2 = 0;
      e = head();
    } else {
      const Edge &pe = E[e];
      if (pe.wcnt * pe.wdelta < 0) {
        if ((pe.wcnt < 0 ? -pe.wcnt : pe.wcnt) > 1) {
          if (pe.wdelta * edge.wdelta < 0) edge.wcnt = pe.wcnt;
          else edge.wcnt = pe.wcnt + edge.wdelta;
        } else {
          edge.wcnt = edge.wdelta == 0 ? 1 : edge.wdelta;
        }
      } else {
        if (edge.wdelta == 0) edge.wcnt = pe.wcnt < 0 ? pe.wcnt - 1 : pe.wcnt + 1;
        else if (pe.wdelta * edge.wdelta < 0) edge.wcnt = pe.wcnt;
        else edge.wcnt = pe.wcnt + edge.wdelta;
      }
      edge.wcnt2 = pe.wcnt2;
      e = nxt(e);
    }
    while (e != ei) {
      if (e == kNil || ++g > 2 * n_edges) { fail = true; return; }
      edge.wcnt2 += E[e].wdelta;
      e = nxt(e);
    }
  }
  // positive fill for the subject, union with an empty positive clip side
  CU_HD bool is_contributing(int e) const { return E[e].wcnt == 1 && E[e].wcnt2 <= 0; }

  // ---- output polygons ------------------------------------------------------
  CU_HD void set_hole_state(int e, int orec) {
    int tmp = kNil;
    for (int k = E[e].ael_pos - 1; k >= 0; --k) {
      const int e2 = AEL[k];
      if (E[e2].out_idx >= 0 && E[e2].wdelta != 0) {
        if (tmp == kNil) tmp = e2;
        else if (E[tmp].out_idx == E[e2].out_idx) tmp = kNil;
      }
    }
    if (tmp == kNil) {
      OR[orec].first_left = kNil;
      OR[orec].is_hole = 0;
    } else {
      OR[orec].first_left = E[tmp].out_idx;
      OR[orec].is_hole = !OR[OR[orec].first_left].is_hole;
    }
  }
  CU_HD int add_out_pt(int e, long long x, long long y) {
    if (E[e].out_idx < 0) {
      const int r = create_outrec();
      const int np = new_outpt();
      OR[r].pts = np;
      OP[np].idx = OR[r].idx;
      OP[np].x = (int)x; OP[np].y = (int)y;
      OP[np].next = OP[np].prev = np;
      set_hole_state(e, r);
      E[e].out_idx = OR[r].idx;
      return np;
    }
    const int r = E[e].out_idx;
    const int op = OR[r].pts;
    const bool to_front = E[e].side == kSideLeft;
    if (to_front && x == OP[op].x && y == OP[op].y) return op;
    if (!to_front && x == OP[OP[op].prev].x && y == OP[OP[op].prev].y) return OP[op].prev;
    const int np = new_outpt();
    OP[np].idx = OR[r].idx;
    OP[np].x = (int)x; OP[np].y = (int)y;
    OP[np].next = op;
    OP[np].prev = OP[op].prev;
    OP[OP[np].prev].next = np;
    OP[op].prev = np;
    if (to_front) OR[r].pts = np;
    return np;
  }
  CU_HD int last_out_pt(int e) const {
    const int r = E[e].out_idx;
    return E[e].side == kSideLeft ? OR[r].pts : OP[OR[r].pts].prev;
  }
  CU_HD int add_local_min_poly(int e1, int e2, long long x, long long y) {
    int result, e, prev_e;
    if (is_horz(e2) || E[e1].dx > E[e2].dx) {
      result = add_out_pt(e1, x, y);
      E[e2].out_idx = E[e1].out_idx;
      E[e1].side = kSideLeft;
      E[e2].side = kSideRight;
      e = e1;
      prev_e = prv(e) == e2 ? prv(e2) : prv(e);
    } else {
      result = add_out_pt(e2, x, y);
      E[e1].out_idx = E[e2].out_idx;
      E[e1].side = kSideRight;
      E[e2].side = kSideLeft;
      e = e2;
      prev_e = prv(e) == e1 ? prv(e1) : prv(e);
    }
    if (prev_e != kNil && E[prev_e].out_idx >= 0 && E[prev_e].ty < y && E[e].ty < y) {
      const long long xp = top_x(prev_e, y), xe = top_x(e, y);
      if (xp == xe && E[e].wdelta != 0 && E[prev_e].wdelta != 0 &&
          slopes4(xp, y, E[prev_e].tx, E[prev_e].ty, xe, y, E[e].tx, E[e].ty)) {
        const int op = add_out_pt(prev_e, x, y);
        add_join(result, op, E[e].tx, E[e].ty);
      }
    }
    return result;
  }
  CU_HD void reverse_links(int pp) {
    if (pp == kNil) return;
    int p1 = pp;
    do {
      if (!tick()) return;
      const int p2 = OP[p1].next;
      OP[p1].next = OP[p1].prev;
      OP[p1].prev = p2;
      p1 = p2;
    } while (p1 != pp);
  }
  CU_HD bool outrec1_right_of_outrec2(int r1, int r2) {
    do {
      if (!tick()) return false;
      r1 = OR[r1].first_left;
      if (r1 == r2) return true;
    } while (r1 != kNil);
    return false;
  }
  CU_HD double area_op(int op) {
    if (op == kNil) return 0;
    const int start = op;
    double a = 0;
    do {
      if (!tick()) return 0;
      const OutPt &p = OP[op], &q = OP[OP[op].prev];
      // an exact integer sum at these coordinates (fused or not)
      a += (double)((long long)q.x + p.x) * (double)((long long)q.y - p.y);
      op = OP[op].next;
    } while (op != start);
    return a * 0.5;
  }
  CU_HD bool first_is_bottom_pt(int b1, int b2) {
    auto side_dx = [&](int b, bool prev_dir) {
      int p = prev_dir ? OP[b].prev : OP[b].next;
      while (OP[p].x == OP[b].x && OP[p].y == OP[b].y && p != b) {
        if (!tick()) break;
        p = prev_dir ? OP[p].prev : OP[p].next;
      }
      return fabs(get_dx(OP[b].x, OP[b].y, OP[p].x, OP[p].y));
    };
    const double dx1p = side_dx(b1, true), dx1n = side_dx(b1, false);
    const double dx2p = side_dx(b2, true), dx2n = side_dx(b2, false);
    const double mx1 = dx1p > dx1n ? dx1p : dx1n, mx2 = dx2p > dx2n ? dx2p : dx2n;
    const double mn1 = dx1p < dx1n ? dx1p : dx1n, mn2 = dx2p < dx2n ? dx2p : dx2n;
    if (mx1 == mx2 && mn1 == mn2) return area_op(b1) > 0;
    return (dx1p >= dx2p && dx1p >= dx2n) || (dx1n >= dx2p && dx1n >= dx2n);
  }
  CU_HD int get_bottom_pt(int pp) {
    int dups = kNil;
    int p = OP[pp].next;
    while (p != pp) {
      if (!tick()) return pp;
      if (OP[p].y > OP[pp].y) {
        pp = p;
        dups = kNil;
      } else if (OP[p].y == OP[pp].y && OP[p].x <= OP[pp].x) {
        if (OP[p].x < OP[pp].x) {
          dups = kNil;
          pp = p;
        } else if (OP[p].next != pp && OP[p].prev != pp) {
          dups = p;
        }
      }
      p = OP[p].next;
    }
    if (dups != kNil) {
      while (dups != p) {
        if (!tick()) return pp;
        if (!first_is_bottom_pt(p, dups)) pp = dups;
        dups = OP[dups].next;
        while (OP[dups].x != OP[pp].x || OP[dups].y != OP[pp].y) {
          if (!tick()) return pp;
          dups = OP[dups].next;
        }
      }
    }
    return pp;
  }
  CU_HD int lowermost_rec(int r1, int r2) {
    if (OR[r1].bottom_pt == kNil) OR[r1].bottom_pt = get_bottom_pt(OR[r1].pts);
    if (OR[r2].bottom_pt == kNil) OR[r2].bottom_pt = get_bottom_pt(OR[r2].pts);
    const int p1 = OR[r1].bottom_pt, p2 = OR[r2].bottom_pt;
    if (OP[p1].y > OP[p2].y) return r1;
    if (OP[p1].y < OP[p2].y) return r2;
    if (OP[p1].x < OP[p2].x) return r1;
    if (OP[p1].x > OP[p2].x) return r2;
    if (OP[p1].next == p1) return r2;
    if (OP[p2].next == p2) return r1;
    return first_is_bottom_pt(p1, p2) ? r1 : r2;
  }
  CU_HD void append_polygon(int e1, int e2) {
    const int r1 = E[e1].out_idx, r2 = E[e2].out_idx;
    int hole_rec;
    if (outrec1_right_of_outrec2(r1, r2)) hole_rec = r2;
    else if (outrec1_right_of_outrec2(r2, r1)) hole_rec = r1;
    else hole_rec = lowermost_rec(r1, r2);
    const int p1_l = OR[r1].pts, p1_r = OP[p1_l].prev;
    const int p2_l = OR[r2].pts, p2_r = OP[p2_l].prev;
    if (E[e1].side == kSideLeft) {
      if (E[e2].side == kSideLeft) {
        reverse_links(p2_l);
        OP[p2_l].next = p1_l; OP[p1_l].prev = p2_l;
        OP[p1_r].next = p2_r; OP[p2_r].prev = p1_r;
        OR[r1].pts = p2_r;
      } else {
        OP[p2_r].next = p1_l; OP[p1_l].prev = p2_r;
        OP[p2_l].prev = p1_r; OP[p1_r].next = p2_l;
        OR[r1].pts = p2_l;
      }
    } else {
      if (E[e2].side == kSideRight) {
        reverse_links(p2_l);
        OP[p1_r].next = p2_r; OP[p2_r].prev = p1_r;
        OP[p2_l].next = p1_l; OP[p1_l].prev = p2_l;
      } else {
        OP[p1_r].next = p2_l; OP[p2_l].prev = p1_r;
        OP[p1_l].prev = p2_r; OP[p2_r].next = p1_l;
      }
    }
    OR[r1].bottom_pt = kNil;
    if (hole_rec == r2) {
      if (OR[r2].first_left != r1) OR[r1].first_left = OR[r2].first_left;
      OR[r1].is_hole = OR[r2].is_hole;
    }
    OR[r2].pts = kNil;
    OR[r2].bottom_pt = kNil;
    OR[r2].first_left = r1;
    const int ok = E[e1].out_idx, obsolete = E[e2].out_idx;
    E[e1].out_idx = kUnassigned;
    E[e2].out_idx = kUnassigned;
    const int k = bulk(kOpFindOut, obsolete);
    if (k < ael_n) {
      const int e = AEL[k];
      E[e].out_idx = ok;
      E[e].side = E[e1].side;
    }
    OR[r2].idx = OR[r1].idx;
  }
  CU_HD void add_local_max_poly(int e1, int e2, long long x, long long y) {
    add_out_pt(e1, x, y);
    if (E[e2].wdelta == 0) add_out_pt(e2, x, y);
    if (E[e1].out_idx == E[e2].out_idx) {
      E[e1].out_idx = kUnassigned;
      E[e2].out_idx = kUnassigned;
    } else if (E[e1].out_idx < E[e2].out_idx) {
      append_polygon(e1, e2);
    } else {
      append_polygon(e2, e1);
    }
  }

  // ---- intersections ---------------------------------------------------------
  CU_HD void intersect_edges(int e1, int e2, long long x, long long y) {
    const bool c1 = E[e1].out_idx >= 0, c2 = E[e2].out_idx >= 0;
    // same poly type, non-zero (positive) fill: update winding counts
    if (E[e1].wcnt + E[e2].wdelta == 0) E[e1].wcnt = -E[e1].wcnt;
    else E[e1].wcnt += E[e2].wdelta;
    if (E[e2].wcnt - E[e1].wdelta == 0) E[e2].wcnt = -E[e2].wcnt;
    else E[e2].wcnt -= E[e1].wdelta;
    const long long w1 = E[e1].wcnt, w2 = E[e2].wcnt;
    if (c1 && c2) {
      if ((w1 != 0 && w1 != 1) || (w2 != 0 && w2 != 1)) {
        add_local_max_poly(e1, e2, x, y);
      } else {
        add_out_pt(e1, x, y);
        add_out_pt(e2, x, y);
        const int s = E[e1].side; E[e1].side = E[e2].side; E[e2].side = s;
        const int o = E[e1].out_idx; E[e1].out_idx = E[e2].out_idx; E[e2].out_idx = o;
      }
    } else if (c1) {
      if (w2 == 0 || w2 == 1) {
        add_out_pt(e1, x, y);
        const int s = E[e1].side; E[e1].side = E[e2].side; E[e2].side = s;
        const int o = E[e1].out_idx; E[e1].out_idx = E[e2].out_idx; E[e2].out_idx = o;
      }
    } else if (c2) {
      if (w1 == 0 || w1 == 1) {
        add_out_pt(e2, x, y);
        const int s = E[e1].side; E[e1].side = E[e2].side; E[e2].side = s;
        const int o = E[e1].out_idx; E[e1].out_idx = E[e2].out_idx; E[e2].out_idx = o;
      }
    } else if ((w1 == 0 || w1 == 1) && (w2 == 0 || w2 == 1)) {
      const long long v1 = E[e1].wcnt2, v2 = E[e2].wcnt2;
      if (w1 == 1 && w2 == 1) {
        if (v1 <= 0 && v2 <= 0) add_local_min_poly(e1, e2, x, y);
      } else {
        const int s = E[e1].side; E[e1].side = E[e2].side; E[e2].side = s;
      }
    }
  }
  // Clipper's IntersectPoint; the two multiply-adds are fused as the
  // reference build (-O3 -march=x86-64-v3) compiles them.
  CU_HD void intersect_point(int a, int b, long long *ox, long long *oy) const {
    const Edge &e1 = E[a], &e2 = E[b];
    long long x, y;
    if (e1.dx == e2.dx) {
      y = e1.cy;
      *oy = y;
      *ox = top_x(a, y);
      return;
    } else if (e1.dx == 0) {
      x = e1.bx;
      if (e2.dx == kHorizontal) {
        y = e2.by;
      } else {
        const double b2 = (double)e2.by - ((double)e2.bx / e2.dx);
        y = round_c((double)x / e2.dx + b2);
      }
    } else if (e2.dx == 0) {
      x = e2.bx;
      if (e1.dx == kHorizontal) {
        y = e1.by;
      } else {
        const double b1 = (double)e1.by - ((double)e1.bx / e1.dx);
        y = round_c((double)x / e1.dx + b1);
      }
    } else {
      const double b1 = fma(-(double)e1.by, e1.dx, (double)e1.bx);
      const double b2 = fma(-(double)e2.by, e2.dx, (double)e2.bx);
      const double q = (b2 - b1) / (e1.dx - e2.dx);
      y = round_c(q);
      if (fabs(e1.dx) < fabs(e2.dx)) x = round_c(fma(e1.dx, q, b1));
      else x = round_c(fma(e2.dx, q, b2));
    }
    if (y < e1.ty || y < e2.ty) {
      y = e1.ty > e2.ty ? e1.ty : e2.ty;
      x = fabs(e1.dx) < fabs(e2.dx) ? top_x(a, y) : top_x(b, y);
    }
    if (y > e1.cy) {
      y = e1.cy;
      x = fabs(e1.dx) > fabs(e2.dx) ? top_x(b, y) : top_x(a, y);
    }
    *ox = x;
    *oy = y;
  }
  // Clipper's BuildIntersectList sorts a copy of the AEL (the SEL) by the
  // edges' x at top_y with a bubble sort and records an intersection for
  // every adjacent swap, in swap order. Restated exactly but without walking
  // the whole list once per pass: the list splits into clusters at every
  // position where the prefix maximum is <= the suffix minimum; no swap
  // crosses such a position and every pass meets the clusters in list order
  // (a pass's carrier enters a cluster below all of its keys and leaves it
  // below all of the next one's), so each cluster is bubble-sorted on its
  // own, its swaps tagged with their pass, and the records are put in (pass,
  // cluster, swap) order. Equal keys never swap (strict comparison).
  CU_HD void build_intersect_list(long long top_y) {
    if (ael_n == 0) return;
    // keys at the top and the clusters with an inversion (kOpKeys)
    const int n_cl = bulk(kOpKeys, 0, 0, top_y);
    int n_nodes = 0, max_pass = 0;
    for (int ci = 0; ci < n_cl; ++ci) {
      const int s = CLS[2 * ci], i = CLS[2 * ci + 1];
      {  // cluster [s, i]: Clipper's passes on it
        int end = i, pass = 0;
        for (;;) {
          bool modified = false;
          for (int j = s + 1; j <= end; ++j) {
            if (KEY[j - 1] > KEY[j]) {
              const int a = ARR[j - 1], b = ARR[j];
              long long px, py;
              intersect_point(a, b, &px, &py);
              if (py < top_y) { px = top_x(a, top_y); py = top_y; }
              if (n_nodes >= cap.inodes) { fail = true; return; }
              IN2[n_nodes] = INode{a, b, (int)px, (int)py};
              PASS[n_nodes] = pass;
              ++n_nodes;
              ARR[j - 1] = b; ARR[j] = a;
              const int k = KEY[j - 1]; KEY[j - 1] = KEY[j]; KEY[j] = k;
              modified = true;
            }
          }
          if (!tick()) return;
          if (pass > max_pass) max_pass = pass;
          ++pass;
          if (!modified || --end <= s) break;
        }
      }
    }
    // stable counting sort of the records by pass
    for (int p2 = 0; p2 <= max_pass + 1; ++p2) SUF[p2] = 0;
    for (int k = 0; k < n_nodes; ++k) ++SUF[PASS[k] + 1];
    for (int p2 = 1; p2 <= max_pass + 1; ++p2) SUF[p2] += SUF[p2 - 1];
    for (int k = 0; k < n_nodes; ++k) IN[SUF[PASS[k]]++] = IN2[k];
    n_in = n_nodes;
    sorted = kNil;
  }
  CU_HD bool edges_adjacent(const INode &n) const {
    return E[n.e1].next_sel == n.e2 || E[n.e1].prev_sel == n.e2;
  }
  CU_HD bool fixup_intersection_order() {
    copy_ael_to_sel();
    std_sort(IN, n_in, [](const INode &a, const INode &b) { return b.y < a.y; }, STK,
             cap.stack, &fail);
    for (int i = 0; i < n_in; ++i) {
      if (!tick()) return false;
      if (!edges_adjacent(IN[i])) {
        int j = i + 1;
        while (j < n_in && !edges_adjacent(IN[j])) ++j;
        if (j == n_in) return false;
        const INode t = IN[i]; IN[i] = IN[j]; IN[j] = t;
      }
      swap_in_sel(IN[i].e1, IN[i].e2);
    }
    return true;
  }
  CU_HD bool process_intersections(long long top_y) {
    if (ael_n == 0) return true;
    n_in = 0;
    build_intersect_list(top_y);
    if (fail) return false;
    if (n_in == 0) return true;
    if (n_in == 1 || fixup_intersection_order()) {
      for (int i = 0; i < n_in; ++i) {
        if (fail) return false;
        intersect_edges(IN[i].e1, IN[i].e2, IN[i].x, IN[i].y);
        swap_in_ael(IN[i].e1, IN[i].e2);
      }
      n_in = 0;
    } else {
      return false;
    }
    sorted = kNil;
    return true;
  }

  // ---- horizontals -----------------------------------------------------------
  CU_HD int maxima_pair(int e) const {
    const int n = E[e].next, p = E[e].prev;
    if (E[n].tx == E[e].tx && E[n].ty == E[e].ty && E[n].next_lml == kNil) return n;
    if (E[p].tx == E[e].tx && E[p].ty == E[e].ty && E[p].next_lml == kNil) return p;
    return kNil;
  }
  CU_HD int maxima_pair_ex(int e) const {
    const int r = maxima_pair(e);
    if (r != kNil && nxt(r) == prv(r) && !is_horz(r)) return kNil;
    return r;
  }
  CU_HD static bool horz_overlap(long long a1, long long a2, long long b1, long long b2) {
    if (a1 > a2) { const long long t = a1; a1 = a2; a2 = t; }
    if (b1 > b2) { const long long t = b1; b1 = b2; b2 = t; }
    return a1 < b2 && b1 < a2;
  }
  CU_HD void process_horizontal(int horz) {
    bool l2r;
    long long left, right;
    auto dir = [&]() {
      if (E[horz].bx < E[horz].tx) { left = E[horz].bx; right = E[horz].tx; l2r = true; }
      else { left = E[horz].tx; right = E[horz].bx; l2r = false; }
    };
    dir();
    int last_h = horz, max_pair = kNil;
    while (E[last_h].next_lml != kNil && is_horz(E[last_h].next_lml)) {
      if (!tick()) return;
      last_h = E[last_h].next_lml;
    }
    if (E[last_h].next_lml == kNil) max_pair = maxima_pair(last_h);
    int op1 = kNil;
    for (;;) {
      if (!tick()) return;
      const bool is_last = horz == last_h;
      int e = l2r ? nxt(horz) : prv(horz), g = 0;
      while (e != kNil) {
        if (++g > n_edges) { fail = true; return; }
        if ((l2r && E[e].cx > right) || (!l2r && E[e].cx < left)) break;
        if (E[e].cx == E[horz].tx && E[horz].next_lml != kNil && E[e].dx < E[E[horz].next_lml].dx)
          break;
        if (E[horz].out_idx >= 0) {
          op1 = add_out_pt(horz, E[e].cx, E[e].cy);
          for (int nh = sorted; nh != kNil; nh = E[nh].next_sel) {
            if (!tick()) return;
            if (E[nh].out_idx >= 0 && horz_overlap(E[horz].bx, E[horz].tx, E[nh].bx, E[nh].tx))
              add_join(last_out_pt(nh), op1, E[nh].tx, E[nh].ty);
          }
          add_ghost(op1, E[horz].bx, E[horz].by);
        }
        if (e == max_pair && is_last) {
          if (E[horz].out_idx >= 0) add_local_max_poly(horz, max_pair, E[horz].tx, E[horz].ty);
          delete_from_ael(horz);
          delete_from_ael(max_pair);
          return;
        }
        if (l2r) intersect_edges(horz, e, E[e].cx, E[horz].cy);
        else intersect_edges(e, horz, E[e].cx, E[horz].cy);
        const int en = l2r ? nxt(e) : prv(e);
        swap_in_ael(horz, e);
        e = en;
      }
      if (E[horz].next_lml == kNil || !is_horz(E[horz].next_lml)) break;
      update_edge_into_ael(horz);
      if (fail) return;
      if (E[horz].out_idx >= 0) add_out_pt(horz, E[horz].bx, E[horz].by);
      dir();
    }
    if (E[horz].out_idx >= 0 && op1 == kNil) {
      op1 = last_out_pt(horz);
      for (int nh = sorted; nh != kNil; nh = E[nh].next_sel) {
        if (!tick()) return;
        if (E[nh].out_idx >= 0 && horz_overlap(E[horz].bx, E[horz].tx, E[nh].bx, E[nh].tx))
          add_join(last_out_pt(nh), op1, E[nh].tx, E[nh].ty);
      }
      add_ghost(op1, E[horz].tx, E[horz].ty);
    }
    if (E[horz].next_lml != kNil) {
      if (E[horz].out_idx >= 0) {
        op1 = add_out_pt(horz, E[horz].tx, E[horz].ty);
        update_edge_into_ael(horz);
        if (fail) return;
        if (E[horz].wdelta == 0) return;
        const int ep = prv(horz), en = nxt(horz);
        if (ep != kNil && E[ep].cx == E[horz].bx && E[ep].cy == E[horz].by && E[ep].wdelta != 0 &&
            E[ep].out_idx >= 0 && E[ep].cy > E[ep].ty && slopes_edges(horz, ep)) {
          const int op2 = add_out_pt(ep, E[horz].bx, E[horz].by);
          add_join(op1, op2, E[horz].tx, E[horz].ty);
        } else if (en != kNil && E[en].cx == E[horz].bx && E[en].cy == E[horz].by &&
                   E[en].wdelta != 0 && E[en].out_idx >= 0 && E[en].cy > E[en].ty &&
                   slopes_edges(horz, en)) {
          const int op2 = add_out_pt(en, E[horz].bx, E[horz].by);
          add_join(op1, op2, E[horz].tx, E[horz].ty);
        }
      } else {
        update_edge_into_ael(horz);
      }
    } else {
      if (E[horz].out_idx >= 0) add_out_pt(horz, E[horz].tx, E[horz].ty);
      delete_from_ael(horz);
    }
  }
  CU_HD void process_horizontals() {
    while (sorted != kNil && tick()) {
      const int h = sorted;
      delete_from_sel(h);
      process_horizontal(h);
    }
  }

  // ---- local minima ------------------------------------------------------------
  CU_HD void insert_local_minima(long long bot_y) {
    while (cur_lm < n_lm && LM[cur_lm].y == bot_y) {
      if (!tick()) return;
      const int lb = LM[cur_lm].left, rb = LM[cur_lm].right;
      ++cur_lm;
      int op1 = kNil;
      // closed paths always have both bounds
      insert_into_ael(lb, kNil);
      insert_into_ael(rb, lb);
      set_winding_count(lb);
      E[rb].wcnt = E[lb].wcnt;
      E[rb].wcnt2 = E[lb].wcnt2;
      if (is_contributing(lb)) op1 = add_local_min_poly(lb, rb, E[lb].bx, E[lb].by);
      sb_push(E[lb].ty);
      if (is_horz(rb)) {
        add_to_sel(rb);
        if (E[rb].next_lml != kNil) sb_push(E[E[rb].next_lml].ty);
      } else {
        sb_push(E[rb].ty);
      }
      if (fail) return;
      if (op1 != kNil && is_horz(rb) && n_gj > 0 && E[rb].wdelta != 0) {
        for (int i = 0; i < n_gj; ++i) {
          const Join &g = GJ[i];
          if (horz_overlap(OP[g.op1].x, g.offx, E[rb].bx, E[rb].tx))
            add_join(g.op1, op1, g.offx, g.offy);
        }
      }
      const int lp = prv(lb);
      if (E[lb].out_idx >= 0 && lp != kNil && E[lp].cx == E[lb].bx && E[lp].out_idx >= 0 &&
          slopes4(E[lp].bx, E[lp].by, E[lp].tx, E[lp].ty, E[lb].cx, E[lb].cy, E[lb].tx, E[lb].ty) &&
          E[lb].wdelta != 0 && E[lp].wdelta != 0) {
        const int op2 = add_out_pt(lp, E[lb].bx, E[lb].by);
        add_join(op1, op2, E[lb].tx, E[lb].ty);
      }
      if (nxt(lb) != rb) {
        const int rp = prv(rb);
        if (E[rb].out_idx >= 0 && E[rp].out_idx >= 0 &&
            slopes4(E[rp].cx, E[rp].cy, E[rp].tx, E[rp].ty, E[rb].cx, E[rb].cy, E[rb].tx, E[rb].ty) &&
            E[rb].wdelta != 0 && E[rp].wdelta != 0) {
          const int op2 = add_out_pt(rp, E[rb].bx, E[rb].by);
          add_join(op1, op2, E[rb].tx, E[rb].ty);
        }
        int e = nxt(lb);
        if (e != kNil) {
          while (e != rb) {
            if (e == kNil || !tick()) { fail = true; return; }
            intersect_edges(rb, e, E[lb].cx, E[lb].cy);
            e = nxt(e);
          }
        }
      }
    }
  }

  // ---- top of scanbeam -------------------------------------------------------
  CU_HD void do_maxima(int e) {
    const int mp = maxima_pair_ex(e);
    if (mp == kNil) {
      if (E[e].out_idx >= 0) add_out_pt(e, E[e].tx, E[e].ty);
      delete_from_ael(e);
      return;
    }
    int en = nxt(e);
    while (en != kNil && en != mp) {
      if (!tick()) return;
      intersect_edges(e, en, E[e].tx, E[e].ty);
      swap_in_ael(e, en);
      en = nxt(e);
    }
    if (E[e].out_idx == kUnassigned && E[mp].out_idx == kUnassigned) {
      delete_from_ael(e);
      delete_from_ael(mp);
    } else if (E[e].out_idx >= 0 && E[mp].out_idx >= 0) {
      add_local_max_poly(e, mp, E[e].tx, E[e].ty);
      delete_from_ael(e);
      delete_from_ael(mp);
    } else {
      fail = true;  // Clipper throws "DoMaxima error"
    }
  }
  // ProcessEdgesAtTopOfScanbeam, walking the AEL array by index: after
  // DoMaxima Clipper resumes at ePrev->NextInAEL, which is the same index
  // (DoMaxima only moves and removes edges from e onwards).
  CU_HD void process_edges_at_top(long long top_y) {
    // kOpTop: every edge that does not end at top_y gets its Curr at top_y
    // (nothing below reads the Curr of another edge before the horizontals),
    // the edges that end there are listed in list order; the walk over them
    // below meets them in the order of Clipper's walk over the whole AEL
    // (DoMaxima only moves and removes edges from e onwards).
    const int n_end = bulk(kOpTop, 0, 0, top_y);
    for (int j = 0; j < n_end; ++j) {
      if (!tick()) return;
      int e = SPL[j];
      if (E[e].ael_pos < 0) continue;  // removed with an earlier maxima pair
      bool is_max = E[e].next_lml == kNil;
      if (is_max) {
        const int mp = maxima_pair_ex(e);
        is_max = mp == kNil || !is_horz(mp);
      }
      if (is_max) {
        do_maxima(e);
        if (fail) return;
        continue;
      }
      if (E[e].next_lml != kNil && is_horz(E[e].next_lml)) {
        update_edge_into_ael(e);
        if (fail) return;
        if (E[e].out_idx >= 0) add_out_pt(e, E[e].bx, E[e].by);
        add_to_sel(e);
      } else {
        E[e].cx = (int)top_x(e, top_y);
        E[e].cy = (int)top_y;
      }
    }
    process_horizontals();
    if (fail) return;
    // intermediate vertices at top_y, in list order (kOpPromote)
    const int n_pro = bulk(kOpPromote, 0, 0, top_y);
    for (int j = 0; j < n_pro; ++j) {
      int e = SPL[j];
      {
        int op = kNil;
        if (E[e].out_idx >= 0) op = add_out_pt(e, E[e].tx, E[e].ty);
        update_edge_into_ael(e);
        if (fail) return;
        const int ep = prv(e), en = nxt(e);
        if (ep != kNil && E[ep].cx == E[e].bx && E[ep].cy == E[e].by && op != kNil &&
            E[ep].out_idx >= 0 && E[ep].cy > E[ep].ty &&
            slopes4(E[e].cx, E[e].cy, E[e].tx, E[e].ty, E[ep].cx, E[ep].cy, E[ep].tx, E[ep].ty) &&
            E[e].wdelta != 0 && E[ep].wdelta != 0) {
          const int op2 = add_out_pt(ep, E[e].bx, E[e].by);
          add_join(op, op2, E[e].tx, E[e].ty);
        } else if (en != kNil && E[en].cx == E[e].bx && E[en].cy == E[e].by && op != kNil &&
                   E[en].out_idx >= 0 && E[en].cy > E[en].ty &&
                   slopes4(E[e].cx, E[e].cy, E[e].tx, E[e].ty, E[en].cx, E[en].cy, E[en].tx,
                           E[en].ty) &&
                   E[e].wdelta != 0 && E[en].wdelta != 0) {
          const int op2 = add_out_pt(en, E[e].bx, E[e].by);
          add_join(op, op2, E[e].tx, E[e].ty);
        }
      }
    }
  }

  // ---- joins -------------------------------------------------------------------
  CU_HD int dup_out_pt(int op, bool after) {
    const int r = new_outpt();
    OP[r].x = OP[op].x;
    OP[r].y = OP[op].y;
    OP[r].idx = OP[op].idx;
    if (after) {
      OP[r].next = OP[op].next;
      OP[r].prev = op;
      OP[OP[op].next].prev = r;
      OP[op].next = r;
    } else {
      OP[r].prev = OP[op].prev;
      OP[r].next = op;
      OP[OP[op].prev].next = r;
      OP[op].prev = r;
    }
    return r;
  }
  CU_HD bool join_horz(int op1, int op1b, int op2, int op2b, long long px, long long py,
                       bool discard_left) {
    const bool d1_l2r = !(OP[op1].x > OP[op1b].x);
    const bool d2_l2r = !(OP[op2].x > OP[op2b].x);
    if (d1_l2r == d2_l2r) return false;
    auto walk = [&](int &op, int &opb, bool l2r) {
      if (l2r) {
        while (OP[OP[op].next].x <= px && OP[OP[op].next].x >= OP[op].x && OP[OP[op].next].y == py) {
          if (!tick()) return;
          op = OP[op].next;
        }
        if (discard_left && OP[op].x != px) op = OP[op].next;
        opb = dup_out_pt(op, !discard_left);
        if (OP[opb].x != px || OP[opb].y != py) {
          op = opb;
          OP[op].x = (int)px; OP[op].y = (int)py;
          opb = dup_out_pt(op, !discard_left);
        }
      } else {
        while (OP[OP[op].next].x >= px && OP[OP[op].next].x <= OP[op].x && OP[OP[op].next].y == py) {
          if (!tick()) return;
          op = OP[op].next;
        }
        if (!discard_left && OP[op].x != px) op = OP[op].next;
        opb = dup_out_pt(op, discard_left);
        if (OP[opb].x != px || OP[opb].y != py) {
          op = opb;
          OP[op].x = (int)px; OP[op].y = (int)py;
          opb = dup_out_pt(op, discard_left);
        }
      }
    };
    walk(op1, op1b, d1_l2r);
    walk(op2, op2b, d2_l2r);
    if (d1_l2r == discard_left) {
      OP[op1].prev = op2; OP[op2].next = op1;
      OP[op1b].next = op2b; OP[op2b].prev = op1b;
    } else {
      OP[op1].next = op2; OP[op2].prev = op1;
      OP[op1b].prev = op2b; OP[op2b].next = op1b;
    }
    return true;
  }
  CU_HD bool join_points(int ji, int r1, int r2) {
    Join &j = JN[ji];
    int op1 = j.op1, op2 = j.op2, op1b, op2b;
    const bool horizontal = OP[j.op1].y == j.offy;
    if (horizontal && j.offx == OP[j.op1].x && j.offy == OP[j.op1].y && j.offx == OP[j.op2].x &&
        j.offy == OP[j.op2].y) {
      // strictly simple joins: only created with StrictlySimple (not here)
      if (r1 != r2) return false;
      op1b = OP[j.op1].next;
      while (op1b != op1 && OP[op1b].x == j.offx && OP[op1b].y == j.offy) { if (!tick()) return false; op1b = OP[op1b].next; }
      const bool rev1 = OP[op1b].y > j.offy;
      op2b = OP[j.op2].next;
      while (op2b != op2 && OP[op2b].x == j.offx && OP[op2b].y == j.offy) { if (!tick()) return false; op2b = OP[op2b].next; }
      const bool rev2 = OP[op2b].y > j.offy;
      if (rev1 == rev2) return false;
      if (rev1) {
        op1b = dup_out_pt(op1, false);
        op2b = dup_out_pt(op2, true);
        OP[op1].prev = op2; OP[op2].next = op1;
        OP[op1b].next = op2b; OP[op2b].prev = op1b;
      } else {
        op1b = dup_out_pt(op1, true);
        op2b = dup_out_pt(op2, false);
        OP[op1].next = op2; OP[op2].prev = op1;
        OP[op1b].prev = op2b; OP[op2b].next = op1b;
      }
      j.op1 = op1;
      j.op2 = op1b;
      return true;
    } else if (horizontal) {
      op1b = op1;
      while (OP[OP[op1].prev].y == OP[op1].y && OP[op1].prev != op1b && OP[op1].prev != op2) {
        if (!tick()) return false;
        op1 = OP[op1].prev;
      }
      while (OP[OP[op1b].next].y == OP[op1b].y && OP[op1b].next != op1 && OP[op1b].next != op2) {
        if (!tick()) return false;
        op1b = OP[op1b].next;
      }
      if (OP[op1b].next == op1 || OP[op1b].next == op2) return false;
      op2b = op2;
      while (OP[OP[op2].prev].y == OP[op2].y && OP[op2].prev != op2b && OP[op2].prev != op1b) {
        if (!tick()) return false;
        op2 = OP[op2].prev;
      }
      while (OP[OP[op2b].next].y == OP[op2b].y && OP[op2b].next != op2 && OP[op2b].next != op1) {
        if (!tick()) return false;
        op2b = OP[op2b].next;
      }
      if (OP[op2b].next == op2 || OP[op2b].next == op1) return false;
      long long l, r;
      {
        const long long a1 = OP[op1].x, a2 = OP[op1b].x, b1 = OP[op2].x, b2 = OP[op2b].x;
        if (a1 < a2) {
          if (b1 < b2) { l = a1 > b1 ? a1 : b1; r = a2 < b2 ? a2 : b2; }
          else { l = a1 > b2 ? a1 : b2; r = a2 < b1 ? a2 : b1; }
        } else {
          if (b1 < b2) { l = a2 > b1 ? a2 : b1; r = a1 < b2 ? a1 : b2; }
          else { l = a2 > b2 ? a2 : b2; r = a1 < b1 ? a1 : b1; }
        }
        if (!(l < r)) return false;
      }
      long long px, py;
      bool discard_left;
      if (OP[op1].x >= l && OP[op1].x <= r) {
        px = OP[op1].x; py = OP[op1].y; discard_left = OP[op1].x > OP[op1b].x;
      } else if (OP[op2].x >= l && OP[op2].x <= r) {
        px = OP[op2].x; py = OP[op2].y; discard_left = OP[op2].x > OP[op2b].x;
      } else if (OP[op1b].x >= l && OP[op1b].x <= r) {
        px = OP[op1b].x; py = OP[op1b].y; discard_left = OP[op1b].x > OP[op1].x;
      } else {
        px = OP[op2b].x; py = OP[op2b].y; discard_left = OP[op2b].x > OP[op2].x;
      }
      j.op1 = op1;
      j.op2 = op2;
      return join_horz(op1, op1b, op2, op2b, px, py, discard_left);
    } else {
      op1b = OP[op1].next;
      while (OP[op1b].x == OP[op1].x && OP[op1b].y == OP[op1].y && op1b != op1) {
        if (!tick()) return false;
        op1b = OP[op1b].next;
      }
      const bool rev1 = OP[op1b].y > OP[op1].y ||
                        !slopes3(OP[op1].x, OP[op1].y, OP[op1b].x, OP[op1b].y, j.offx, j.offy);
      if (rev1) {
        op1b = OP[op1].prev;
        while (OP[op1b].x == OP[op1].x && OP[op1b].y == OP[op1].y && op1b != op1) {
          if (!tick()) return false;
          op1b = OP[op1b].prev;
        }
        if (OP[op1b].y > OP[op1].y ||
            !slopes3(OP[op1].x, OP[op1].y, OP[op1b].x, OP[op1b].y, j.offx, j.offy))
          return false;
      }
      op2b = OP[op2].next;
      while (OP[op2b].x == OP[op2].x && OP[op2b].y == OP[op2].y && op2b != op2) {
        if (!tick()) return false;
        op2b = OP[op2b].next;
      }
      const bool rev2 = OP[op2b].y > OP[op2].y ||
                        !slopes3(OP[op2].x, OP[op2].y, OP[op2b].x, OP[op2b].y, j.offx, j.offy);
      if (rev2) {
        op2b = OP[op2].prev;
        while (OP[op2b].x == OP[op2].x && OP[op2b].y == OP[op2].y && op2b != op2) {
          if (!tick()) return false;
          op2b = OP[op2b].prev;
        }
        if (OP[op2b].y > OP[op2].y ||
            !slopes3(OP[op2].x, OP[op2].y, OP[op2b].x, OP[op2b].y, j.offx, j.offy))
          return false;
      }
      if (op1b == op1 || op2b == op2 || op1b == op2b || (r1 == r2 && rev1 == rev2)) return false;
      if (rev1) {
        op1b = dup_out_pt(op1, false);
        op2b = dup_out_pt(op2, true);
        OP[op1].prev = op2; OP[op2].next = op1;
        OP[op1b].next = op2b; OP[op2b].prev = op1b;
      } else {
        op1b = dup_out_pt(op1, true);
        op2b = dup_out_pt(op2, false);
        OP[op1].next = op2; OP[op2].prev = op1;
        OP[op1b].prev = op2b; OP[op2b].next = op1b;
      }
      j.op1 = op1;
      j.op2 = op1b;
      return true;
    }
  }
  CU_HD int get_outrec(int idx) {
    int r = idx;
    while (r != OR[r].idx) {
      if (!tick()) return r;
      r = OR[r].idx;
    }
    return r;
  }
  CU_HD int point_in_polygon(long long px, long long py, int op) {
    int result = 0;
    const int start = op;
    for (;;) {
      if (!tick()) return 0;
      const OutPt &a = OP[op], &b = OP[OP[op].next];
      if (b.y == py) {
        if (b.x == px || (a.y == py && ((b.x > px) == (a.x < px)))) return -1;
      }
      if ((a.y < py) != (b.y < py)) {
        if (a.x >= px) {
          if (b.x > px) {
            result = 1 - result;
          } else {
            // integer products below 2^53: exact however it is evaluated
            const double d = (double)(a.x - px) * (double)(b.y - py) -
                             (double)(b.x - px) * (double)(a.y - py);
            if (d == 0) return -1;
            if ((d > 0) == (b.y > a.y)) result = 1 - result;
          }
        } else if (b.x > px) {
          const double d = (double)(a.x - px) * (double)(b.y - py) -
                           (double)(b.x - px) * (double)(a.y - py);
          if (d == 0) return -1;
          if ((d > 0) == (b.y > a.y)) result = 1 - result;
        }
      }
      op = OP[op].next;
      if (op == start) break;
    }
    return result;
  }
  CU_HD bool poly2_contains_poly1(int p1, int p2) {
    int op = p1;
    do {
      if (!tick()) return false;
      const int res = point_in_polygon(OP[op].x, OP[op].y, p2);
      if (res >= 0) return res > 0;
      op = OP[op].next;
    } while (op != p1);
    return true;
  }
  CU_HD void update_outpt_idxs(int r) {
    int op = OR[r].pts;
    do {
      if (!tick()) return;
      OP[op].idx = OR[r].idx;
      op = OP[op].prev;
    } while (op != OR[r].pts);
  }
  CU_HD void join_common_edges() {
    for (int i = 0; i < n_jn; ++i) {
      if (fail) return;
      int r1 = get_outrec(OP[JN[i].op1].idx);
      int r2 = get_outrec(OP[JN[i].op2].idx);
      if (OR[r1].pts == kNil || OR[r2].pts == kNil) continue;
      int hole_rec;
      if (r1 == r2) hole_rec = r1;
      else if (outrec1_right_of_outrec2(r1, r2)) hole_rec = r2;
      else if (outrec1_right_of_outrec2(r2, r1)) hole_rec = r1;
      else hole_rec = lowermost_rec(r1, r2);
      if (!join_points(i, r1, r2)) continue;
      if (fail) return;
      if (r1 == r2) {
        OR[r1].pts = JN[i].op1;
        OR[r1].bottom_pt = kNil;
        r2 = create_outrec();
        OR[r2].pts = JN[i].op2;
        update_outpt_idxs(r2);
        if (poly2_contains_poly1(OR[r2].pts, OR[r1].pts)) {
          OR[r2].is_hole = !OR[r1].is_hole;
          OR[r2].first_left = r1;
          if ((OR[r2].is_hole != 0) == (area_op(OR[r2].pts) > 0)) reverse_links(OR[r2].pts);
        } else if (poly2_contains_poly1(OR[r1].pts, OR[r2].pts)) {
          OR[r2].is_hole = OR[r1].is_hole;
          OR[r1].is_hole = !OR[r2].is_hole;
          OR[r2].first_left = OR[r1].first_left;
          OR[r1].first_left = r2;
          if ((OR[r1].is_hole != 0) == (area_op(OR[r1].pts) > 0)) reverse_links(OR[r1].pts);
        } else {
          OR[r2].is_hole = OR[r1].is_hole;
          OR[r2].first_left = OR[r1].first_left;
        }
      } else {
        OR[r2].pts = kNil;
        OR[r2].bottom_pt = kNil;
        OR[r2].idx = OR[r1].idx;
        OR[r1].is_hole = OR[hole_rec].is_hole;
        if (hole_rec == r2) OR[r1].first_left = OR[r2].first_left;
        OR[r2].first_left = r1;
      }
    }
  }
  CU_HD void fixup_out_polygon(int r) {
    int last_ok = kNil;
    OR[r].bottom_pt = kNil;
    int pp = OR[r].pts;
    for (;;) {
      if (!tick()) return;
      if (OP[pp].prev == pp || OP[pp].prev == OP[pp].next) {
        OR[r].pts = kNil;
        return;
      }
      const OutPt &a = OP[OP[pp].prev], &b = OP[pp], &c = OP[OP[pp].next];
      if ((b.x == c.x && b.y == c.y) || (b.x == a.x && b.y == a.y) ||
          slopes3(a.x, a.y, b.x, b.y, c.x, c.y)) {
        last_ok = kNil;
        OP[OP[pp].prev].next = OP[pp].next;
        OP[OP[pp].next].prev = OP[pp].prev;
        pp = OP[pp].prev;
      } else if (pp == last_ok) {
        break;
      } else {
        if (last_ok == kNil) last_ok = pp;
        pp = OP[pp].next;
      }
    }
    OR[r].pts = pp;
  }

  // ---- the whole union -------------------------------------------------------
  // Runs Execute(ctUnion, pftPositive) on path[0..n). Returns false on a
  // capacity/bound failure (result unusable) and true otherwise; the output
  // rings are then the OutRecs with pts != kNil.
  CU_HD bool execute(const P2 *path, int n) {
#if !defined(__CUDA_ARCH__)
    if (bk == nullptr) {  // host: the list-wide steps run on this thread
      BulkArgs local;
      set_bulk(&local, g_host_runner ? g_host_lanes : 1);
      const bool ok = execute_impl(path, n);
      set_bulk(nullptr, 1);
      return ok;
    }
#endif
    if (bk == nullptr) { fail = true; return false; }
    return execute_impl(path, n);
  }
  CU_HD bool execute_impl(const P2 *path, int n) {
    if (!add_path(path, n)) return !fail;  // nothing added: empty solution
    std_sort(LM, n_lm, [](const LocMin &a, const LocMin &b) { return b.y < a.y; }, STK,
             cap.stack, &fail);
    if (fail) return false;
    cur_lm = 0;
    n_sb = 0;
    for (int i = 0; i < n_lm; ++i) {
      sb_push(LM[i].y);
      const int l = LM[i].left, r = LM[i].right;
      E[l].cx = E[l].bx; E[l].cy = E[l].by; E[l].side = kSideLeft; E[l].out_idx = kUnassigned;
      E[r].cx = E[r].bx; E[r].cy = E[r].by; E[r].side = kSideRight; E[r].out_idx = kUnassigned;
    }
    ael_n = 0;
    sorted = kNil;
    long long bot_y, top_y;
    if (!pop_scanbeam(&bot_y)) return !fail;
    insert_local_minima(bot_y);
    while (tick() && (pop_scanbeam(&top_y) || cur_lm < n_lm)) {
      process_horizontals();
      n_gj = 0;
      if (fail) return false;
      if (!process_intersections(top_y)) return false;
      process_edges_at_top(top_y);
      if (fail) return false;
      bot_y = top_y;
      insert_local_minima(bot_y);
    }
    if (fail) return false;
    for (int i = 0; i < n_or; ++i) {
      if (OR[i].pts == kNil) continue;
      if ((OR[i].is_hole != 0) == (area_op(OR[i].pts) > 0)) reverse_links(OR[i].pts);
    }
    if (n_jn > 0) join_common_edges();
    if (fail) return false;
    for (int i = 0; i < n_or; ++i)
      if (OR[i].pts != kNil) fixup_out_polygon(i);
    return !fail;
  }

  // Point count of a ring, or 0.
  CU_HD int ring_count(int pts) {
    if (pts == kNil) return 0;
    int n = 0, p = pts;
    do {
      if (!tick()) return 0;
      ++n;
      p = OP[p].next;
    } while (p != pts);
    return n;
  }
  // Signed area of a solution path as ClipperLib::Area(const Path&) computes
  // it on the BuildResult order (Pts->Prev, walking Prev).
  CU_HD double path_area(int pts) {
    const int cnt = ring_count(pts);
    if (cnt < 3) return 0;
    // path[i] = the i-th point walking prev from pts->prev
    double a = 0;
    int pj = OP[pts].prev;            // path[0]
    for (int k = 0; k < cnt - 1; ++k) pj = OP[pj].prev;  // path[cnt-1]
    int pi = OP[pts].prev;
    for (int i = 0; i < cnt; ++i) {
      if (!tick()) return 0;
      a = fma((double)OP[pj].x + (double)OP[pi].x, (double)OP[pj].y - (double)OP[pi].y, a);
      pj = pi;
      pi = OP[pi].prev;
    }
    return -a * 0.5;
  }
  // The ring unclip keeps: std::max_element by Area over the solution paths
  // in BuildResult order (rings of fewer than 2 points are not paths).
  // Writes it to out (cap points) in path order; returns its length, 0 when
  // the solution is empty, -1 on failure or overflow.
  CU_HD int best_ring(P2 *out, int out_cap) {
    int best = kNil;
    double best_area = 0;
    for (int i = 0; i < n_or; ++i) {
      if (OR[i].pts == kNil) continue;
      const int cnt = ring_count(OP[OR[i].pts].prev);
      if (cnt < 2) continue;
      const double a = path_area(OR[i].pts);
      if (best == kNil || best_area < a) {
        best = i;
        best_area = a;
      }
    }
    if (fail) return -1;
    if (best == kNil) return 0;
    const int cnt = ring_count(OR[best].pts);
    if (cnt > out_cap) return -1;
    int p = OP[OR[best].pts].prev;
    for (int i = 0; i < cnt; ++i) {
      out[i].x = (int)OP[p].x;
      out[i].y = (int)OP[p].y;
      p = OP[p].prev;
    }
    return cnt;
  }
};

}  // namespace cu
}  // namespace db
}  // namespace tocr
