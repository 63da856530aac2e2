// Test-infrastructure wrapper (oracle only): the reference's vendored
// Clipper 6.4.2 (third_party/clipper/clipper.cpp, compiled unchanged by
// oracle/Makefile) driven exactly like unclip() in
// src/detection/det_postprocess.cpp:72-101 — ClipperOffset with its default
// MiterLimit 2 / ArcTolerance 0.25, jtRound, etClosedPolygon, Execute(delta),
// largest ring by Area. Also exposes the raw offset vertices (before the
// union) for the GPU restatement's tests.
#include <algorithm>
#include <vector>

// Test access to the offsetter's intermediate (pre-union) path.
#define private public
#define protected public
#include "clipper/clipper.hpp"
#undef private
#undef protected

using namespace ClipperLib;

extern "C" {

// Returns the number of points of the largest ring written to out_xy (pairs),
// 0 when the solution is empty, or -needed if cap is too small.
int clipper_ref_unclip(const int *xy, int n, double distance, long long *out_xy, int cap,
                       int *n_rings) {
  ClipperOffset co;
  Path subj;
  for (int i = 0; i < n; ++i) subj.emplace_back(xy[2 * i], xy[2 * i + 1]);
  co.AddPath(subj, jtRound, etClosedPolygon);
  Paths sol;
  co.Execute(sol, distance);
  *n_rings = (int)sol.size();
  if (sol.empty()) return 0;
  const Path *best = &sol.front();
  if (sol.size() > 1) {
    best = &*std::max_element(sol.begin(), sol.end(), [](const Path &a, const Path &b) {
      return Area(a) < Area(b);
    });
  }
  const int m = (int)best->size();
  if (m > cap) return -m;
  for (int i = 0; i < m; ++i) {
    out_xy[2 * i] = (*best)[i].X;
    out_xy[2 * i + 1] = (*best)[i].Y;
  }
  return m;
}

// The raw offset path of ClipperOffset (after FixOrientations + DoOffset,
// before the union that Execute applies). Returns its point count, 0 if the
// offsetter produced no path, or -needed if cap is too small.
int clipper_ref_raw_offset(const int *xy, int n, double distance, long long *out_xy, int cap) {
  ClipperOffset co;
  Path subj;
  for (int i = 0; i < n; ++i) subj.emplace_back(xy[2 * i], xy[2 * i + 1]);
  co.AddPath(subj, jtRound, etClosedPolygon);
  co.FixOrientations();
  co.DoOffset(distance);
  if (co.m_destPolys.empty()) return 0;
  const Path &p = co.m_destPolys.front();
  const int m = (int)p.size();
  if (m > cap) return -m;
  for (int i = 0; i < m; ++i) {
    out_xy[2 * i] = p[i].X;
    out_xy[2 * i + 1] = p[i].Y;
  }
  return m;
}

}  // extern "C"
