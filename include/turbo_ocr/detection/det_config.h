// Detection resize policy and DB parameters with the names, fields, defaults,
// environment variables and clamps of the reference
// (include/turbo_ocr/detection/det_config.h:13-163 in TurboOCR), so callers
// that build a DetResizeParams / DbParams keep compiling unchanged.
//
//   compute_det_resize  det_config.h:58-81   PaddleOCR resize_image_type0 + cap
//   round32_floor       det_config.h:50-52   std::round(v / 32) * 32, floor 32
//   read_det_resize     det_config.h:89-127  DET_LIMIT_TYPE / DET_LIMIT_SIDE_LEN /
//                                            DET_MAX_SIDE_LIMIT / DET_MAX_SIDE
//   read_db_params      det_config.h:132-141 DET_DB_THRESH / DET_BOX_THRESH / DET_UNCLIP
//   effective_det_max_side det_config.h:158-163
#pragma once

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <utility>

namespace turbo_ocr::detection {

inline constexpr int kDetMaxSideMin = 32;
inline constexpr int kDetMaxSideMax = 4096;

// limit_type "max": shrink the longer side to limit_side_len; "min": grow the
// shorter side to it. Either way the output's longer side is capped at
// max_side_limit.
struct DetResizeParams {
  const char *limit_type;
  int limit_side_len;
  int max_side_limit;
};

inline constexpr DetResizeParams kDetResizeDefault{"min", 64, 1280};

struct DbParams {
  float thresh;        // bitmap = prob > thresh
  float box_thresh;    // keep a box when its mean prob >= box_thresh
  float unclip_ratio;  // offset distance = area * ratio / perimeter
};

inline constexpr DbParams kDbDefaults{0.2f, 0.45f, 1.4f};

// Nearest multiple of 32 (halves away from zero, as std::round), at least 32.
[[nodiscard]] inline int round32_floor(double v) {
  const int r = static_cast<int>(std::round(v / 32.0) * 32);
  return r < 32 ? 32 : r;
}

namespace detail {
inline bool is_max_policy(const char *t) { return t && t[0] == 'm' && t[1] == 'a'; }
inline int env_side(const char *v) {
  return std::clamp(std::atoi(v), kDetMaxSideMin, kDetMaxSideMax);
}
}  // namespace detail

// (resize_h, resize_w): scale by a float ratio (the side times the ratio is
// a float product), round both sides to /32, then, when the longer result
// exceeds max_side_limit, rescale both by max_side_limit / longer (double)
// and round again.
[[nodiscard]] inline std::pair<int, int> compute_det_resize(int h, int w,
                                                            const DetResizeParams &p) {
  float ratio = 1.0f;
  if (detail::is_max_policy(p.limit_type)) {
    const int longer = h > w ? h : w;
    if (longer > p.limit_side_len) ratio = static_cast<float>(p.limit_side_len) / longer;
  } else {
    const int shorter = h < w ? h : w;
    if (shorter < p.limit_side_len) ratio = static_cast<float>(p.limit_side_len) / shorter;
  }
  int rh = round32_floor(h * ratio);
  int rw = round32_floor(w * ratio);
  const int longer = rh > rw ? rh : rw;
  if (longer > p.max_side_limit) {
    const double k = static_cast<double>(p.max_side_limit) / longer;
    rh = round32_floor(rh * k);
    rw = round32_floor(rw * k);
  }
  return {rh, rw};
}

// Environment overrides on top of a per-model base; a field changes only when
// its variable is set and non-empty. Numeric values clamp to [32, 4096].
// DET_MAX_SIDE can only lower max_side_limit (it also sizes the buffers).
// Switching a "min" base to "max" without DET_LIMIT_SIDE_LEN makes the
// max-side cap the limit (a "max" policy at 64 px would thumbnail pages).
[[nodiscard]] inline DetResizeParams read_det_resize(DetResizeParams base = kDetResizeDefault) {
  const bool base_min = !detail::is_max_policy(base.limit_type);
  bool len_set = false;
  if (const char *v = std::getenv("DET_LIMIT_TYPE")) {
    const bool mx = std::tolower(static_cast<unsigned char>(v[0])) == 'm' &&
                    std::tolower(static_cast<unsigned char>(v[0] ? v[1] : 0)) == 'a';
    base.limit_type = mx ? "max" : "min";
  }
  if (const char *v = std::getenv("DET_LIMIT_SIDE_LEN"); v && *v) {
    base.limit_side_len = detail::env_side(v);
    len_set = true;
  }
  if (const char *v = std::getenv("DET_MAX_SIDE_LIMIT"); v && *v)
    base.max_side_limit = detail::env_side(v);
  if (const char *v = std::getenv("DET_MAX_SIDE"); v && *v)
    base.max_side_limit = std::min(base.max_side_limit, detail::env_side(v));
  if (base_min && !len_set && detail::is_max_policy(base.limit_type)) {
    base.limit_side_len = base.max_side_limit;
    std::fprintf(stderr,
                 "[DetConfig] DET_LIMIT_TYPE=max set without DET_LIMIT_SIDE_LEN; "
                 "defaulting limit_side_len to the max-side cap (%d)\n",
                 base.max_side_limit);
  }
  return base;
}

[[nodiscard]] inline DbParams read_db_params(DbParams base = kDbDefaults) {
  if (const char *v = std::getenv("DET_DB_THRESH"); v && *v)
    base.thresh = static_cast<float>(std::atof(v));
  if (const char *v = std::getenv("DET_BOX_THRESH"); v && *v)
    base.box_thresh = static_cast<float>(std::atof(v));
  if (const char *v = std::getenv("DET_UNCLIP"); v && *v)
    base.unclip_ratio = static_cast<float>(std::atof(v));
  return base;
}

// Largest side the detector's buffers must hold: max_side_limit (DET_MAX_SIDE
// wins when set), clamped to [32, 4096] and rounded up to /32, because the
// re-rounding in compute_det_resize can exceed a non-/32 cap by up to 16 px.
[[nodiscard]] inline int effective_det_max_side(const DetResizeParams &p = kDetResizeDefault) {
  int v = p.max_side_limit;
  if (const char *e = std::getenv("DET_MAX_SIDE"); e && *e) v = std::atoi(e);
  v = std::clamp(v, kDetMaxSideMin, kDetMaxSideMax);
  return (v + 31) / 32 * 32;
}

}  // namespace turbo_ocr::detection
