// Box type and box utilities of the reference
// (include/turbo_ocr/common/geometry/box.h:18-77 in TurboOCR): the same names,
// layout and semantics, so pipeline code compiles unchanged against them.
#pragma once

#include <algorithm>
#include <array>
#include <compare>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <utility>
#include <vector>

namespace turbo_ocr {

// Four corners [tl, tr, br, bl], each [x, y].
struct Box {
  std::array<std::array<int, 2>, 4> pts;

  constexpr auto &operator[](std::size_t i) noexcept { return pts[i]; }
  constexpr const auto &operator[](std::size_t i) const noexcept { return pts[i]; }
  constexpr auto operator<=>(const Box &) const noexcept = default;
};

// A crop is vertical text when its height is at least 1.5x its width.
inline constexpr float kVerticalAspectRatio = 1.5f;

// [x0, y0, x1, y1] over all four corners (rotated quads included).
[[nodiscard]] inline std::array<int, 4> aabb(const Box &b) noexcept {
  int x0 = b[0][0], x1 = b[0][0], y0 = b[0][1], y1 = b[0][1];
  for (int k = 1; k < 4; ++k) {
    x0 = std::min(x0, b[k][0]);
    x1 = std::max(x1, b[k][0]);
    y0 = std::min(y0, b[k][1]);
    y1 = std::max(y1, b[k][1]);
  }
  return {x0, y0, x1, y1};
}

// The AABB clamped to [0, cols) x [0, rows) as [x0, y0, w, h], w and h >= 1.
[[nodiscard]] inline std::array<int, 4> clamped_crop_rect(const Box &b, int cols,
                                                          int rows) noexcept {
  const auto r = aabb(b);
  const int x0 = std::clamp(r[0], 0, std::max(0, cols - 1));
  const int y0 = std::clamp(r[1], 0, std::max(0, rows - 1));
  const int x1 = std::clamp(r[2], x0, cols);
  const int y1 = std::clamp(r[3], y0, rows);
  return {x0, y0, std::max(1, x1 - x0), std::max(1, y1 - y0)};
}

// Vertical when h >= 1.5 w, in integers: h^2 >= w^2 * 225 / 100, with w and h
// the longer of each pair of opposite edge extents.
[[nodiscard]] inline bool is_vertical_box(const Box &b) noexcept {
  const int w = std::max(std::abs(b[1][0] - b[0][0]), std::abs(b[2][0] - b[3][0]));
  const int h = std::max(std::abs(b[3][1] - b[0][1]), std::abs(b[2][1] - b[1][1]));
  return static_cast<int64_t>(h) * h >= static_cast<int64_t>(w) * w * 225 / 100;
}

// Reading order: stable sort by (top-left y / 10, top-left x).
inline void sorted_boxes(std::vector<Box> &dt_boxes) {
  constexpr int kSameLine = 10;
  std::stable_sort(dt_boxes.begin(), dt_boxes.end(), [](const Box &a, const Box &b) {
    const int ya = a[0][1] / kSameLine, yb = b[0][1] / kSameLine;
    if (ya != yb) return ya < yb;
    return a[0][0] < b[0][0];
  });
}

[[nodiscard]] inline std::pair<float, float> quad_centroid(const Box &b) noexcept {
  float cx = 0.0f, cy = 0.0f;
  for (int k = 0; k < 4; ++k) {
    cx += static_cast<float>(b[k][0]);
    cy += static_cast<float>(b[k][1]);
  }
  return {cx * 0.25f, cy * 0.25f};
}

[[nodiscard]] inline bool centroid_in_aabb(const Box &b, const std::array<int, 4> &r) noexcept {
  const auto [cx, cy] = quad_centroid(b);
  return cx >= static_cast<float>(r[0]) && cx <= static_cast<float>(r[2]) &&
         cy >= static_cast<float>(r[1]) && cy <= static_cast<float>(r[3]);
}

}  // namespace turbo_ocr
