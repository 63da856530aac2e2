"""ORACLE (test infrastructure only) for subsystem 3, DB post-processing.

Line-for-line restatement of the reference's CPU path
src/detection/det_postprocess.cpp in Python with OpenCV (cv2) and the
reference's own vendored Clipper 6.4.2 (third_party/clipper, compiled
unchanged into oracle/_ref/libclipper_ref.so by oracle/Makefile):

  extract_boxes_from_bitmap ... det_postprocess.cpp:145-222
  box_score_fast .............. det_postprocess.cpp:15-55
  unclip ...................... det_postprocess.cpp:57-102
  order_quad_tl_tr_br_bl ...... det_postprocess.cpp:104-126
  get_mini_boxes .............. det_postprocess.cpp:128-143
  threshold (cv::compare GT) .. src/detection/cpu_paddle_det.cpp:115

Unlike the reference (which returns only quads), every kept box also
carries its box_score_fast value. OpenCV is not pinned in the reference
(docker/Dockerfile.gpu:30 installs Ubuntu's libopencv-dev); this oracle uses
the cv2 of the build image, whose version tests record.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from ._loader import load

K_MAX_CANDIDATES = 3000  # det_postprocess.cpp:165-167


def _clipper():
    lib = load("_ref/libclipper_ref.so")
    if not getattr(lib, "_tocr_ready", False):
        lib.clipper_ref_unclip.argtypes = [C.c_void_p, C.c_int, C.c_double, C.c_void_p, C.c_int,
                                           C.POINTER(C.c_int)]
        lib.clipper_ref_unclip.restype = C.c_int
        lib._tocr_ready = True
    return lib


def cv2_version() -> str:
    import cv2
    return cv2.__version__


def _round_half_away(v) -> int:
    """std::round on a float value (half away from zero)."""
    v = float(np.float32(v))
    return int(math.copysign(math.floor(abs(v) + 0.5), v))


def order_quad(xs, ys):
    """Stable x-sort, then tl/bl by y on the left pair, tr/br on the right."""
    idx = sorted(range(4), key=lambda k: xs[k])  # Python sort is stable
    xs = [xs[k] for k in idx]
    ys = [ys[k] for k in idx]
    tl = 0 if ys[0] < ys[1] else 1
    bl = 1 - tl
    tr = 2 if ys[2] < ys[3] else 3
    br = 5 - tr
    return [xs[tl], xs[tr], xs[br], xs[bl]], [ys[tl], ys[tr], ys[br], ys[bl]]


def get_mini_boxes(contour: np.ndarray):
    """-> (box [[x,y]*4] ints tl,tr,br,bl ; min_side float32)."""
    import cv2
    rect = cv2.minAreaRect(contour)
    min_side = np.float32(min(rect[1][0], rect[1][1]))
    pts = cv2.boxPoints(rect)  # RotatedRect::points order, float32
    xs, ys = order_quad([np.float32(p[0]) for p in pts], [np.float32(p[1]) for p in pts])
    box = [[_round_half_away(xs[k]), _round_half_away(ys[k])] for k in range(4)]
    return box, min_side


def box_score_fast(pred: np.ndarray, contour: np.ndarray) -> float:
    import cv2
    h, w = pred.shape
    xmin, xmax, ymin, ymax = w, 0, h, 0
    for x, y in contour:
        xmin = min(xmin, max(0, int(x)))
        xmax = max(xmax, min(w - 1, int(x)))
        ymin = min(ymin, max(0, int(y)))
        ymax = max(ymax, min(h - 1, int(y)))
    if xmax <= xmin or ymax <= ymin:
        return 0.0
    shifted = (contour - np.array([xmin, ymin], dtype=contour.dtype)).astype(np.int32)
    mask = np.zeros((ymax - ymin + 1, xmax - xmin + 1), dtype=np.uint8)
    cv2.fillPoly(mask, [shifted.reshape(-1, 1, 2)], 1)
    roi = pred[ymin:ymax + 1, xmin:xmax + 1]
    return float(np.float32(cv2.mean(roi, mask)[0]))


def unclip(polygon: np.ndarray, unclip_ratio: float) -> np.ndarray:
    import cv2
    poly = polygon.reshape(-1, 1, 2).astype(np.int32)
    perimeter = cv2.arcLength(poly, True)
    if perimeter == 0.0:
        return polygon
    area = cv2.contourArea(poly)
    distance = area * float(np.float32(unclip_ratio)) / perimeter
    xy = np.ascontiguousarray(polygon.reshape(-1, 2), dtype=np.int32)
    cap = 1 << 16
    out = np.zeros(2 * cap, dtype=np.int64)
    nr = C.c_int()
    m = _clipper().clipper_ref_unclip(xy.ctypes.data, len(xy), C.c_double(distance),
                                      out.ctypes.data, cap, C.byref(nr))
    assert m >= 0, "ring larger than buffer"
    if m == 0:
        return polygon
    return out[: 2 * m].reshape(m, 2).astype(np.int32)


def find_contours(bitmap: np.ndarray):
    import cv2
    contours, _ = cv2.findContours(bitmap, cv2.RETR_LIST, cv2.CHAIN_APPROX_SIMPLE)
    return [c.reshape(-1, 2) for c in contours]


def extract_boxes_from_bitmap(pred: np.ndarray, bitmap: np.ndarray, orig_h: int, orig_w: int,
                              resize_h: int, resize_w: int, box_thresh: float,
                              unclip_ratio: float, min_box_side: float = 3.0,
                              min_unclipped_side: float = 5.0, unclip_fn=None):
    """-> list of (box [[x,y]*4], score) in the reference's contour order.
    unclip_fn(contour, ratio) replaces unclip() when given (tests use it to
    isolate the union step of Clipper's offset)."""
    import cv2
    ratio_h = np.float32(resize_h) / np.float32(orig_h)
    ratio_w = np.float32(resize_w) / np.float32(orig_w)
    contours = find_contours(bitmap)
    out = []
    for contour in contours[:K_MAX_CANDIDATES]:
        if len(contour) <= 2:
            continue
        _, _, bw, bh = cv2.boundingRect(contour.reshape(-1, 1, 2))
        if bw < 3 or bh < 3:
            continue
        _, ssid = get_mini_boxes(contour)
        if ssid < np.float32(min_box_side):
            continue
        score = box_score_fast(pred, contour)
        if np.float32(score) < np.float32(box_thresh):
            continue
        unclipped = (unclip_fn or unclip)(contour, unclip_ratio)
        if len(unclipped) < 3:
            continue
        box, ssid2 = get_mini_boxes(unclipped)
        if ssid2 < np.float32(min_unclipped_side):
            continue
        for k in range(4):
            box[k][0] = min(max(_round_half_away(np.float32(box[k][0]) / ratio_w), 0), orig_w - 1)
            box[k][1] = min(max(_round_half_away(np.float32(box[k][1]) / ratio_h), 0), orig_h - 1)
        dx01, dy01 = box[0][0] - box[1][0], box[0][1] - box[1][1]
        dx03, dy03 = box[0][0] - box[3][0], box[0][1] - box[3][1]
        rw = int(math.sqrt(float(dx01 * dx01 + dy01 * dy01)))
        rh = int(math.sqrt(float(dx03 * dx03 + dy03 * dy03)))
        if rw <= 3 or rh <= 3:
            continue
        out.append((box, float(np.float32(score))))
    return out


def threshold(pred: np.ndarray, thresh: float) -> np.ndarray:
    """cv::compare(pred, thresh, CMP_GT): 255 where pred > thresh."""
    return np.where(pred > np.float32(thresh), 255, 0).astype(np.uint8)


def db_postprocess(pred: np.ndarray, thresh=0.3, box_thresh=0.6, unclip_ratio=1.5,
                   unclip_fn=None):
    """Config-1 post-process of one map (orig == resize dims)."""
    h, w = pred.shape
    return extract_boxes_from_bitmap(pred, threshold(pred, thresh), h, w, h, w, box_thresh,
                                     unclip_ratio, unclip_fn=unclip_fn)


def unclip_distance(polygon: np.ndarray, unclip_ratio: float):
    """Offset distance of unclip (det_postprocess.cpp:59-66), None if the
    perimeter is 0."""
    import cv2
    poly = polygon.reshape(-1, 1, 2).astype(np.int32)
    perimeter = cv2.arcLength(poly, True)
    if perimeter == 0.0:
        return None
    return cv2.contourArea(poly) * float(np.float32(unclip_ratio)) / perimeter
