"""Detection resize policy and DB parameters (the reference's
include/turbo_ocr/detection/det_config.h), computed by the library's C++
(include/turbo_ocr/detection/det_config.h here) through the C-ABI, so the
Python path, the C++ modules and the benchmark share one arithmetic."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from ._lib import check, lib

K_DET_MAX_SIDE_MIN, K_DET_MAX_SIDE_MAX = 32, 4096


@dataclass(frozen=True)
class DetResizeParams:
    limit_type: str = "min"      # "max": shrink the longer side; "min": grow the shorter
    limit_side_len: int = 64
    max_side_limit: int = 1280


@dataclass(frozen=True)
class DbParams:
    thresh: float = 0.2
    box_thresh: float = 0.45
    unclip_ratio: float = 1.4


K_DET_RESIZE_DEFAULT = DetResizeParams()
K_DB_DEFAULTS = DbParams()


def compute_det_resize(h: int, w: int, p: DetResizeParams = K_DET_RESIZE_DEFAULT):
    """(resize_h, resize_w) of an h x w image (det_config.h:58-81)."""
    oh, ow = C.c_int(), C.c_int()
    check(lib().tocr_compute_det_resize(h, w, 1 if p.limit_type.startswith("ma") else 0,
                                        p.limit_side_len, p.max_side_limit, C.byref(oh),
                                        C.byref(ow)), "compute_det_resize")
    return oh.value, ow.value


def read_det_resize(base: DetResizeParams = K_DET_RESIZE_DEFAULT) -> DetResizeParams:
    """Environment overrides (DET_LIMIT_TYPE, DET_LIMIT_SIDE_LEN,
    DET_MAX_SIDE_LIMIT, DET_MAX_SIDE) on top of `base`."""
    t = C.c_int(1 if base.limit_type.startswith("ma") else 0)
    n, m = C.c_int(base.limit_side_len), C.c_int(base.max_side_limit)
    check(lib().tocr_read_det_resize(C.byref(t), C.byref(n), C.byref(m)), "read_det_resize")
    return DetResizeParams("max" if t.value else "min", n.value, m.value)


def read_db_params(base: DbParams = K_DB_DEFAULTS) -> DbParams:
    """Environment overrides (DET_DB_THRESH, DET_BOX_THRESH, DET_UNCLIP)."""
    a, b, c = C.c_float(base.thresh), C.c_float(base.box_thresh), C.c_float(base.unclip_ratio)
    check(lib().tocr_read_db_params(C.byref(a), C.byref(b), C.byref(c)), "read_db_params")
    return DbParams(a.value, b.value, c.value)


def effective_det_max_side(p: DetResizeParams = K_DET_RESIZE_DEFAULT) -> int:
    return int(lib().tocr_effective_det_max_side(p.max_side_limit))
