"""ORACLE: the reference's compute_crop_transform
(include/turbo_ocr/common/geometry/perspective.h:25-67), compiled from the
reference header into oracle/_ref/libcrop_ref.so (test infrastructure)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._loader import load


def _lib():
    L = load("_ref/libcrop_ref.so")
    if not getattr(L, "_tocr_ready", False):
        L.crop_ref_transform.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                         C.c_void_p]
        L._tocr_ready = True
    return L


def crop_transform_full(box, target_h: int, max_width: int):
    """-> (M_inv float32[9], crop width, vertical flag)."""
    b = np.ascontiguousarray(np.asarray(box, np.int32).reshape(8))
    m = np.zeros(9, np.float32)
    cw, v = C.c_int(), C.c_int()
    _lib().crop_ref_transform(b.ctypes.data, target_h, max_width, m.ctypes.data, C.byref(cw),
                              C.byref(v))
    return m, cw.value, v.value


def crop_transform(box, target_h: int, max_width: int) -> np.ndarray:
    return crop_transform_full(box, target_h, max_width)[0]
