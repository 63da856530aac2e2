"""ORACLE (test infrastructure only) for subsystem 1, det preprocessing:
ctypes access to oracle/preprocess_oracle.c, the CPU restatement of
src/kernels/preprocess_kernels.cu:19-54,128-201 and of compute_det_resize
(include/turbo_ocr/detection/det_config.h:58-81)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._loader import load

DET_MEAN = np.array([0.485, 0.456, 0.406], dtype=np.float32)
DET_INV_STD = np.array([1.0 / np.float32(0.229), 1.0 / np.float32(0.224),
                        1.0 / np.float32(0.225)], dtype=np.float32)


def _lib():
    lib = load("_build/liboracle.so")
    lib.oracle_preprocess_image.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                            C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                            C.c_void_p]
    lib.oracle_det_resize.argtypes = [C.c_int] * 5 + [C.POINTER(C.c_int)] * 2
    return lib


def det_resize(h: int, w: int, limit_type: str = "max", limit_side_len: int = 960,
               max_side_limit: int = 960) -> tuple[int, int]:
    oh, ow = C.c_int(), C.c_int()
    _lib().oracle_det_resize(h, w, 1 if limit_type == "max" else 0, limit_side_len,
                             max_side_limit, C.byref(oh), C.byref(ow))
    return oh.value, ow.value


def preprocess_image(src: np.ndarray, content_hw, canvas_hw, mean=DET_MEAN,
                     inv_std=DET_INV_STD, hw=None, step: int | None = None) -> np.ndarray:
    """src u8 [h, w, 3] contiguous, or a pitched byte buffer with explicit
    hw=(h, w) and step -> fp32 [3, H, W]."""
    src = np.ascontiguousarray(src)
    h, w = hw if hw is not None else src.shape[:2]
    step = step if step is not None else w * 3
    H, W = canvas_hw
    out = np.empty((3, H, W), dtype=np.float32)
    m = np.ascontiguousarray(mean, dtype=np.float32)
    s = np.ascontiguousarray(inv_std, dtype=np.float32)
    _lib().oracle_preprocess_image(src.ctypes.data, h, w, step, content_hw[0], content_hw[1],
                                   out.ctypes.data, H, W, m.ctypes.data, s.ctypes.data)
    return out
