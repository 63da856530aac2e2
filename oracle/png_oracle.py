"""Test infrastructure only: the reference's PNG decode on the host.

FastPngDecoder::decode (src/decode/fast_png_decoder.cpp:48-128) restated as
a driver of the real thing: the reference's vendored Wuffs v0.4 compiled in
place into _ref/libpng_ref.so (png_ref_wrap.c, driven the way lines 64-127
drive it), and for 16-bit files the reference's OpenCV route
(fast_png_decoder.cpp:46-62: the same caps read from the IHDR, then
cv::imdecode(IMREAD_COLOR)). Returns BGR u8 HWC like the reference's cv::Mat,
or None where the reference returns an empty Mat."""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np

from ._loader import load


def _env_int(name: str, default: int, lo: int, hi: int) -> int:
    v = os.environ.get(name)
    if not v:
        return default
    try:
        x = int(v, 10)
    except ValueError:
        return default
    return min(max(x, lo), hi)


def max_image_dim() -> int:  # image_config.h:13-16
    return _env_int("MAX_IMAGE_DIM", 16384, 64, 65535)


def max_image_pixels() -> int:  # image_config.h:31-36
    return _env_int("MAX_IMAGE_PIXELS_MP", 128, 1, 4096) * 1000000


def _lib() -> C.CDLL:
    L = load("_ref/libpng_ref.so")
    L.png_ref_decode_bgr.argtypes = [C.c_void_p, C.c_size_t, C.c_uint32, C.c_int64, C.c_void_p,
                                     C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
    L.png_ref_decode_bgr.restype = C.c_int
    L.png_ref_info.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32),
                               C.POINTER(C.c_uint32)]
    L.png_ref_last_status.restype = C.c_char_p
    return L


def wuffs_decode(data: bytes, max_dim: int | None = None, max_pixels: int | None = None):
    """(image or None, Wuffs status text) for the 8-bit path."""
    L = _lib()
    md = max_image_dim() if max_dim is None else max_dim
    mp = max_image_pixels() if max_pixels is None else max_pixels
    w, h = C.c_uint32(), C.c_uint32()
    if L.png_ref_info(data, len(data), C.byref(w), C.byref(h)) != 0:
        return None, L.png_ref_last_status().decode()
    ww, hh = w.value, h.value
    if ww == 0 or hh == 0 or ww > md or hh > md or ww * hh > mp:
        return None, "over the caps"
    out = np.empty(ww * hh * 3, np.uint8)
    rc = L.png_ref_decode_bgr(data, len(data), md, mp, out.ctypes.data, out.size, C.byref(w),
                              C.byref(h))
    if rc != 0:
        return None, L.png_ref_last_status().decode() or f"rc {rc}"
    return out.reshape(hh, ww, 3), ""


def reference_decode(data: bytes, max_dim: int | None = None, max_pixels: int | None = None):
    """FastPngDecoder::decode: BGR u8 (h, w, 3) or None."""
    md = max_image_dim() if max_dim is None else max_dim
    mp = max_image_pixels() if max_pixels is None else max_pixels
    if len(data) >= 26 and data[:4] == b"\x89PNG" and data[24] == 16:
        w, h = struct.unpack(">II", data[16:24])
        if w == 0 or h == 0 or w > md or h > md or w * h > mp:
            return None
        import cv2
        img = cv2.imdecode(np.frombuffer(data, np.uint8), cv2.IMREAD_COLOR)
        return img
    return wuffs_decode(data, md, mp)[0]
