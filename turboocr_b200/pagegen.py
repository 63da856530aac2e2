"""Seeded synthetic document pages and their PNG files: the input of the
PNG-decode benchmark (both arms decode the same bytes) and of the decode
tests. A page is white with dark text-like strokes, a few coloured blocks
and one noisy band, so its DEFLATE stream holds both long matches and
literal runs, like a scanned or rendered document."""
from __future__ import annotations

import numpy as np


def page_like(h: int, w: int, seed: int, channels: int = 3) -> np.ndarray:
    rng = np.random.default_rng(seed)
    img = np.full((h, w, channels), 250, np.uint8)
    for _ in range(max(1, h // 24)):
        y = int(rng.integers(0, max(1, h - 12)))
        x = int(rng.integers(0, max(1, w - 40)))
        L = int(rng.integers(10, max(11, w // 2)))
        img[y:y + 8, x:x + L] = rng.integers(0, 60, (1, 1, channels))
        for k in range(0, L, 7):
            img[y:y + 8, x + k:x + k + 2] = 245
    for _ in range(3):
        y, x = int(rng.integers(0, h)), int(rng.integers(0, w))
        img[y:y + h // 10, x:x + w // 10] = rng.integers(0, 256, (1, 1, channels))
    band = slice(h // 3, h // 3 + max(1, h // 20))
    img[band] = np.clip(img[band].astype(np.int32) + rng.integers(-20, 21, img[band].shape), 0,
                        255).astype(np.uint8)
    return img


A4_150DPI = (1754, 1240)  # rows, columns


def png_pages(n: int, seed: int, shape=A4_150DPI) -> list[bytes]:
    """n pages encoded by OpenCV's PNG writer with its default parameters
    (libpng adaptive filters, zlib), as a client would send them."""
    import cv2
    out = []
    for k in range(n):
        ok, enc = cv2.imencode(".png", page_like(shape[0], shape[1], seed + k))
        if not ok:
            raise RuntimeError("cv2.imencode failed")
        out.append(enc.tobytes())
    return out
