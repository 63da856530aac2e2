"""ORACLE-side input generation (test infrastructure and the bench's
reference arm only): numpy restatements of the seeded counter-based
generators that libtocr_synth.so runs on the device, so that the CPU
reference path can build the same synthetic workload without loading any
of this repository's native libraries.

Value i of stream s under seed k is mix64(k + golden * (mix64(s) + i + 1))
(splitmix64 finaliser). Config seeds are 0x7EC00000 + config index.
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


def _mix64_arr(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def mix64(z: int) -> int:
    z &= M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def hash3(seed: int, stream: int, i: int) -> int:
    return mix64(seed + GOLDEN * (mix64(stream) + i + 1))


def hash3_arr(seed: int, stream: int, i: np.ndarray) -> np.ndarray:
    base = np.uint64((mix64(stream) + 1) & M64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed & M64) + np.uint64(GOLDEN) * (base + i.astype(np.uint64))
    return _mix64_arr(z)


def unif(h: int) -> np.float32:
    return np.float32(h >> 40) * np.float32(1.0 / 16777216.0)


def unif_int(h: int, lo: int, hi: int) -> int:
    return lo + (h >> 32) % (hi - lo + 1)


# ---- config 5 pages -------------------------------------------------------------
def page_lines(H: int, W: int, seed: int, page: int):
    """Line layout of page `page` (page_lines_kernel): [(y0, y1, [(x0, x1), ...])]."""
    n_lines = unif_int(hash3(seed, 5000 + page, 0), 30, 80)
    pitch = np.float32(H) / np.float32(n_lines)
    out = []
    for line in range(n_lines):
        ls = (page << 8) + line
        ctr = 0
        hmax = min(14, int(pitch) - 3)
        gh = unif_int(hash3(seed, ls, ctr), 6, max(6, hmax)); ctr += 1
        yc = int(np.float32(np.float32(line) + np.float32(0.5)) * pitch)
        y0 = max(0, yc - gh // 2)
        y1 = min(H, y0 + gh)
        left = unif_int(hash3(seed, ls, ctr), 16, 160); ctr += 1
        length = unif_int(hash3(seed, ls, ctr), 120, max(120, W - 40 - left)); ctr += 1
        end = min(W - 8, left + length)
        x, glyphs = left, []
        while x < end and len(glyphs) < 512:
            nw = unif_int(hash3(seed, ls, ctr), 2, 8); ctr += 1
            g = 0
            while g < nw and x < end and len(glyphs) < 512:
                gw = unif_int(hash3(seed, ls, ctr), 4, 10); ctr += 1
                glyphs.append((x, min(end, x + gw)))
                x += gw + 2
                g += 1
            x += unif_int(hash3(seed, ls, ctr), 6, 12) - 2; ctr += 1
        out.append((y0, y1, glyphs))
    return out


def make_page(H: int = 960, W: int = 960, seed: int = 0x7EC00005, page: int = 0) -> np.ndarray:
    """u8 [H, W, 3]: white page with black glyph rectangles (tocr_synth_pages)."""
    img = np.full((H, W, 3), 255, np.uint8)
    for y0, y1, glyphs in page_lines(H, W, seed, page):
        for x0, x1 in glyphs:
            img[y0:y1, x0:x1] = 0
    return img


def ink_map(page: np.ndarray, gain: float = 12.0, radius: int = 7) -> np.ndarray:
    """fp32 [H, W] probability map of the synthetic run (ink_kernel): sigmoid of
    gain * (15-pixel horizontal max of the ink level - 0.5). Same formula as the
    device kernel; its exp is the fast hardware one, so values can differ in
    the last bits (this map feeds CPU timing, not parity)."""
    ink = 1.0 - page.astype(np.float32).sum(axis=2) * np.float32(1.0 / 765.0)
    H, W = ink.shape
    pad = np.zeros((H, W + 2 * radius), np.float32)
    pad[:, radius:radius + W] = ink
    m = pad[:, 0:W].copy()
    for d in range(1, 2 * radius + 1):
        np.maximum(m, pad[:, d:d + W], out=m)
    return (1.0 / (1.0 + np.exp(-np.float32(gain) * (m - np.float32(0.5))))).astype(np.float32)


# ---- config 5 stand-in recognition logits ----------------------------------------
def _noise_table(seed: int) -> np.ndarray:
    h = hash3_arr(seed, 9000, np.arange(1024, dtype=np.uint64))
    b = ((h[:, None] >> (np.arange(8, dtype=np.uint64) * np.uint64(8))[None, :]) & np.uint64(0xFF))
    return (b.astype(np.float32) * np.float32(8.0 / 256.0) - np.float32(4.0)).astype(np.float16)


def rec_logits(n_crops: int, T: int, V: int, seed: int = 0x7EC00005, first_crop: int = 0,
               dtype=np.float16) -> np.ndarray:
    """[n_crops, T, V] stand-in logits (rec_noise_kernel + rec_plant_kernel) for
    crops first_crop .. first_crop + n_crops - 1 of a micro-batch."""
    table = _noise_table(seed).view(np.complex128).reshape(1024)   # 16-byte chunks
    n_el = n_crops * T * V
    base = first_crop * T * V
    assert base % 8 == 0, "crop range must start on a 16-byte chunk"
    i = np.arange(base // 8, (base + n_el + 7) // 8, dtype=np.int64)
    chunks = np.take(table, (i * 7 + (i >> 10)) & 1023)
    flat = chunks.view(np.float16)[:n_el]
    if n_el % 8:
        flat = flat.copy()
        flat[n_el - n_el % 8:] = 0      # the device writes zeros after the last full chunk
    flat = flat.astype(dtype, copy=dtype != np.float16)
    out = flat.reshape(n_crops, T, V)
    for c in range(n_crops):
        cc = first_crop + c
        for tt in range(0, T, 3):
            th = hash3(seed, 7000 + cc, tt // 3)
            tok = 0 if (th & 1) else unif_int(th, 1, V - 1)
            out[c, tt:tt + 3, tok] = 8.0
    return out


# ---- config 1 DB maps ----------------------------------------------------------------
def db_map(H: int, W: int, kmin: int, kmax: int, seed: int, map_index: int) -> np.ndarray:
    """fp32 [H, W] (tocr_synth_db_map_host): background U[0, 0.1), k rotated
    rectangles filled with U[0.6, 1.0); pixel centres tested in double."""
    st = 3000 + map_index
    n = H * W
    bg = hash3_arr(seed, st + (1 << 40), np.arange(n, dtype=np.uint64))
    out = (np.float32(0.1) * ((bg >> np.uint64(40)).astype(np.float32)
                              * np.float32(1.0 / 16777216.0))).reshape(H, W)
    ctr = 0
    k = unif_int(hash3(seed, st, ctr), kmin, kmax); ctr += 1
    for r in range(k):
        w = 20.0 + 380.0 * float(unif(hash3(seed, st, ctr))); ctr += 1
        h = 8.0 + 52.0 * float(unif(hash3(seed, st, ctr))); ctr += 1
        th = (-15.0 + 30.0 * float(unif(hash3(seed, st, ctr)))) * 3.141592653589793 / 180.0; ctr += 1
        cx = W * float(unif(hash3(seed, st, ctr))); ctr += 1
        cy = H * float(unif(hash3(seed, st, ctr))); ctr += 1
        c, s = np.cos(th), np.sin(th)
        ex = 0.5 * (abs(w * c) + abs(h * s))
        ey = 0.5 * (abs(w * s) + abs(h * c))
        x0 = int(max(0.0, np.floor(cx - ex - 1))); x1 = int(min(W - 1.0, np.ceil(cx + ex + 1)))
        y0 = int(max(0.0, np.floor(cy - ey - 1))); y1 = int(min(H - 1.0, np.ceil(cy + ey + 1)))
        if x1 < x0 or y1 < y0:
            continue
        ys, xs = np.mgrid[y0:y1 + 1, x0:x1 + 1]
        dx = xs + 0.5 - cx
        dy = ys + 0.5 - cy
        u = dx * c + dy * s
        v = -dx * s + dy * c
        inside = (np.abs(u) <= 0.5 * w) & (np.abs(v) <= 0.5 * h)
        idx = (ys * W + xs)[inside].astype(np.uint64)
        fh = hash3_arr(seed, st + (2 << 40) + r, idx)
        vals = np.float32(0.6) + np.float32(0.4) * ((fh >> np.uint64(40)).astype(np.float32)
                                                    * np.float32(1.0 / 16777216.0))
        out[ys[inside], xs[inside]] = vals
    return out


# ---- config 2 CTC logits -------------------------------------------------------------
def ctc_plan(B: int, T: int, V: int, seed: int) -> np.ndarray:
    """[B, T] planted index per step or -1 (ctc_plan_kernel)."""
    plan = np.full((B, T), -1, np.int32)
    for b in range(B):
        st, ctr = 1000 + b, 0
        n_tok = unif_int(hash3(seed, st, ctr), 5, 40); ctr += 1
        tok, run, gap = [], [], []
        for _ in range(n_tok):
            tok.append(unif_int(hash3(seed, st, ctr), 1, V - 1)); ctr += 1
            run.append(unif_int(hash3(seed, st, ctr), 1, 4)); ctr += 1
            gap.append(unif_int(hash3(seed, st, ctr), 1, 3)); ctr += 1
        total = sum(run) + sum(gap)
        for k in range(n_tok):
            if total <= T:
                break
            total -= gap[k] - 1; gap[k] = 1
        for k in range(n_tok):
            if total <= T:
                break
            total -= run[k] - 1; run[k] = 1
        t = 0
        for k in range(n_tok):
            if t >= T:
                break
            for _ in range(gap[k]):
                if t < T:
                    plan[b, t] = 0; t += 1
            for _ in range(run[k]):
                if t < T:
                    plan[b, t] = tok[k]; t += 1
    return plan


def ctc_logits(B: int, T: int, V: int, seed: int, dtype=np.float32) -> np.ndarray:
    """[B, T, V] config-2 logits: N(0, 4^2) by Box-Muller on the counter
    stream (normal_f16_kernel; libm's log/sincos, so the last bits of a value
    can differ from the device's), planted index = row max + 2."""
    n = B * T * V
    i = np.arange((n + 1) // 2, dtype=np.uint64)
    h = hash3_arr(seed, 1, i)
    u1 = ((h >> np.uint64(40)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 16777216.0)
    u2 = ((h >> np.uint64(16)) & np.uint64(0xFFFFFF)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    r = np.sqrt(np.float32(-2.0) * np.log(u1)) * np.float32(4.0)
    ang = np.float32(2.0 * np.pi) * u2
    x = np.empty(2 * len(i), np.float32)
    x[0::2] = r * np.cos(ang)
    x[1::2] = r * np.sin(ang)
    x = x[:n].astype(np.float16).reshape(B, T, V)
    plan = ctc_plan(B, T, V, seed)
    rows = np.nonzero(plan >= 0)
    m = x[rows].astype(np.float32).max(axis=-1)
    x[rows[0], rows[1], plan[rows]] = (m + np.float32(2.0)).astype(np.float16)
    return x.astype(dtype)


# ---- config 3 images ------------------------------------------------------------------
def preprocess_dims(n: int, seed: int):
    return [(600 + (hash3(seed, 2000 + i, 0) >> 32) % 1401,
             600 + (hash3(seed, 2000 + i, 1) >> 32) % 1401) for i in range(n)]


def fill_u8(n: int, seed: int, stream: int) -> np.ndarray:
    """n uniform bytes (fill_u8_kernel): byte 8i+k is byte k of hash i."""
    h = hash3_arr(seed, stream, np.arange((n + 7) // 8, dtype=np.uint64))
    return h.astype("<u8").view(np.uint8)[:n].copy()
