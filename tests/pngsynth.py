"""Seeded synthetic PNG files for the decode tests: a small PNG writer on the
standard library's zlib (RFC 2083 chunk layout, RFC 1950/1951 streams), so
the tests control what cv2.imencode cannot: every colour type and bit depth,
per-row filter choice, Adam7 interlacing, palettes with tRNS, IDAT split
sizes, zlib strategies (fixed-Huffman, Huffman-only, RLE, stored blocks) and
deliberately damaged files."""
from __future__ import annotations

import struct
import zlib

import numpy as np

from turboocr_b200.pagegen import page_like  # noqa: F401  (re-exported for the tests)

SIG = b"\x89PNG\r\n\x1a\n"
CHANNELS = {0: 1, 2: 3, 3: 1, 4: 2, 6: 4}
ADAM7 = [(0, 0, 8, 8), (4, 0, 8, 8), (0, 4, 4, 8), (2, 0, 4, 4), (0, 2, 2, 4), (1, 0, 2, 2),
         (0, 1, 1, 2)]  # (x0, y0, dx, dy)


def chunk(kind: bytes, data: bytes) -> bytes:
    return struct.pack(">I", len(data)) + kind + data + struct.pack(
        ">I", zlib.crc32(kind + data) & 0xFFFFFFFF)


def _pack_row(samples: np.ndarray, depth: int) -> bytes:
    """samples: 1-D array of channel samples of one row."""
    if depth == 16:
        return samples.astype(">u2").tobytes()
    if depth == 8:
        return samples.astype(np.uint8).tobytes()
    per = 8 // depth
    n = len(samples)
    out = bytearray((n + per - 1) // per)
    for i, v in enumerate(samples.astype(np.int64)):
        out[i // per] |= (int(v) & ((1 << depth) - 1)) << (8 - depth * (i % per + 1))
    return bytes(out)


def _paeth(a, b, c):
    p = a + b - c
    pa, pb, pc = abs(p - a), abs(p - b), abs(p - c)
    if pa <= pb and pa <= pc:
        return a
    return b if pb <= pc else c


def _filter_row(kind: int, row: bytes, prev: bytes, bpp: int) -> bytes:
    out = bytearray(len(row))
    for i, x in enumerate(row):
        a = row[i - bpp] if i >= bpp else 0
        b = prev[i] if prev else 0
        c = prev[i - bpp] if prev and i >= bpp else 0
        pred = (0, a, b, (a + b) >> 1, _paeth(a, b, c))[kind]
        out[i] = (x - pred) & 0xFF
    return bytes(out)


def _filter_rows_np(kind: int, row: np.ndarray, prev: np.ndarray, bpp: int) -> np.ndarray:
    """Vectorised filters 0-3 (Paeth goes through _filter_row)."""
    r = row.astype(np.int32)
    if len(r) > bpp:
        a = np.concatenate([np.zeros(bpp, np.int32), r[:-bpp]])
    else:
        a = np.zeros_like(r)
    b = prev.astype(np.int32) if prev is not None else np.zeros_like(r)
    pred = [np.zeros_like(r), a, b, (a + b) >> 1][kind]
    return ((r - pred) & 0xFF).astype(np.uint8)


def raw_stream(img: np.ndarray, color_type: int, depth: int, filters, rng, interlace: int) -> bytes:
    """The filtered scanline stream (what the zlib stream inflates to)."""
    h, w = img.shape[:2]
    ch = CHANNELS[color_type]
    bpp = max(1, ch * depth // 8)
    flat = img.reshape(h, w, ch)
    passes = [(0, 0, 1, 1)] if interlace == 0 else ADAM7
    out = bytearray()
    for x0, y0, dx, dy in passes:
        sub = flat[y0::dy, x0::dx]
        if sub.shape[0] == 0 or sub.shape[1] == 0:
            continue
        prev = None
        for y in range(sub.shape[0]):
            row = _pack_row(sub[y].reshape(-1), depth)
            if isinstance(filters, str):
                kind = int(rng.integers(0, 5))
            elif isinstance(filters, (list, tuple)):
                kind = filters[y % len(filters)]
            else:
                kind = int(filters)
            if kind == 4:
                f = _filter_row(4, row, prev, bpp)
            else:
                f = _filter_rows_np(kind, np.frombuffer(row, np.uint8),
                                    None if prev is None else np.frombuffer(prev, np.uint8),
                                    bpp).tobytes()
            out.append(kind)
            out += f
            prev = row
    return bytes(out)


def zlib_stream(raw: bytes, level: int = 6, strategy: int = zlib.Z_DEFAULT_STRATEGY,
                flush_every: int = 0) -> bytes:
    co = zlib.compressobj(level, zlib.DEFLATED, 15, 9, strategy)
    if not flush_every:
        return co.compress(raw) + co.flush()
    out = bytearray()
    for i in range(0, len(raw), flush_every):
        out += co.compress(raw[i:i + flush_every])
        out += co.flush(zlib.Z_FULL_FLUSH)
    return bytes(out) + co.flush()


def encode(img: np.ndarray, color_type: int, depth: int = 8, *, filters="random", seed: int = 0,
           level: int = 6, strategy: int = zlib.Z_DEFAULT_STRATEGY, interlace: int = 0,
           palette: np.ndarray | None = None, trns: bytes | None = None, idat_size: int = 8192,
           flush_every: int = 0, extra_chunks: list[tuple[bytes, bytes]] | None = None) -> bytes:
    """img: (h, w) or (h, w, channels) samples for the colour type (palette
    indices for colour type 3; 16-bit samples as uint16)."""
    rng = np.random.default_rng(seed)
    h, w = img.shape[:2]
    ihdr = struct.pack(">IIBBBBB", w, h, depth, color_type, 0, 0, interlace)
    z = zlib_stream(raw_stream(img, color_type, depth, filters, rng, interlace), level, strategy,
                    flush_every)
    body = chunk(b"IHDR", ihdr)
    for kind, data in extra_chunks or []:
        body += chunk(kind, data)
    if palette is not None:
        body += chunk(b"PLTE", np.asarray(palette, np.uint8).reshape(-1).tobytes())
    if trns is not None:
        body += chunk(b"tRNS", trns)
    for i in range(0, max(len(z), 1), idat_size):
        body += chunk(b"IDAT", z[i:i + idat_size])
    return SIG + body + chunk(b"IEND", b"")


def premul(c, a):
    """Wuffs' 8-bit premultiplication (colour and alpha widened by 0x101)."""
    c = np.asarray(c, np.uint64)
    a = np.asarray(a, np.uint64)
    return ((c * (a * 0x10201)) // 0xFFFF >> 8).astype(np.uint8)


def expected_bgr(img: np.ndarray, color_type: int, depth: int, palette=None,
                 trns: bytes | None = None) -> np.ndarray:
    """What the reference's decode makes of the samples: Wuffs' BGR for 1-8
    bit files (grey scaled to 8 bits, tRNS keys black, alpha premultiplied,
    palette indices past the PLTE black), OpenCV's for 16 bit (high byte,
    alpha dropped)."""
    h, w = img.shape[:2]
    x = img.reshape(h, w, -1).astype(np.uint32)
    if depth == 16:
        hi = (x >> 8).astype(np.uint8)
        if color_type in (0, 4):
            return np.repeat(hi[..., :1], 3, axis=2)
        return hi[..., 2::-1][..., :3].copy()
    if color_type == 3:
        pal = np.zeros((256, 3), np.uint8)
        n = 0 if palette is None else len(palette)
        for i in range(n):
            a = trns[i] if trns is not None and i < len(trns) else 255
            r, g, b = (int(v) for v in palette[i])
            pal[i] = [premul(b, a), premul(g, a), premul(r, a)]
        return pal[x[..., 0]]
    mask = (1 << depth) - 1
    if color_type == 0:
        g = (x[..., 0] * (255 // mask)).astype(np.uint8)
        if trns is not None:
            key = struct.unpack(">H", trns)[0] & mask
            g[x[..., 0] == key] = 0
        return np.repeat(g[..., None], 3, axis=2)
    if color_type == 2:
        out = x[..., ::-1].astype(np.uint8).copy()
        if trns is not None:
            k = np.array(struct.unpack(">HHH", trns), np.uint32) & 0xFF
            out[np.all(x == k, axis=2)] = 0
        return out
    if color_type == 4:
        g = premul(x[..., 0], x[..., 1])
        return np.repeat(g[..., None], 3, axis=2)
    a = x[..., 3]
    return np.stack([premul(x[..., 2], a), premul(x[..., 1], a), premul(x[..., 0], a)], axis=2)


def _samples(rng, h, w, ct, depth):
    ch = CHANNELS[ct]
    hi = (1 << depth) - 1
    if depth == 16:
        return rng.integers(0, 65536, (h, w, ch), dtype=np.uint16).squeeze(-1) if ch == 1 else \
            rng.integers(0, 65536, (h, w, ch), dtype=np.uint16)
    a = rng.integers(0, hi + 1, (h, w, ch), dtype=np.uint16).astype(np.uint8)
    return a[..., 0] if ch == 1 else a


def valid_cases(seed: int = 7):
    """(name, png bytes, expected BGR) for files the reference decodes."""
    rng = np.random.default_rng(seed)
    out = []
    combos = [(0, 1), (0, 2), (0, 4), (0, 8), (0, 16), (2, 8), (2, 16), (3, 1), (3, 2), (3, 4),
              (3, 8), (4, 8), (4, 16), (6, 8), (6, 16)]
    for ct, d in combos:
        for il in (0, 1):
            for (h, w) in ((1, 1), (3, 5), (29, 37), (64, 48)):
                img = _samples(rng, h, w, ct, d)
                pal = trns = None
                if ct == 3:
                    n = int(rng.integers(1, 1 << d)) if d < 8 else 200
                    pal = rng.integers(0, 256, (n, 3), dtype=np.uint8)
                    if rng.random() < 0.6:
                        trns = rng.integers(0, 256, int(rng.integers(0, n + 1)), dtype=np.uint8).tobytes()
                elif ct == 0 and d <= 8 and rng.random() < 0.5:
                    trns = struct.pack(">H", int(img.flat[0]) | (0x100 if d == 8 else 0))
                elif ct == 2 and d == 8 and rng.random() < 0.5:
                    img[h // 2] = img[0]
                    trns = struct.pack(">HHH", *[int(v) for v in img[0, 0]])
                b = encode(img, ct, d, interlace=il, palette=pal, trns=trns, seed=int(rng.integers(1 << 30)),
                           idat_size=int(rng.choice([1, 7, 64, 8192])))
                out.append((f"ct{ct}_d{d}_il{il}_{h}x{w}", b, expected_bgr(img, ct, d, pal, trns)))
    img = rng.integers(0, 256, (33, 17, 3), dtype=np.uint8)
    for f in range(5):
        out.append((f"filter{f}", encode(img, 2, 8, filters=f), expected_bgr(img, 2, 8)))
    page = page_like(300, 260, seed)
    for name, lvl, strat, fe in (("stored", 0, zlib.Z_DEFAULT_STRATEGY, 0),
                                 ("fixed", 6, zlib.Z_FIXED, 0),
                                 ("huffman_only", 6, zlib.Z_HUFFMAN_ONLY, 0),
                                 ("rle", 6, zlib.Z_RLE, 0), ("level1", 1, 0, 0), ("level9", 9, 0, 0),
                                 ("full_flush", 6, 0, 5000), ("stored_flush", 0, 0, 3000)):
        out.append((f"page_{name}", encode(page, 2, 8, level=lvl, strategy=strat, flush_every=fe),
                    expected_bgr(page, 2, 8)))
    solid = np.full((200, 180, 3), 247, np.uint8)
    out.append(("solid_none", encode(solid, 2, 8, filters=0), expected_bgr(solid, 2, 8)))
    wide = np.tile(rng.integers(0, 256, (1, 10700, 3), dtype=np.uint8), (4, 1, 1))
    out.append(("far_distance", encode(wide, 2, 8, filters=0, level=9), expected_bgr(wide, 2, 8)))
    gray = page_like(257, 190, seed + 1, channels=1)[..., 0]
    out.append(("page_gray", encode(gray, 0, 8), expected_bgr(gray, 0, 8)))
    return out


def _with_ihdr(w, h, d, ct, il, tail: bytes) -> bytes:
    return SIG + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, d, ct, 0, 0, il)) + tail


def invalid_cases(seed: int = 9):
    """(name, bytes) for files the reference rejects."""
    rng = np.random.default_rng(seed)
    img = rng.integers(0, 256, (6, 7, 3), dtype=np.uint8)
    raw = raw_stream(img, 2, 8, 0, rng, 0)
    z = zlib_stream(raw)
    def idat(zz):
        return _with_ihdr(7, 6, 8, 2, 0, chunk(b"IDAT", zz) + chunk(b"IEND", b""))
    good = idat(z)
    out = []
    b = bytearray(good); i = b.find(b"IDAT"); n = struct.unpack(">I", b[i - 4:i])[0]; b[i + 4 + n] ^= 1
    out.append(("idat_crc", bytes(b)))
    b = bytearray(good); b[29] ^= 1
    out.append(("ihdr_crc", bytes(b)))
    out.append(("extra_raw", idat(zlib_stream(raw + bytes(50)))))
    out.append(("short_raw", idat(zlib_stream(raw[:-5]))))
    out.append(("trailing_garbage", idat(z + b"garbage")))
    out.append(("no_adler", idat(z[:-4])))
    out.append(("truncated_stream", idat(z[:-10])))
    out.append(("chunk_between_idats", _with_ihdr(7, 6, 8, 2, 0, chunk(b"IDAT", z[:5]) +
                                                  chunk(b"tEXt", b"a\x00b") + chunk(b"IDAT", z[5:]) +
                                                  chunk(b"IEND", b""))))
    r5 = bytearray(raw); r5[0] = 5
    out.append(("filter5", idat(zlib_stream(bytes(r5)))))
    pi = np.array([[0, 1, 2, 3, 4, 255]], np.uint8)
    out.append(("no_plte", encode(pi, 3, 8)))
    out.append(("rgb_trns_len", encode(img, 2, 8, trns=b"\x00\x01")))
    out.append(("plte_len4", _with_ihdr(6, 1, 8, 3, 0, chunk(b"PLTE", b"\x01\x02\x03\x04") +
                                        chunk(b"IDAT", zlib_stream(b"\x00" + bytes(6))) +
                                        chunk(b"IEND", b""))))
    zz = bytearray(z); zz[0] = 0x78; zz[1] = 0x9C ^ 1
    out.append(("fcheck", idat(bytes(zz))))
    zz = bytearray(z); zz[0] = 0x88; zz[1] = (31 - (0x88 * 256) % 31) % 31
    out.append(("cinfo8", idat(bytes(zz))))
    zz = bytearray(z); zz[1] = (zz[1] & 0xC0) | 0x20; zz[1] |= (31 - ((zz[0] << 8) | zz[1]) % 31) % 31
    out.append(("fdict", idat(bytes(zz))))
    out.append(("gray_plte", encode(img[..., 0], 0, 8, palette=np.zeros((2, 3), np.uint8))))
    out.append(("unknown_critical", encode(img, 2, 8, extra_chunks=[(b"ABCD", b"xyz")])))
    out.append(("bad_ihdr_len", SIG + chunk(b"IHDR", struct.pack(">IIBBBBB", 4, 5, 8, 6, 0, 0, 0) +
                                            b"\x00") + chunk(b"IEND", b"")))
    out.append(("trns_before_plte", _with_ihdr(2, 1, 8, 3, 0, chunk(b"tRNS", b"\x80") +
                                               chunk(b"PLTE", b"\x01\x02\x03") +
                                               chunk(b"IDAT", zlib_stream(b"\x00\x00\x00")) +
                                               chunk(b"IEND", b""))))
    out.append(("filter_method1", SIG + chunk(b"IHDR", struct.pack(">IIBBBBB", 2, 1, 8, 2, 0, 1, 0)) +
                chunk(b"IDAT", zlib_stream(b"\x00" + bytes(6))) + chunk(b"IEND", b"")))
    out.append(("bad_depth", SIG + chunk(b"IHDR", struct.pack(">IIBBBBB", 2, 1, 4, 2, 0, 0, 0)) +
                chunk(b"IEND", b"")))
    out.append(("sig_only", SIG))
    out.append(("not_png", b"GIF89a" + bytes(40)))
    out.append(("empty", b""))
    # DEFLATE-level damage: a block type of 3, a distance before the start.
    zz = bytearray(z); zz[2] = (zz[2] & ~0x06) | 0x06
    out.append(("btype3", idat(bytes(zz))))
    bad = bytearray(b"\x78\x01")  # fixed block: one match of length 3 at distance 1 first
    bits = [1, 1, 0]  # BFINAL=1, BTYPE=01 (LSB first)
    code257 = [0, 0, 0, 0, 0, 0, 1]  # 7-bit code 0000001 (symbol 257), sent MSB first
    bits += code257 + [0, 0, 0, 0, 0] + [0] * 7  # distance code 0 (5 bits); then EOB (0000000)
    v = 0
    for k, bit in enumerate(bits):
        v |= bit << k
    nb = (len(bits) + 7) // 8
    bad += v.to_bytes(nb, "little") + b"\x00\x00\x00\x00"
    out.append(("distance_before_start", _with_ihdr(1, 1, 8, 0, 0, chunk(b"IDAT", bytes(bad)) +
                                                    chunk(b"IEND", b""))))
    return out
