"""Host side of the PNG decode (no GPU): the oracle pinned against the
reference's own decode, the synthetic-file generator, the IHDR peek and the
size caps, and the reference's PNG guard tests (tests/decode/test_png_guards.cpp)
restated against tocr_png_peek."""
import struct
import zlib

import numpy as np
import pytest

import pngsynth as ps
from oracle import png_oracle as po
from turboocr_b200 import decode as D


def _forge(png: bytes, w: int, h: int) -> bytes:
    """Rewrites the IHDR dimensions and re-seals its CRC (test_png_guards.cpp:45-50)."""
    b = bytearray(png)
    b[16:20] = struct.pack(">I", w)
    b[20:24] = struct.pack(">I", h)
    b[29:33] = struct.pack(">I", zlib.crc32(bytes(b[12:29])) & 0xFFFFFFFF)
    return bytes(b)


def test_expected_model_is_the_reference_decode():
    for name, b, exp in ps.valid_cases():
        got = po.reference_decode(b)
        assert got is not None, name
        assert got.shape == exp.shape and np.array_equal(got, exp), name


def test_damaged_files_are_rejected_by_the_reference():
    for name, b in ps.invalid_cases():
        assert po.reference_decode(b) is None, name


def test_generator_round_trips_through_opencv():
    cv2 = pytest.importorskip("cv2")
    rng = np.random.default_rng(3)
    img = rng.integers(0, 256, (40, 50, 3), dtype=np.uint8)
    for il in (0, 1):
        b = ps.encode(img, 2, 8, interlace=il)
        assert np.array_equal(cv2.imdecode(np.frombuffer(b, np.uint8), cv2.IMREAD_COLOR),
                              img[..., ::-1])


def test_peek_sizes_match_the_scanline_stream():
    rng = np.random.default_rng(1)
    for name, b, exp in ps.valid_cases()[::5]:
        info = D.peek(b)
        assert info is not None, name
        assert (info.height, info.width) == exp.shape[:2]
        depth, ct, il = b[24], b[25], b[28]
        h, w = exp.shape[:2]
        img = np.zeros((h, w, ps.CHANNELS[ct]), np.uint16 if depth == 16 else np.uint8)
        assert info.raw_bytes == len(ps.raw_stream(img, ct, depth, 0, rng, il)), name
        assert info.scratch_bytes >= 64 + info.raw_bytes + len(b) + 16


def test_peek_rejects_what_the_reference_rejects(monkeypatch):
    good = ps.encode(np.zeros((8, 8, 3), np.uint8), 2, 8)
    assert D.peek(good) is not None
    assert D.peek(good[:20]) is None
    assert D.peek(b"") is None
    assert D.peek(b"\xff\xd8\xff\xe0" + bytes(40)) is None
    # test_png_guards.cpp:86-115: absurd, one huge side, zero.
    for w, h in ((0x40000000, 0x40000000), (1 << 20, 8), (0, 8), (8, 0)):
        forged = _forge(good, w, h)
        assert D.peek(forged) is None
        assert po.reference_decode(forged) is None
    sixteen = ps.encode(np.ones((8, 8), np.uint16), 0, 16)
    assert sixteen[24] == 16
    for w, h in ((0x40000000, 0x40000000), (1 << 20, 8), (0, 8)):
        assert D.peek(_forge(sixteen, w, h)) is None
        assert po.reference_decode(_forge(sixteen, w, h)) is None
    # The caps follow the reference's environment knobs (image_config.h).
    img = ps.encode(np.zeros((100, 120), np.uint8), 0, 8)
    monkeypatch.setenv("MAX_IMAGE_DIM", "110")
    assert D.max_image_dim() == 110 and D.peek(img) is None and po.reference_decode(img) is None
    monkeypatch.setenv("MAX_IMAGE_DIM", "7")  # clamped to 64
    assert D.max_image_dim() == 64
    monkeypatch.setenv("MAX_IMAGE_DIM", "junk")
    assert D.max_image_dim() == 16384
    monkeypatch.delenv("MAX_IMAGE_DIM")
    monkeypatch.setenv("MAX_IMAGE_PIXELS_MP", "0")  # clamped to 1 MP
    assert D.max_image_pixels() == 1000000
    wide = _forge(img, 1001, 1000)
    assert D.peek(wide) is None and po.reference_decode(wide) is None
    assert D.peek(_forge(img, 1000, 1000)) is not None


def test_sixteen_bit_files_take_the_opencv_route():
    """test_png_guards.cpp:70-81: a 16-bit file decodes to 8-bit BGR."""
    img = np.full((12, 17), 40000, np.uint16)
    b = ps.encode(img, 0, 16)
    out = po.reference_decode(b)
    assert out.shape == (12, 17, 3) and out.dtype == np.uint8
    assert np.all(out == 40000 >> 8)


def test_plan_lays_out_aligned_buffers():
    files = [ps.encode(np.zeros((h, w, 3), np.uint8), 2, 8) for h, w in ((3, 5), (7, 11), (1, 1))]
    jobs, ok, nsrc, nscr, ndst = D.PngBatchDecoder("cpu").plan(files + [b"junk"])
    assert ok == [0, 1, 2]
    assert all(int(j["scratch_off"]) % 16 == 0 for j in jobs[ok])
    assert all(int(j["dst_pitch"]) % 16 == 0 and int(j["dst_pitch"]) >= 3 * int(j["width"])
               for j in jobs[ok])
    assert nsrc == sum(len(f) for f in files)
