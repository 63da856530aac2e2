"""Device PNG decode (csrc/png.cu via turboocr_b200.decode) against the
reference's own decode (oracle/png_oracle.py: the reference's vendored Wuffs
compiled in place, and its OpenCV route for 16-bit files): byte-exact BGR
for every file the reference decodes, a failure status for every file it
rejects, all in one mixed batch."""
import zlib

import numpy as np
import pytest

import pngsynth as ps
from oracle import png_oracle as po
from turboocr_b200 import decode as D

pytestmark = pytest.mark.gpu


def _check_batch(cuda, files, expected):
    dec = D.PngBatchDecoder(cuda)
    out = dec.decode(files)
    bad = []
    for (name, exp), img, st in zip(expected, out.images, out.status):
        if exp is None:
            if st == D.PNG_OK:
                bad.append(f"{name}: decoded, the reference rejects it")
            continue
        if st != D.PNG_OK:
            bad.append(f"{name}: status {st} ({D.STATUS_NAMES.get(st)})")
            continue
        got = img.cpu().numpy()
        if got.shape != exp.shape or not np.array_equal(got, exp):
            diff = np.argwhere(got != exp)[:3].tolist() if got.shape == exp.shape else got.shape
            bad.append(f"{name}: pixels differ {diff}")
    assert not bad, "\n".join(bad)
    return out


def test_every_format_filter_and_stream_layout(cuda):
    cases = ps.valid_cases()
    files = [b for _, b, _ in cases]
    for (name, b, exp) in cases:  # the expected model is the reference's output
        ref = po.reference_decode(b)
        assert ref is not None and np.array_equal(ref, exp), name
    _check_batch(cuda, files, [(n, e) for n, _, e in cases])


def test_rejected_files_fail_and_do_not_disturb_their_neighbours(cuda):
    valid = ps.valid_cases(seed=11)[::9]
    invalid = ps.invalid_cases()
    for name, b in invalid:
        assert po.reference_decode(b) is None, name
    mixed = []
    for i, (name, b) in enumerate(invalid):
        mixed.append((name, b, None))
        v = valid[i % len(valid)]
        mixed.append((v[0] + f"#{i}", v[1], v[2]))
    out = _check_batch(cuda, [b for _, b, _ in mixed], [(n, e) for n, _, e in mixed])
    assert sum(s != D.PNG_OK for s in out.status) == len(invalid)


def test_opencv_encoded_pages_at_full_size(cuda):
    cv2 = pytest.importorskip("cv2")
    files, exp = [], []
    for k, (h, w) in enumerate([(1754, 1240), (2200, 1700), (1123, 794)]):
        page = ps.page_like(h, w, 100 + k)
        for lvl in (1, 3, 9):
            ok, enc = cv2.imencode(".png", page, [cv2.IMWRITE_PNG_COMPRESSION, lvl])
            assert ok
            b = enc.tobytes()
            files.append(b)
            exp.append((f"page{k}_z{lvl}", po.reference_decode(b)))
    _check_batch(cuda, files, exp)


def test_batch_of_64_pages_checksums(cuda):
    rng = np.random.default_rng(5)
    files, exp = [], []
    for k in range(64):
        h, w = int(rng.integers(600, 1400)), int(rng.integers(500, 1100))
        ct = int(rng.choice([0, 2, 6]))
        page = ps.page_like(h, w, 1000 + k, channels=ps.CHANNELS[ct])
        if ct == 6:
            page[..., 3] = rng.integers(0, 256, (h, w), dtype=np.uint8)
        if ct == 0:
            page = page[..., 0]
        b = ps.encode(page, ct, 8, filters="random", seed=k,
                      strategy=int(rng.choice([zlib.Z_DEFAULT_STRATEGY, zlib.Z_RLE, zlib.Z_FIXED])),
                      idat_size=int(rng.choice([8192, 65536, 1 << 30])))
        files.append(b)
        exp.append((f"p{k}", po.reference_decode(b)))
    _check_batch(cuda, files, exp)


def test_batch_with_several_files_per_sm(cuda):
    """448 files in one call: three or more inflate CTAs resident per SM
    (the bench's batch shape), every image byte-exact with the reference."""
    rng = np.random.default_rng(8)
    files, exp = [], []
    for k in range(448):
        h, w = int(rng.integers(40, 160)), int(rng.integers(40, 200))
        ct = int(rng.choice([0, 2, 6]))
        page = ps.page_like(h, w, 5000 + k, channels=ps.CHANNELS[ct])
        if ct == 0:
            page = page[..., 0]
        b = ps.encode(page, ct, 8, filters="random", seed=k,
                      strategy=int(rng.choice([zlib.Z_DEFAULT_STRATEGY, zlib.Z_RLE, zlib.Z_FIXED])))
        files.append(b)
        exp.append((f"s{k}", po.reference_decode(b)))
    _check_batch(cuda, files, exp)


def test_size_caps_reject_on_the_host(cuda, monkeypatch):
    big = ps.encode(np.zeros((70, 90, 3), np.uint8), 2, 8)
    monkeypatch.setenv("MAX_IMAGE_DIM", "80")
    assert po.reference_decode(big) is None
    out = D.PngBatchDecoder(cuda).decode([big])
    assert out.status == [-1] and out.images == [None]
    monkeypatch.setenv("MAX_IMAGE_DIM", "16384")
    monkeypatch.setenv("MAX_IMAGE_PIXELS_MP", "1")
    huge = ps.encode(np.zeros((1001, 1000), np.uint8), 0, 8, filters=0)
    assert po.reference_decode(huge) is None
    assert D.PngBatchDecoder(cuda).decode([huge]).status == [-1]
