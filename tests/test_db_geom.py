"""DB post-process geometry (subsystem 3) on the CPU: the routines of
turboocr_b200/csrc/db_geom.cuh, built for the host by tests/db_native.py,
against OpenCV (cv2, the library the reference calls in
src/detection/det_postprocess.cpp) and the reference's vendored Clipper.

Bit-exact bars: contour starts, border following, the contour order, area,
arc length, polygon mask and the raw Clipper offset. minAreaRect is
bit-exact as well: OpenCV 4.13 advances the caliper with the exact smallest
angle (not the rounded float cosine), which the restatement reproduces in
integer arithmetic. The one residue is a tie between two different
rectangles of exactly the same area on contours that repeat points: which
one wins depends on the hull's starting vertex, which OpenCV takes from an
unstable sort (about 1 in 10^4 noise contours, none on text-line contours)."""
import ctypes as C

import numpy as np
import pytest

cv2 = pytest.importorskip("cv2")
ndimage = pytest.importorskip("scipy.ndimage")

import db_native as dn  # noqa: E402
from oracle import db_oracle as do  # noqa: E402


def contour_starts(bm: np.ndarray):
    """Start pixels of every border OpenCV's RETR_LIST finds: the raster-first
    pixel of each 8-connected foreground component (outer border) and the
    pixel left of the raster-first pixel of each 4-connected background
    component that does not reach the image frame (hole border). Returned in
    the order cv2 lists the contours: descending raster order."""
    fg = bm > 0
    lab8, n8 = ndimage.label(fg, structure=np.ones((3, 3)))
    lab4, n4 = ndimage.label(np.pad(~fg, 1, constant_values=True))
    outer = lab4[0, 0]
    starts = []
    for lab in range(1, n8 + 1):
        ys, xs = np.nonzero(lab8 == lab)
        k = np.lexsort((xs, ys))[0]
        starts.append((int(ys[k]), int(xs[k]), False))
    for lab in range(1, n4 + 1):
        if lab == outer:
            continue
        ys, xs = np.nonzero(lab4 == lab)
        k = np.lexsort((xs, ys))[0]
        starts.append((int(ys[k]) - 1, int(xs[k]) - 2, True))
    return sorted(starts, key=lambda s: (s[0], s[1]), reverse=True)


def noise_bitmaps(n, seed, hmax=30):
    rng = np.random.default_rng(seed)
    for _ in range(n):
        H, W = rng.integers(3, hmax, 2)
        yield (rng.random((H, W)) < rng.uniform(0.2, 0.9)).astype(np.uint8) * 255


def synth_map(H, W, kmin, kmax, map_index):
    from turboocr_b200._lib import synth
    m = np.zeros((H, W), np.float32)
    synth().tocr_synth_db_map_host(m.ctypes.data, H, W, kmin, kmax, 0x7EC00001, map_index)
    return m


def test_contours_match_cv2_on_noise():
    """Start rule + border following + list order == cv2.findContours."""
    for bm in noise_bitmaps(400, 1):
        ref = [c.reshape(-1, 2).tolist() for c in
               cv2.findContours(bm.copy(), cv2.RETR_LIST, cv2.CHAIN_APPROX_SIMPLE)[0]]
        mine = [dn.trace(bm, x, y, hole).tolist() for y, x, hole in contour_starts(bm)]
        assert mine == ref
        bits = [dn.trace(bm, x, y, hole, bits=True).tolist() for y, x, hole in contour_starts(bm)]
        assert bits == ref


def test_contours_match_cv2_on_db_maps():
    m = synth_map(240, 320, 5, 20, 0)
    bm = do.threshold(m, 0.3)
    ref = [c.tolist() for c in do.find_contours(bm)]
    mine = [dn.trace(bm, x, y, hole).tolist() for y, x, hole in contour_starts(bm)]
    assert len(ref) > 3 and mine == ref
    bits = [dn.trace(bm, x, y, hole, bits=True).tolist() for y, x, hole in contour_starts(bm)]
    assert bits == ref


def test_bit_packed_trace_wide_noise():
    """Word boundaries of the bit-packed walk (widths above 32 columns)."""
    for bm in noise_bitmaps(60, 9, hmax=140):
        ref = [c.reshape(-1, 2).tolist() for c in
               cv2.findContours(bm.copy(), cv2.RETR_LIST, cv2.CHAIN_APPROX_SIMPLE)[0]]
        bits = [dn.trace(bm, x, y, hole, bits=True).tolist() for y, x, hole in contour_starts(bm)]
        assert bits == ref


def test_trace_single_pixel_and_frame():
    bm = np.zeros((5, 7), np.uint8)
    bm[2, 3] = 255
    assert dn.trace(bm, 3, 2, False).tolist() == [[3, 2]]
    full = np.full((4, 6), 255, np.uint8)   # touches every image edge
    ref = do.find_contours(full)[0].tolist()
    assert dn.trace(full, 0, 0, False).tolist() == ref


def test_area_arclen_mask_exact():
    n = 0
    for bm in noise_bitmaps(250, 2):
        for c in do.find_contours(bm):
            p = c.reshape(-1, 1, 2)
            assert dn.area(c) == cv2.contourArea(p)
            assert dn.arclen(c) == cv2.arcLength(p, True)
            x, y, w, h = cv2.boundingRect(p)
            ref = np.zeros((h, w), np.uint8)
            cv2.fillPoly(ref, [(c - [x, y]).reshape(-1, 1, 2).astype(np.int32)], 1)
            assert (dn.poly_mask(c, x, y, w, h) == ref).all()
            assert (dn.poly_mask(c, x, y, w, h, parity=True) == ref).all()
            n += 1
    assert n > 2000


def _clipper_raw(c, dist):
    L = do._clipper()
    L.clipper_ref_raw_offset.argtypes = [C.c_void_p, C.c_int, C.c_double, C.c_void_p, C.c_int]
    xy = np.ascontiguousarray(c, np.int32)
    out = np.zeros(1 << 17, np.int64)
    m = L.clipper_ref_raw_offset(xy.ctypes.data, len(xy), C.c_double(dist), out.ctypes.data,
                                 1 << 16)
    assert m >= 0
    return [tuple(q) for q in out[: 2 * m].reshape(m, 2).tolist()]


def test_raw_offset_matches_clipper():
    """Clipper's round-join offset before its union (DoOffset), vertex for
    vertex, at the unclip distance area * 1.5 / perimeter."""
    n = 0
    for bm in noise_bitmaps(250, 3):
        for c in do.find_contours(bm):
            per = cv2.arcLength(c.reshape(-1, 1, 2), True)
            if len(c) < 3 or per == 0:
                continue
            d = cv2.contourArea(c.reshape(-1, 1, 2)) * float(np.float32(1.5)) / per
            assert dn.offset_raw(c, d) == _clipper_raw(c, d)
            n += 1
    assert n > 1000


def test_min_area_rect_and_mini_box():
    total = bad = 0
    for bm in noise_bitmaps(500, 4):
        for c in do.find_contours(bm):
            r = cv2.minAreaRect(c)
            ref = np.array([r[0][0], r[0][1], r[1][0], r[1][1], r[2]], np.float32)
            got = dn.min_area_rect(c)
            total += 1
            if not (got == ref).all():
                # only a different rectangle of exactly the same area
                bad += 1
                assert abs(float(ref[2]) * float(ref[3]) - float(got[2]) * float(got[3])) <= \
                    1e-5 * float(ref[2]) * float(ref[3]), (c.tolist(), ref, got)
    assert total > 5000 and bad * 5000 <= total, (bad, total)
    # config-1 style maps: text-line contours and their raw offset rings
    n = 0
    for mi in range(4):
        m = synth_map(480, 640, 20, 40, mi)
        for c in do.find_contours(do.threshold(m, 0.3)):
            for pts in (c, np.array(dn.offset_raw(c, 4.5) or c.tolist(), np.int32)):
                assert dn.mini_box(pts) == do.get_mini_boxes(pts), c.tolist()
                n += 1
    assert n > 80


def test_column_table_hull_equals_sorted_hull():
    """The device's shared-memory hull (lowest and highest point of every x
    column with their first index, chain over those, optionally after
    dropping the points strictly inside the polygon of the extreme points of
    16 directions) returns the same
    vertices, orientation and starting vertex as the sorted monotone chain,
    including repeated points, vertical columns, collinear runs and
    degenerate sets."""
    rng = np.random.default_rng(21)
    sets = []
    for _ in range(3000):  # small ranges: many repeats and collinear points
        n = int(rng.integers(1, 60))
        r = int(rng.integers(1, 8))
        sets.append(rng.integers(-r, r + 1, (n, 2)))
    for _ in range(300):
        n = int(rng.integers(3, 400))
        sets.append(rng.integers(-2000, 2000, (n, 2)))
    sets += [[[5, 5]] * 4, [[1, 2], [1, 9], [1, 4]], [[0, 0], [3, 3], [6, 6], [3, 3]],
             [[0, 0], [0, 0], [1, 0], [1, 0]], [[7, -3]]]
    for mi in range(3):  # contours and offset rings of config-1 style maps
        m = synth_map(480, 640, 20, 60, mi)
        for c in do.find_contours(do.threshold(m, 0.3)):
            sets.append(c)
            if len(c) > 2:
                sets.append(np.array(dn.offset_raw(c, 9.5) or c.tolist(), np.int32))
    for p in sets:
        ref = dn.hull(p).tolist()
        assert dn.hull_table(p).tolist() == ref, np.asarray(p).tolist()
        assert dn.hull_table(p, interior_filter=True).tolist() == ref, np.asarray(p).tolist()
    wide = rng.integers(0, 5000, (500, 2))
    assert dn.hull_table(wide, col_cap=64) == -2


def test_parallel_offset_emission():
    """With k = j - 1 at every vertex (the device's one-thread-per-vertex
    emission), the ring equals Clipper's serial DoOffset whenever no joint
    before the last keeps k; otherwise the device emits serially. Contour
    joints turn by multiples of 45 degrees, so k is only kept for distances
    below 1/sin(45)."""
    same = serial = 0
    for mi in range(3):
        m = synth_map(480, 640, 20, 60, mi)
        for c in do.find_contours(do.threshold(m, 0.3)):
            if len(c) < 3:
                continue
            for d in (0.7, 3.0, 9.5, 40.0):
                par = dn.offset_parallel(c, d)
                if par is None:
                    assert d < 1.42
                    serial += 1
                else:
                    assert par == dn.offset_raw(c, d)
                    same += 1
    assert same > 100 and serial > 10, (same, serial)


def test_cta_offset_prepare_rule():
    """The CTA's path preparation (keep a point iff it differs from its
    predecessor, orientation from the int64 shoelace sum) equals Clipper's
    sequential AddPath + FixOrientations restatement, including repeated
    points, closing repeats and both orientations."""
    rng = np.random.default_rng(5)
    sets = []
    for bm in noise_bitmaps(300, 9):
        sets += [c for c in do.find_contours(bm)]
    for _ in range(2000):
        n = int(rng.integers(1, 40))
        pts = rng.integers(-3, 4, (n, 2))
        if rng.random() < 0.3 and n > 1:
            pts[-1] = pts[0]            # closing repeat
        sets.append(pts)
    same = 0
    for p in sets:
        assert dn.offset_prepare(p, rule=True) == dn.offset_prepare(p), np.asarray(p).tolist()
        same += 1
    assert same > 3000


# ---- property tests of the CTA geometry path (hypothesis) -------------------
from hypothesis import given, settings, strategies as st  # noqa: E402

_coord = st.integers(min_value=-300000, max_value=300000)
_small = st.integers(min_value=-6, max_value=6)


@settings(max_examples=300, deadline=None)
@given(st.lists(st.tuples(_coord, _coord), min_size=1, max_size=80)
       | st.lists(st.tuples(_small, _small), min_size=1, max_size=60))
def test_property_column_hull(pts):
    """Column-table hull, with and without the interior filter, equals the
    sorted monotone chain on arbitrary point sets (wide coordinates or
    heavy repetition)."""
    p = np.array(pts, np.int32)
    ref = dn.hull(p).tolist()
    assert dn.hull_table(p).tolist() == ref
    assert dn.hull_table(p, interior_filter=True).tolist() == ref


@settings(max_examples=300, deadline=None)
@given(st.lists(st.tuples(_small, _small), min_size=1, max_size=50))
def test_property_offset_prepare_rule(pts):
    p = np.array(pts, np.int32)
    assert dn.offset_prepare(p, rule=True) == dn.offset_prepare(p)


@settings(max_examples=200, deadline=None)
@given(st.lists(st.tuples(st.integers(0, 60), st.integers(0, 60)), min_size=3, max_size=40),
       st.floats(min_value=0.5, max_value=60.0))
def test_property_parallel_offset(pts, d):
    """Per-vertex emission equals the serial offset whenever no joint before
    the last keeps Clipper's previous vertex (the device then uses it)."""
    p = np.array(pts, np.int32)
    par = dn.offset_parallel(p, d)
    if par is not None:
        assert par == dn.offset_raw(p, d)
