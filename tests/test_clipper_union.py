"""Clipper's union step of unclip (clipper_union.cuh, host build) against the
reference's own Clipper 6.4.2 (oracle/_ref/libclipper_ref.so, driven as
det_postprocess.cpp:57-102 drives it): the kept ring must be identical point
for point and in order, so every box built from it is bit-exact. Also pins
the restated libstdc++ std::sort, whose order of equal keys Clipper's output
depends on, against the host's std::sort."""
import numpy as np
import pytest

import db_native as dn
from oracle import db_oracle as do
from oracle import synth_host as sh

cv2 = pytest.importorskip("cv2")


def same_ring(c, ratio):
    d = do.unclip_distance(c, ratio)
    if d is None:
        return True
    ref = np.asarray(do.unclip(c, ratio)).reshape(-1, 2)
    got = dn.unclip_union(c, d)
    if len(got) == 0:
        got = c.reshape(-1, 2)
    return np.array_equal(ref, got.reshape(-1, 2))


def test_std_sort_matches_libstdcxx():
    rng = np.random.default_rng(0)
    for n in list(range(0, 40)) + [63, 64, 65, 100, 257, 1000, 4096]:
        for span in (1, 3, 10, 1 << 20):
            keys = rng.integers(0, span, n)
            a, b = dn.sort_check(keys)
            assert np.array_equal(a, b), (n, span)
    for keys in (np.zeros(500), np.arange(500), np.arange(500)[::-1], np.tile([3, 1, 2], 300)):
        a, b = dn.sort_check(keys)
        assert np.array_equal(a, b)


def test_union_config1_maps():
    n = 0
    for mi in (0, 5):
        pred = sh.db_map(960, 960, 40, 200, 0x7EC00000, mi)
        for c in do.find_contours(do.threshold(pred, 0.3)):
            if len(c) > 2:
                assert same_ring(c, 1.5), (mi, len(c))
                n += 1
    assert n > 20


def test_union_noise_contours():
    rng = np.random.default_rng(1)
    n = 0
    for _ in range(60):
        h, w = rng.integers(8, 48, 2)
        bm = (rng.random((h, w)) < rng.uniform(0.3, 0.7)).astype(np.uint8) * 255
        for c in do.find_contours(bm):
            if len(c) > 2:
                for ratio in (1.5, float(rng.uniform(0.3, 3.0))):
                    assert same_ring(c, ratio)
                    n += 1
    assert n > 1000


def test_union_rotated_shapes_and_blobs():
    rng = np.random.default_rng(2)
    for _ in range(40):
        bm = np.zeros((200, 200), np.uint8)
        cx, cy = rng.uniform(60, 140, 2)
        a = rng.uniform(-90, 90)
        size = (rng.uniform(5, 150), rng.uniform(3, 60))
        if rng.random() < 0.5:
            cv2.fillPoly(bm, [cv2.boxPoints(((cx, cy), size, a)).astype(np.int32)], 255)
        else:
            cv2.ellipse(bm, ((cx, cy), size, a), 255, -1)
        for c in do.find_contours(bm):
            if len(c) > 2:
                assert same_ring(c, 1.5)
    for _ in range(3):   # large blobs with many concavities (rings of thousands of points)
        f = cv2.GaussianBlur(rng.random((300, 400)).astype(np.float32), (0, 0), 4)
        bm = (f > np.median(f)).astype(np.uint8) * 255
        for c in sorted(do.find_contours(bm), key=len)[-2:]:
            for ratio in (1.5, 0.6):
                assert same_ring(c, ratio)


def test_axis_rectangle_rings_need_no_union():
    """The device skips the sweep for axis-aligned rectangle contours (text
    lines): their round-join offset is a convex rounded rectangle, and its
    min-area box equals the one of Clipper's union ring."""
    rng = np.random.default_rng(3)
    for _ in range(400):
        bm = np.zeros((120, 200), np.uint8)
        x0, y0 = rng.integers(2, 100), rng.integers(2, 60)
        w, h = rng.integers(1, 95), rng.integers(1, 55)
        bm[y0:y0 + h, x0:x0 + w] = 255
        for c in do.find_contours(bm):
            ratio = float(rng.uniform(0.2, 3.0))
            d = do.unclip_distance(c, ratio)
            if len(c) != 4 or d is None:
                continue
            raw = np.array(dn.offset_raw(c, d), np.int32).reshape(-1, 2)
            full = np.asarray(do.unclip(c, ratio), np.int32).reshape(-1, 2)
            assert do.get_mini_boxes(raw) == do.get_mini_boxes(full)


@pytest.mark.parametrize("lanes", [32, 5])
def test_union_list_steps_split_over_lanes(lanes):
    """The sweep's list-wide steps split over the lanes of a warp (emulated
    by threads meeting at a barrier where the device's lanes meet at
    __syncwarp) give the reference's ring point for point."""
    lib = dn.lib()
    lib.dbh_set_union_lanes(lanes)
    try:
        n = 0
        pred = sh.db_map(960, 960, 40, 200, 0x7EC00000, 3)
        for c in do.find_contours(do.threshold(pred, 0.3)):
            if len(c) > 2:
                assert same_ring(c, 1.5), len(c)
                n += 1
        assert n > 20
        rng = np.random.default_rng(4)
        f = cv2.GaussianBlur(rng.random((300, 400)).astype(np.float32), (0, 0), 4)
        bm = (f > np.median(f)).astype(np.uint8) * 255
        for c in sorted(do.find_contours(bm), key=len)[-2:]:
            assert same_ring(c, 1.5)
    finally:
        lib.dbh_set_union_lanes(1)
