"""Crop geometry (compute_crop_transform, perspective.h:25-67) on the CPU: the
restatement in turboocr_b200/csrc/crop_geom.cuh, built for the host, against
the reference's own header compiled with the reference's flags
(oracle/_ref/libcrop_ref.so). M_inv, crop width and the vertical flag must
be bit-identical."""
import ctypes as C

import numpy as np
import pytest

import db_native as dn
from oracle._loader import load


def ref_lib():
    L = load("_ref/libcrop_ref.so")
    L.crop_ref_transform.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                     C.c_void_p]
    return L


def both(box, th=48, mw=320):
    b = np.ascontiguousarray(np.asarray(box, np.int32).reshape(8))
    out = []
    for fn in (ref_lib().crop_ref_transform, dn.crop_lib().crop_host_transform):
        m = np.zeros(9, np.float32)
        cw = C.c_int()
        v = C.c_int()
        fn(b.ctypes.data, th, mw, m.ctypes.data, C.byref(cw), C.byref(v))
        out.append((m, cw.value, v.value))
    return out


def rotated_boxes(n, seed):
    rng = np.random.default_rng(seed)
    for _ in range(n):
        cx, cy = rng.uniform(0, 960, 2)
        w, h = rng.uniform(4, 800), rng.uniform(4, 120)
        if rng.random() < 0.2:
            w, h = h, w  # vertical lines
        a = np.deg2rad(rng.uniform(-20, 20))
        c, s = np.cos(a), np.sin(a)
        pts = [(cx + dx * c - dy * s, cy + dx * s + dy * c)
               for dx, dy in ((-w / 2, -h / 2), (w / 2, -h / 2), (w / 2, h / 2), (-w / 2, h / 2))]
        yield np.rint(pts).astype(np.int32)


def test_crop_transform_bit_exact():
    n = 0
    for box in rotated_boxes(3000, 5):
        (m1, w1, v1), (m2, w2, v2) = both(box)
        assert w1 == w2 and v1 == v2
        assert (m1.view(np.uint32) == m2.view(np.uint32)).all(), (box.tolist(), m1, m2)
        n += v1
    assert n > 100  # vertical crops exercised


@pytest.mark.parametrize("box", [[[0, 0], [0, 0], [0, 0], [0, 0]],        # degenerate
                                 [[5, 5], [6, 5], [6, 5], [5, 5]],        # zero height
                                 [[10, 10], [2000, 10], [2000, 30], [10, 30]],  # clamp to max_w
                                 [[10, 10], [20, 10], [20, 100], [10, 100]]])  # vertical
def test_crop_transform_edge_cases(box):
    (m1, w1, v1), (m2, w2, v2) = both(box)
    assert w1 == w2 and v1 == v2
    assert (m1.view(np.uint32) == m2.view(np.uint32)).all()
