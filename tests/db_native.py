"""Builds and loads the test-only host build of the DB geometry header
(tests/native/db_geom_host.cpp), so CPU tests can compare each routine with
OpenCV and with the reference's Clipper."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "native" / "db_geom_host.cpp"
HDR = ROOT / "turboocr_b200" / "csrc" / "db_geom.cuh"
UNION_HDR = ROOT / "turboocr_b200" / "csrc" / "clipper_union.cuh"
OUT = ROOT / "tests" / "native" / "_build" / "libdbgeom_host.so"

_lib = None
_crop = None
CROP_SRC = ROOT / "tests" / "native" / "crop_host.cpp"
CROP_HDR = ROOT / "turboocr_b200" / "csrc" / "crop_geom.cuh"
CROP_OUT = ROOT / "tests" / "native" / "_build" / "libcrop_host.so"


def crop_lib():
    """Host build of crop_geom.cuh (no FMA contraction beyond its explicit fma())."""
    global _crop
    if _crop is not None:
        return _crop
    CROP_OUT.parent.mkdir(exist_ok=True)
    if not CROP_OUT.exists() or CROP_OUT.stat().st_mtime < max(CROP_SRC.stat().st_mtime,
                                                               CROP_HDR.stat().st_mtime):
        subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared",
                        f"-I{CROP_HDR.parent}", "-o", str(CROP_OUT), str(CROP_SRC)], check=True)
    L = C.CDLL(str(CROP_OUT))
    L.crop_host_transform.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_void_p]
    _crop = L
    return L


def lib():
    global _lib
    if _lib is not None:
        return _lib
    OUT.parent.mkdir(exist_ok=True)
    if not OUT.exists() or OUT.stat().st_mtime < max(SRC.stat().st_mtime, HDR.stat().st_mtime,
                                                     UNION_HDR.stat().st_mtime):
        subprocess.run(["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fPIC", "-shared",
                        "-pthread", f"-I{HDR.parent}", "-o", str(OUT), str(SRC)], check=True)
    L = C.CDLL(str(OUT))
    vp, i, d = C.c_void_p, C.c_int, C.c_double
    L.dbh_trace.argtypes = [vp, i, i, i, i, i, vp, i]
    L.dbh_trace_bits.argtypes = [vp, i, i, i, i, i, vp, i]
    L.dbh_hull.argtypes = [vp, i, vp]
    L.dbh_hull_table.argtypes = [vp, i, vp, i, i, i]
    L.dbh_offset_parallel.argtypes = [vp, i, d, vp, i]
    L.dbh_offset_prepare.argtypes = [vp, i, vp, i]
    L.dbh_min_area_rect.argtypes = [vp, i, vp]
    L.dbh_mini_box.argtypes = [vp, i, vp, vp]
    L.dbh_area.argtypes = [vp, i]
    L.dbh_area.restype = d
    L.dbh_arclen.argtypes = [vp, i]
    L.dbh_arclen.restype = d
    L.dbh_offset_raw.argtypes = [vp, i, d, vp, i]
    L.dbh_unclip_union.argtypes = [vp, i, d, vp, i]
    L.dbh_sort_check.argtypes = [vp, i, vp, vp]
    L.dbh_set_union_lanes.argtypes = [i]
    L.dbh_poly_mask.argtypes = [vp, i, i, i, i, i, vp]
    L.dbh_poly_mask_parity.argtypes = [vp, i, i, i, i, i, vp]
    _lib = L
    return L


def _pts(p):
    return np.ascontiguousarray(np.asarray(p, dtype=np.int32).reshape(-1, 2))


def trace(bm, x0, y0, hole, bits=False):
    bm = np.ascontiguousarray(bm, dtype=np.uint8)
    H, W = bm.shape
    cap = 8 * (H + W) * 4 + 64
    out = np.zeros((cap, 2), np.int32)
    fn = lib().dbh_trace_bits if bits else lib().dbh_trace
    n = fn(bm.ctypes.data, H, W, x0, y0, 1 if hole else 0, out.ctypes.data, cap)
    assert 0 <= n <= cap
    return out[:n]


def hull(p):
    p = _pts(p)
    out = np.zeros((len(p) + 1, 2), np.int32)
    m = lib().dbh_hull(p.ctypes.data, len(p), out.ctypes.data)
    return out[:m]


def hull_table(p, col_cap=1 << 20, hull_cap=1 << 20, interior_filter=False):
    """The column-table hull of the device's shared-memory path."""
    a = _pts(p)
    out = np.zeros((len(a) + 1, 2), np.int32)
    m = lib().dbh_hull_table(a.ctypes.data, len(a), out.ctypes.data, col_cap, hull_cap,
                             1 if interior_filter else 0)
    return m if m < 0 else out[:m]


def offset_prepare(p, rule=False):
    """The prepared offset path (sequential form, or the CTA's rule)."""
    a = _pts(p)
    out = np.zeros((len(a) + 1, 2), np.int32)
    m = lib().dbh_offset_prepare(a.ctypes.data, len(a), out.ctypes.data, 1 if rule else 0)
    return out[:m].tolist()


def offset_parallel(p, delta):
    """Offset ring by independent vertices (None when a joint keeps k)."""
    a = _pts(p)
    cap = 64 * len(a) + 64
    out = np.zeros((cap, 2), np.int32)
    n = lib().dbh_offset_parallel(a.ctypes.data, len(a), float(delta), out.ctypes.data, cap)
    return None if n < 0 else [tuple(v) for v in out[:n].tolist()]


def min_area_rect(p):
    p = _pts(p)
    o = np.zeros(5, np.float32)
    lib().dbh_min_area_rect(p.ctypes.data, len(p), o.ctypes.data)
    return o


def mini_box(p):
    p = _pts(p)
    box = np.zeros(8, np.int32)
    ms = np.zeros(1, np.float32)
    lib().dbh_mini_box(p.ctypes.data, len(p), box.ctypes.data, ms.ctypes.data)
    return box.reshape(4, 2).tolist(), ms[0]


def area(p):
    p = _pts(p)
    return lib().dbh_area(p.ctypes.data, len(p))


def arclen(p):
    p = _pts(p)
    return lib().dbh_arclen(p.ctypes.data, len(p))


def offset_raw(p, delta):
    p = _pts(p)
    cap = 1 << 16
    out = np.zeros((cap, 2), np.int32)
    n = lib().dbh_offset_raw(p.ctypes.data, len(p), delta, out.ctypes.data, cap)
    return [tuple(q) for q in out[:n].tolist()]


def poly_mask(p, x0, y0, w, h, parity=False):
    p = _pts(p)
    m = np.zeros((h, w), np.uint8)
    fn = lib().dbh_poly_mask_parity if parity else lib().dbh_poly_mask
    fn(p.ctypes.data, len(p), x0, y0, w, h, m.ctypes.data)
    return m


def unclip_union(p, delta):
    """The largest ring of Clipper's union of the raw offset (clipper_union.cuh)."""
    p = _pts(p)
    cap = 1 << 20
    out = np.zeros(2 * cap, dtype=np.int32)
    n = lib().dbh_unclip_union(p.ctypes.data, len(p), delta, out.ctypes.data, cap)
    if n < 0:
        raise RuntimeError(f"union sweep failed ({n})")
    return out[: 2 * n].reshape(n, 2)


def sort_check(keys):
    """(std::sort permutation, std_sort permutation) of keys by descending value."""
    k = np.ascontiguousarray(keys, dtype=np.int32)
    a = np.zeros(len(k), np.int32)
    b = np.zeros(len(k), np.int32)
    assert lib().dbh_sort_check(k.ctypes.data, len(k), a.ctypes.data, b.ctypes.data) == 0
    return a, b
