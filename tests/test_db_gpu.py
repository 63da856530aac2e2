"""Subsystem 3 parity on the GPU: tocr_db_postprocess against the CPU
restatement of extract_boxes_from_bitmap (oracle/db_oracle.py: cv2 4.13 +
the reference's Clipper).

The bar: bit-exact boxes, in contour order, against the unmodified oracle,
whose unclip is the reference's own Clipper (offset and union), on the
config-1 maps and on other seeds, sizes and shapes. This pins every device
stage: threshold, labelling, contour order and the 3000 cap, border
following, both min-area boxes, the polygon-mask score, the round-join
offset, Clipper's union sweep, scaling and filters. Scores within 1e-3
(measured: equal to float rounding). The labelling stage is also checked on
its own (tocr_db_components) as a partition against scipy's 8-/4-connected
labelling."""
import numpy as np
import pytest
import torch

from oracle import db_oracle as do

pytestmark = pytest.mark.gpu

cv2 = pytest.importorskip("cv2")
ndimage = pytest.importorskip("scipy.ndimage")

SCORE_TOL = 1e-3


def synth_maps(n, h, w, kmin=40, kmax=200, seed=0x7EC00000, first=0):
    from turboocr_b200._lib import synth
    out = np.zeros((n, h, w), np.float32)
    for i in range(n):
        synth().tocr_synth_db_map_host(out[i].ctypes.data, h, w, kmin, kmax, seed, first + i)
    return out


def run_gpu(cuda, maps, **kw):
    from turboocr_b200.kernels import DbPostprocess
    n, h, w = maps.shape
    db = DbPostprocess(n, h, w, cuda, **kw)
    pred = torch.from_numpy(maps).to(cuda)
    db(pred)
    torch.cuda.synchronize()
    return db.results()


def compare_exact(gpu, ref):
    assert [b for b, _ in gpu] == [b for b, _ in ref]
    for (_, s1), (_, s2) in zip(gpu, ref):
        assert abs(s1 - s2) <= SCORE_TOL


@pytest.mark.parametrize("shortcuts", [True, False])
@pytest.mark.parametrize("hw", [(37, 53), (64, 64), (100, 333), (960, 960)])
def test_components_partition(cuda, hw, shortcuts):
    from turboocr_b200.kernels import db_components
    h, w = hw
    rng = np.random.default_rng(h * w)
    maps = rng.random((3, h, w)).astype(np.float32)
    maps[1] = (maps[1] > 0.5) * 0.9          # coarse blobs after smoothing below
    maps[1] = ndimage.uniform_filter(maps[1], 5)
    maps[2] = synth_maps(1, h, w, 3, 12)[0]
    maps[0][: h // 2] = 0.0      # a band of background-only tiles next to mixed ones
    labels, bitmap = db_components(torch.from_numpy(maps).to(cuda), 0.3, shortcuts=shortcuts)
    labels = labels.cpu().numpy()
    bitmap = bitmap.cpu().numpy()
    for m in range(3):
        fg = maps[m] > np.float32(0.3)
        assert (bitmap[m] == np.where(fg, 255, 0)).all()
        lab = labels[m]
        idx = np.arange(h * w).reshape(h, w) + 1
        l8, n8 = ndimage.label(fg, structure=np.ones((3, 3)))
        for k in range(1, n8 + 1):
            sel = l8 == k
            vals = np.unique(lab[sel])
            assert len(vals) == 1 and vals[0] == idx[sel].min()
        l4, n4 = ndimage.label(np.pad(~fg, 1, constant_values=True))
        l4 = l4[1:-1, 1:-1]
        outer = set(np.unique(np.concatenate([l4[0], l4[-1], l4[:, 0], l4[:, -1]]))) - {0}
        for k in range(1, n4 + 1):
            sel = l4 == k
            if not sel.any():
                continue
            vals = np.unique(lab[sel])
            want = 0 if k in outer else idx[sel].min()
            assert len(vals) == 1 and vals[0] == want


def test_db_config1_exact(cuda):
    """BASELINE config 1 at full size: 8 maps 960x960, 40-200 rectangles."""
    maps = synth_maps(8, 960, 960)
    got = run_gpu(cuda, maps)
    n = 0
    for m in range(8):
        ref = do.db_postprocess(maps[m])
        compare_exact(got[m], ref)
        n += len(ref)
    assert n > 60


@pytest.mark.parametrize("hw,k", [((240, 320), (5, 30)), ((97, 131), (2, 8)), ((512, 96), (3, 10))])
def test_db_small_maps_exact(cuda, hw, k):
    maps = synth_maps(4, hw[0], hw[1], k[0], k[1], first=100)
    got = run_gpu(cuda, maps)
    for m in range(4):
        compare_exact(got[m], do.db_postprocess(maps[m]))


def test_db_noise_and_holes_exact(cuda):
    """Blobby noise: many contours, hole borders, thin and one-pixel parts."""
    rng = np.random.default_rng(7)
    maps = ndimage.uniform_filter(rng.random((6, 128, 160)).astype(np.float32), (1, 3, 3))
    maps = np.clip((maps - 0.45) * 4, 0, 1).astype(np.float32)
    got = run_gpu(cuda, maps, box_thresh=0.5)
    for m in range(6):
        compare_exact(got[m], do.db_postprocess(maps[m], box_thresh=0.5))


def test_db_edge_cases(cuda):
    h, w = 64, 96
    maps = np.zeros((4, h, w), np.float32)
    maps[1][:] = 0.9                          # one component covering the map
    maps[2][10:30, 5:80] = 0.95               # one rectangle with a hole
    maps[2][15:22, 20:40] = 0.0
    maps[3][h // 2, :] = 0.9                  # a one-pixel line
    got = run_gpu(cuda, maps)
    assert got[0] == []
    for m in range(1, 4):
        compare_exact(got[m], do.db_postprocess(maps[m]))
    assert len(got[1]) == 1


def test_db_3000_cap(cuda):
    """More than 3000 contours: only the first 3000 in cv2's order (descending
    raster order of their starts) are candidates, so a text rectangle near
    the top of the map, whose contour comes last, is dropped."""
    h, w = 300, 400
    m = np.zeros((h, w), np.float32)
    m[10:40, 20:300] = 0.9                    # early start -> late in the list
    m[60::3, ::3] = 0.9                       # isolated dots: 80 x 134 contours
    maps = m[None].copy()
    total = len(do.find_contours(do.threshold(m, 0.3)))
    assert total > 3000
    got = run_gpu(cuda, maps)
    ref = do.db_postprocess(m)
    compare_exact(got[0], ref)
    assert ref == []
    m2 = m.copy()
    m2[60:, :] = 0                            # without the dots the box is found
    got2 = run_gpu(cuda, m2[None].copy())
    assert len(got2[0]) == 1


def test_db_geometry_scaling(cuda):
    """orig != resize: boxes are scaled back and clamped (det_postprocess.cpp:205-210)."""
    from turboocr_b200.kernels import DbPostprocess
    maps = synth_maps(2, 320, 480, 5, 20, first=200)
    geo = torch.tensor([[500, 700, 320, 480], [160, 240, 320, 480]], dtype=torch.int32,
                       device=cuda)
    db = DbPostprocess(2, 320, 480, cuda)
    db(torch.from_numpy(maps).to(cuda), geometry=geo)
    got = db.results()
    for m, (oh, ow) in enumerate([(500, 700), (160, 240)]):
        ref = do.extract_boxes_from_bitmap(maps[m], do.threshold(maps[m], 0.3), oh, ow, 320, 480,
                                           0.6, 1.5)
        compare_exact(got[m], ref)


@pytest.mark.parametrize("first", [300, 600])
def test_db_more_config1_seeds_exact(cuda, first):
    """Other config-1 seeds: every box equal to the full reference path."""
    maps = synth_maps(8, 960, 960, first=first)
    got = run_gpu(cuda, maps)
    n = 0
    for m in range(8):
        ref = do.db_postprocess(maps[m])
        compare_exact(got[m], ref)
        n += len(ref)
    assert n > 60


@pytest.mark.parametrize("size,angle", [((480, 640), 15), ((800, 1200), -15), ((256, 256), 45),
                                        ((600, 900), 75)])
def test_db_rotated_shapes_exact(cuda, size, angle):
    """Filled rotated rectangles and ellipses (staircase contours whose
    offset paths cross themselves at every step) at one angle each."""
    h, w = size
    rng = np.random.default_rng(h + angle)
    maps = np.zeros((3, h, w), np.float32)
    for m in range(3):
        bm = np.zeros((h, w), np.uint8)
        for _ in range(12):
            cx, cy = rng.uniform(0.1, 0.9) * w, rng.uniform(0.1, 0.9) * h
            a = angle + rng.uniform(-3, 3)
            ww, hh = rng.uniform(20, 0.4 * w), rng.uniform(6, 50)
            if rng.random() < 0.7:
                box = cv2.boxPoints(((cx, cy), (ww, hh), a)).astype(np.int32)
                cv2.fillPoly(bm, [box], 1)
            else:
                cv2.ellipse(bm, ((cx, cy), (ww, hh), a), 1, -1)
        maps[m] = bm * rng.uniform(0.65, 1.0, (h, w)).astype(np.float32)
    got = run_gpu(cuda, maps)
    for m in range(3):
        compare_exact(got[m], do.db_postprocess(maps[m]))


@pytest.fixture
def shared_columns():
    """Sets the shared-memory geometry's column capacity for one test, then
    restores it."""
    from turboocr_b200._lib import lib
    yield lambda v: lib().tocr_debug_db_shared_columns(v)
    lib().tocr_debug_db_shared_columns(-1)


@pytest.mark.parametrize("cap", [0, 300])
def test_db_global_scratch_path_exact(cuda, shared_columns, cap):
    """Point sets wider than the shared-memory column table take the
    one-thread global scratch path (cap 0: every set above 96 points; 300
    columns: a mix): same boxes."""
    shared_columns(cap)
    maps = synth_maps(3, 960, 960, first=400)
    got = run_gpu(cuda, maps)
    for m in range(3):
        compare_exact(got[m], do.db_postprocess(maps[m]))


def test_db_scratch_pool_full_raises(cuda, shared_columns):
    from turboocr_b200.kernels import DbPostprocess
    shared_columns(0)
    maps = synth_maps(2, 960, 960, first=400)
    db = DbPostprocess(2, 960, 960, cuda, offset_cap=64)
    db(torch.from_numpy(maps).to(cuda))
    with pytest.raises(RuntimeError, match="scratch pool"):
        db.results()


@pytest.mark.parametrize("cap", [-1, 1000])
def test_db_wide_jagged_bar_exact(cuda, shared_columns, cap):
    """A contour of ~1300 points over 2560 columns and its ring: through the
    shared-memory table (cap -1) and through the global path (1000 columns)."""
    shared_columns(cap)
    h, w = 48, 2600
    m = np.zeros((h, w), np.float32)
    m[12:36, 20:2580] = 0.9
    for x in range(20, 2580, 8):
        m[10:12, x:x + 4] = 0.9               # jagged top edge
    got = run_gpu(cuda, m[None].copy())
    ref = do.db_postprocess(m)
    assert len(ref) == 1
    compare_exact(got[0], ref)
