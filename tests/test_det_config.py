"""Detection resize policy and DB parameters (det_config.h:13-163 of the
reference) through the library's C++: defaults, rounding, the max-side cap,
and the environment overrides with their clamps."""
import os

import pytest

from turboocr_b200 import det_config as dc

VARS = ("DET_LIMIT_TYPE", "DET_LIMIT_SIDE_LEN", "DET_MAX_SIDE_LIMIT", "DET_MAX_SIDE",
        "DET_DB_THRESH", "DET_BOX_THRESH", "DET_UNCLIP")


@pytest.fixture
def env():
    saved = {k: os.environ.get(k) for k in VARS}
    for k in VARS:
        os.environ.pop(k, None)
    yield os.environ
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


def test_compute_det_resize_policies():
    mx = dc.DetResizeParams("max", 960, 960)
    assert dc.compute_det_resize(2000, 1000, mx) == (960, 480)
    assert dc.compute_det_resize(500, 700, mx) == (512, 704)      # no upscale under "max"
    mn = dc.K_DET_RESIZE_DEFAULT                                  # {"min", 64, 1280}
    assert dc.compute_det_resize(32, 100, mn) == (64, 192)        # grow the shorter side to 64
    assert dc.compute_det_resize(3000, 1000, mn) == (1280, 416)   # cap, then re-round
    assert dc.compute_det_resize(5, 5, mx) == (32, 32)            # floor 32


def test_read_det_resize_env(env):
    assert dc.read_det_resize() == dc.K_DET_RESIZE_DEFAULT
    env["DET_LIMIT_TYPE"] = "MAX"
    p = dc.read_det_resize()
    # a "min" base switched to "max" without a side length takes the cap
    assert p == dc.DetResizeParams("max", 1280, 1280)
    env["DET_LIMIT_SIDE_LEN"] = "960"
    env["DET_MAX_SIDE_LIMIT"] = "99999"                           # clamped to 4096
    assert dc.read_det_resize() == dc.DetResizeParams("max", 960, 4096)
    env["DET_MAX_SIDE"] = "640"                                   # shrink-only
    assert dc.read_det_resize() == dc.DetResizeParams("max", 960, 640)
    env["DET_LIMIT_SIDE_LEN"] = "-5"                              # clamped to 32
    assert dc.read_det_resize().limit_side_len == 32


def test_effective_max_side_and_db_params(env):
    assert dc.effective_det_max_side(dc.DetResizeParams("min", 64, 1000)) == 1024
    env["DET_MAX_SIDE"] = "10"
    assert dc.effective_det_max_side() == 32
    p = dc.read_db_params()
    assert (p.thresh, p.box_thresh, p.unclip_ratio) == pytest.approx((0.2, 0.45, 1.4), abs=1e-6)
    env["DET_DB_THRESH"] = "0.3"
    env["DET_UNCLIP"] = "1.5"
    p = dc.read_db_params()
    assert abs(p.thresh - 0.3) < 1e-7 and p.box_thresh == pytest.approx(0.45)
    assert p.unclip_ratio == 1.5
