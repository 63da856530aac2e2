"""The bench's reference arm and CPU baseline run on the host only: they load
none of this repository's native libraries (only oracle/ builds of the
reference's own sources), and their inputs match the device generators."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]

PROBE = r"""
import json, sys
sys.path.insert(0, %r)
import bench
from oracle.cpu_baselines import BASELINES
vals, desc = BASELINES["ctc"](2, 1, lines=4)
maps = open("/proc/self/maps").read()
libs = sorted({l.split()[-1] for l in maps.splitlines() if l.split()[-1].endswith(".so")
               and %r in l.split()[-1]})
print(json.dumps({"libs": libs, "value": vals[0]}))
"""


def test_reference_arm_loads_no_product_library():
    out = subprocess.run([sys.executable, "-c", PROBE % (str(ROOT), str(ROOT))],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["value"] > 0
    assert res["libs"], "the reference CTC library should be loaded"
    for lib in res["libs"]:
        assert "/oracle/" in lib, lib
        assert "libtocr" not in lib, lib


def test_host_generators_match_the_device_library_generators():
    from oracle import synth_host as sh
    from turboocr_b200._lib import synth
    L = synth()
    for s, st, i in [(0x7EC00005, 5000, 0), (1, 2, 3), (0x7EC00000, 3000 + (1 << 40), 12345)]:
        assert L.tocr_synth_hash(s, st, i) == sh.hash3(s, st, i)
    ref = np.zeros((240, 320), np.float32)
    L.tocr_synth_db_map_host(ref.ctypes.data, 240, 320, 5, 20, 0x7EC00000, 1)
    assert np.array_equal(sh.db_map(240, 320, 5, 20, 0x7EC00000, 1), ref)


def test_round32_rounds_halves_away_from_zero():
    """det_config.h:50-52 uses std::round: 720 / 32 = 22.5 -> 23 * 32 = 736."""
    from oracle import cpu_baselines as cb
    from turboocr_b200.det_config import DetResizeParams, compute_det_resize
    assert cb.round32_floor(720.0) == 736
    assert cb.round32_floor(16.0) == 32
    assert compute_det_resize(960, 1280, DetResizeParams("max", 960, 960)) == (736, 960)
    for h, w in [(600, 2000), (2000, 600), (961, 961), (700, 900), (1, 5000)]:
        assert compute_det_resize(h, w, DetResizeParams("max", 960, 960)) == \
            cb.det_resize_max(h, w)


def test_both_arms_print_the_same_config():
    sys.path.insert(0, str(ROOT))
    import bench
    for name, Wl in bench.WORKLOADS.items():
        a = bench.workload_config(Wl, 1, 0)
        b = bench.workload_config(Wl, 1, 0)
        assert a == b and a["workload"] == Wl.name
    assert bench.workload_config(bench.E2eWorkload, 8, 0)["pages_per_gpu"] == 512
