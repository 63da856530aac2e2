"""The C++ interface of libtocr_b200.so, compiled with g++ against include/
as a reference-side caller would be (tests/native/modules_test.cpp), host
part (no GPU): crop transform and recognizer widths against the reference's
own perspective header, reading order, corner order, the dictionary loader
(one LF then one CR stripped), the CTC helpers, the combine step and the
resize policy."""
import json
import subprocess

import numpy as np

import modules_native as mn
from oracle import ctc_oracle as co
from oracle import db_oracle as do
from oracle._crop import crop_transform_full

QUADS = [[[10, 20], [210, 24], [209, 60], [9, 56]], [[5, 5], [25, 5], [25, 200], [5, 200]],
         [[0, 0], [3000, 0], [3000, 20], [0, 20]]]
BUCKETS = [320, 480, 800, 1200, 1600, 2000, 2500, 3200, 4000]


def run_host(tmp_path):
    d = tmp_path / "dict.txt"
    d.write_bytes(b"a\nb\r\r\nc\r\n")
    out = subprocess.run([str(mn.build()), "host", str(d)], capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0, out.stderr
    return json.loads(out.stdout)


def sorted_boxes(boxes):
    return sorted(boxes, key=lambda b: (b[0][1] // 10, b[0][0]))  # stable


def test_cpp_host_api(tmp_path):
    r = run_host(tmp_path)
    for q, got in zip(QUADS, r["crops"]):
        m, w, v = crop_transform_full(q, 48, 320)
        assert got["w"] == w and got["v"] == v
        assert np.array_equal(np.array(got["m"], np.float32), m)
        rw = max(crop_transform_full(q, 48, 4000)[1], 32)
        assert got["rw"] == rw
        assert got["bucket"] == next(b for b in BUCKETS if b >= min(rw, 4000))
        wq = max(abs(q[1][0] - q[0][0]), abs(q[2][0] - q[3][0]))
        hq = max(abs(q[3][1] - q[0][1]), abs(q[2][1] - q[1][1]))
        assert got["vert"] == int(hq * hq >= wq * wq * 225 // 100)
    boxes = [[[50, 31], [90, 31], [90, 40], [50, 40]], [[10, 35], [40, 35], [40, 45], [10, 45]],
             [[5, 2], [9, 2], [9, 8], [5, 8]], [[1, 39], [4, 39], [4, 49], [1, 49]]]
    assert r["sorted"] == sorted_boxes(boxes)
    xs, ys = do.order_quad([3.0, 1.0, 1.0, 3.0], [5.0, 5.0, 1.0, 1.0])
    assert r["quad"] == [v for p in zip(xs, ys) for v in p]
    assert r["dict_ok"] == 1 and r["labels"] == ["blank", "a", "b\r", "c", " "]
    idx = [0, 1, 1, 0, 2, 2, 3, 0, 3]
    sc = np.array([0.9, 0.8, 0.7, 0.9, 0.6, 0.5, 0.4, 0.9, 0.2], np.float32)
    toks, score = co.collapse(idx, sc, 5)
    text = "".join(r["labels"][t] for t in toks)
    assert r["ctc"][0] == text and r["ctc"][2] == text
    assert np.float32(r["ctc"][1]) == np.float32(score) == np.float32(r["ctc"][3])
    kept, first, deg1, deg2, warning = r["combine"]
    assert (kept, first, deg1, deg2) == (1, "ab", 0, 1)
    assert "no usable text" in warning and "dropped 2 crop(s)" in warning
    assert r["resize"] == [736, 960]
