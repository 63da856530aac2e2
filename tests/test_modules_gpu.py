"""The C++ module layer on the GPU, driven by tests/native/modules_test.cpp
(g++ against include/, linked to libtocr_b200.so): PaddleDet::run_batch and
run -> sorted_boxes -> PaddleRec::run_multi and run -> combine_recognition
on synthetic pages, against the oracle (preprocess restatement, the stand-in
head in numpy, extract_boxes_from_bitmap with the reference's Clipper, the
stand-in recognition tokens); and the reference-signature kernel shims
(cuda_fused_resize_normalize_det, cuda_batch_roi_warp, cuda_threshold_to_u8,
cuda_gpu_ccl_detect, cuda_argmax) against the reference's own kernels or
scipy, plus the exception mapping."""
import json
import subprocess

import numpy as np
import pytest
import torch

import modules_native as mn
from oracle import db_oracle as do
from oracle import preprocess_oracle as po
from oracle import ref_kernels as rk
from oracle import synth_host as sh

pytestmark = pytest.mark.gpu
ndimage = pytest.importorskip("scipy.ndimage")

SEED = 0x7EC00005
N_PAGES = 2
V = 100
BUCKETS = [320, 480, 800, 1200, 1600, 2000, 2500, 3200, 4000]
STD = np.array([0.229, 0.224, 0.225], np.float32)
MEAN = np.array([0.485, 0.456, 0.406], np.float32)


def standin_prob(chw):
    ink = 1 - (chw * STD[:, None, None] + MEAN[:, None, None]).sum(0) * np.float32(1 / 3)
    H, W = ink.shape
    pad = np.zeros((H, W + 14), np.float32)
    pad[:, 7:7 + W] = ink
    m = np.max(np.stack([pad[:, d:d + W] for d in range(15)]), axis=0)
    return (1 / (1 + np.exp(-12 * (m - 0.5)))).astype(np.float32)


def standin_tokens(crop_id, T):
    out = []
    for t in range(T):
        h = sh.hash3(SEED, 7000 + crop_id, t // 3)
        out.append(0 if h & 1 else 1 + (h >> 32) % (V - 1))
    return out


def collapse(tokens):
    res, last = [], -1
    for t in tokens:
        if t != last and t != 0 and t < V:
            res.append(t)
        last = t
    return res


@pytest.fixture(scope="module")
def run(tmp_path_factory):
    d = tmp_path_factory.mktemp("mod")
    pages = np.stack([sh.make_page(960, 960, SEED, 20 + i) for i in range(N_PAGES)])
    (d / "pages.bin").write_bytes(pages.tobytes())
    labels = [f"L{i:02d}" for i in range(V - 2)]
    (d / "dict.txt").write_text("\n".join(labels) + "\n")
    out = subprocess.run([str(mn.build()), "gpu", str(d / "pages.bin"), str(N_PAGES),
                          str(d / "dict.txt"), str(d)], capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr
    return json.loads(out.stdout), pages, ["blank"] + labels + [" "], d


def test_paddle_det_matches_reference_path(run):
    r, pages, _, _ = run
    assert r["single_same"] == 1
    for i in range(N_PAGES):
        canvas = po.preprocess_image(pages[i], (960, 960), (960, 960))
        ref = do.db_postprocess(standin_prob(canvas), 0.3, 0.6, 1.5)
        assert len(ref) >= 15
        got = r["pages"][i]
        ref_sorted = sorted([b for b, _ in ref], key=lambda b: (b[0][1] // 10, b[0][0]))
        assert got["boxes"] == ref_sorted
        assert np.allclose(got["det_scores"], [s for _, s in ref], atol=1e-3)


def test_paddle_rec_and_combine(run):
    r, _, labels, _ = run
    assert r["run_same"] == 1
    crop_id = 0
    p_max = 1 / (1 + (V - 1) * np.exp(np.float32(-16)))
    for page in r["pages"]:
        kept = 0
        for box, (text, score) in zip(page["boxes"], page["texts"]):
            from oracle._crop import crop_transform_full
            rw = max(crop_transform_full(box, 48, 4000)[1], 32)
            bucket = next(b for b in BUCKETS if b >= min(rw, 4000))
            toks = collapse(standin_tokens(crop_id, bucket // 4))
            assert text == "".join(labels[t] for t in toks)
            assert (score == 0 and not toks) or abs(score - p_max) <= 1e-5
            kept += bool(text) and score >= 0.5
            crop_id += 1
        assert page["kept"] == kept and page["degraded"] == int(kept == 0 and len(page["boxes"]) > 0)


def test_kernel_shims_against_reference_kernels(run, cuda):
    r, pages, _, d = run
    page = torch.from_numpy(pages[0]).to(cuda)
    ref = torch.empty(3, 736, 960, dtype=torch.float32, device=cuda)
    assert rk.lib().refk_fused_single(page.data_ptr(), 960, 960, 960 * 3, ref.data_ptr(), 960, 736,
                                      None) == 0
    torch.cuda.synchronize()
    got = np.fromfile(d / "fused_det.f32", np.float32).reshape(3, 736, 960)
    assert np.array_equal(got, ref.cpu().numpy())
    minv = torch.from_numpy(np.fromfile(d / "roi_minv.f32", np.float32)).to(cuda)
    cw = torch.from_numpy(np.fromfile(d / "roi_cw.i32", np.int32)).to(cuda)
    nb = cw.numel()
    warp = torch.empty(nb, 3, 48, 320, dtype=torch.float32, device=cuda)
    assert rk.lib().refk_roi_warp(page.data_ptr(), 960, 960, 960 * 3, minv.data_ptr(), cw.data_ptr(),
                                  warp.data_ptr(), nb, 48, 320, None) == 0
    torch.cuda.synchronize()
    got = np.fromfile(d / "roi_warp.f32", np.float32).reshape(nb, 3, 48, 320)
    assert np.array_equal(got, warp.cpu().numpy())
    prob = np.fromfile(d / "prob.f32", np.float32).reshape(736, 960)
    bm = np.fromfile(d / "threshold.u8", np.uint8).reshape(736, 960)
    assert np.array_equal(bm, np.where(prob > np.float32(0.3), 255, 0).astype(np.uint8))
    lab, n = ndimage.label(bm > 0, structure=np.ones((3, 3)))
    first = ndimage.minimum(np.arange(bm.size).reshape(bm.shape), lab, range(1, n + 1))
    order = np.argsort(first)
    want = []
    for k in order:
        ys, xs = np.nonzero(lab == k + 1)
        if len(xs) < 3 or xs.max() - xs.min() + 1 < 3 or ys.max() - ys.min() + 1 < 3:
            continue
        mean = float(prob[ys, xs].astype(np.float64).mean())
        if mean < 0.6:
            continue
        want.append((xs.min(), ys.min(), xs.max(), ys.max(), len(xs), mean))
    ccl = r["ccl"]
    assert ccl["total"] == n and ccl["kept"] == len(want) > 10
    for g, w in zip(ccl["boxes"], want):
        assert g[:5] == list(w[:5]) and abs(g[5] - w[5]) <= 1e-3
    idx, sc = r["argmax"]
    rows = (np.arange(4 * 37) * 7919 % 101 - 50).astype(np.float32).reshape(4, 37)
    rows[1, 5] = rows[1, 9] = 1000
    assert idx == rows.argmax(1).tolist() and sc == rows.max(1).tolist()
    assert r["throws"] == 1
