"""Mode-2 unclip stages (tocr_jfa_*, the shims of src/kernels/jfa.cu) against
the reference's own jfa.cu kernels compiled into oracle/_ref/libref_kernels.so,
stage by stage on the same inputs: the compact-id map and pre-filter boxes of
tocr_gpu_ccl_detect on config-1 probability maps and on noise bitmaps, with
the reference's mode-2 parameters and with larger discs. Every output is
compared bit for bit (integer maps, float distances, box records including
the oriented corners). Then PaddleDet with GPU_CCL=2 end to end (the C++
harness tests/native/modules_test.cpp) against the reference kernels plus the
host filter of run_gpu_ccl_fast (src/detection/paddle_det_ccl.cpp:222-256)
restated here."""
import ctypes as C
import json
import math
import os
import subprocess

import numpy as np
import pytest
import torch

import modules_native as mn
from oracle import db_oracle as do
from oracle import ref_kernels as rk
from oracle import synth_host as sh

pytestmark = pytest.mark.gpu

KMAX = 3000
REC_INTS = 14  # GpuDetBox = 56 bytes


def ccl(L, bm, prob, box_thresh, dev):
    h, w = bm.shape
    n = h * w
    d_bm = torch.from_numpy(bm).to(dev)
    d_pr = torch.from_numpy(prob).to(dev)
    labels = torch.empty(n, dtype=torch.int32, device=dev)
    cid = torch.empty(n, dtype=torch.int32, device=dev)
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    boxes = torch.zeros(2 * KMAX * REC_INTS, dtype=torch.int32, device=dev)
    nbox = torch.zeros(1, dtype=torch.int32, device=dev)
    h_boxes = torch.zeros(KMAX * REC_INTS, dtype=torch.int32).pin_memory()
    h_n, h_total = C.c_int(0), C.c_int(0)
    st = L.tocr_gpu_ccl_detect(d_bm.data_ptr(), d_pr.data_ptr(), w, h, box_thresh,
                               labels.data_ptr(), cid.data_ptr(), counter.data_ptr(),
                               boxes.data_ptr(), nbox.data_ptr(), h_boxes.data_ptr(),
                               C.byref(h_n), C.byref(h_total), None)
    assert st == 0, L.tocr_last_error_string()
    return d_bm, cid, boxes, min(h_total.value, KMAX), h_n.value


def run_chain(L, R, bm, prob, box_thresh, ratio, emin, emax, dev):
    """Both chains on the same CCL output; returns the stage outputs of each."""
    h, w = bm.shape
    n = h * w
    d_bm, cid, boxes, slots, _ = ccl(L, bm, prob, box_thresh, dev)
    assert slots > 0
    out = {}
    for side in ("own", "own_nolist", "ref"):
        perim = torch.full((KMAX,), -7, dtype=torch.int32, device=dev)
        expand = torch.zeros(KMAX, dtype=torch.float32, device=dev)
        lab = torch.full((n,), 12345, dtype=torch.int32, device=dev)
        seeds = torch.empty(n, dtype=torch.int32, device=dev)
        alt = torch.empty(n, dtype=torch.int32, device=dev)
        bb = torch.zeros(KMAX * REC_INTS, dtype=torch.int32, device=dev)
        ob = torch.zeros(KMAX * REC_INTS, dtype=torch.int32, device=dev)
        mom = torch.empty(KMAX * 6, dtype=torch.int64, device=dev)
        orient = torch.empty(KMAX * 6, dtype=torch.float32, device=dev)
        if side == "ref":
            assert R.refk_jfa_crack(cid.data_ptr(), d_bm.data_ptr(), w, h, slots,
                                    perim.data_ptr(), None) == 0
            assert R.refk_jfa_expand_per_comp(boxes.data_ptr(), perim.data_ptr(), slots, ratio,
                                              emin, emax, box_thresh, expand.data_ptr(),
                                              None) == 0
            assert R.refk_jfa_expand_labels(d_bm.data_ptr(), cid.data_ptr(), expand.data_ptr(),
                                            lab.data_ptr(), w, h, emax, seeds.data_ptr(),
                                            alt.data_ptr(), None) == 0
            assert R.refk_jfa_extract_bboxes(lab.data_ptr(), w, h, bb.data_ptr(), slots,
                                             None) == 0
            assert R.refk_jfa_extract_oriented(lab.data_ptr(), w, h, ob.data_ptr(), slots,
                                               mom.data_ptr(), orient.data_ptr(), None) == 0
        else:
            chk = lambda st: st == 0 or pytest.fail(L.tocr_last_error_string().decode())
            chk(L.tocr_jfa_crack_perimeter(cid.data_ptr(), d_bm.data_ptr(), w, h, slots,
                                           perim.data_ptr(), None))
            chk(L.tocr_jfa_expand_per_comp(boxes.data_ptr(), perim.data_ptr(), slots, ratio,
                                           emin, emax, box_thresh, expand.data_ptr(), None))
            chk(L.tocr_jfa_expand_labels(d_bm.data_ptr(), cid.data_ptr(), expand.data_ptr(),
                                         lab.data_ptr(), w, h, seeds.data_ptr(),
                                         None if side == "own_nolist" else alt.data_ptr(),
                                         None))
            chk(L.tocr_jfa_extract_bboxes(lab.data_ptr(), w, h, bb.data_ptr(), slots, None))
            chk(L.tocr_jfa_extract_oriented(lab.data_ptr(), w, h, ob.data_ptr(), slots,
                                            mom.data_ptr(), orient.data_ptr(), None))
        torch.cuda.synchronize()
        out[side] = dict(perim=perim[:slots].cpu().numpy(),
                         expand=expand[:slots].cpu().numpy().view(np.int32),
                         labels=lab.cpu().numpy().reshape(h, w),
                         bboxes=bb.cpu().numpy().reshape(KMAX, REC_INTS)[:slots],
                         oriented=ob.cpu().numpy().reshape(KMAX, REC_INTS)[:slots])
    return out, slots


def assert_same(out):
    ref = out["ref"]
    for side in ("own", "own_nolist"):
        for k in ("perim", "expand", "labels", "bboxes", "oriented"):
            a, b = out[side][k], ref[k]
            bad = np.argwhere(a != b)
            assert bad.size == 0, (side, k, bad[:5].tolist(), a[tuple(bad[0])], b[tuple(bad[0])])


def noise_bitmap(h, w, seed, density):
    rng = np.random.default_rng(seed)
    small = rng.random((h // 3 + 1, w // 3 + 1)) < density
    bm = np.kron(small, np.ones((3, 3), bool))[:h, :w]
    bm |= rng.random((h, w)) < 0.05
    return np.where(bm, 255, 0).astype(np.uint8), rng.random((h, w)).astype(np.float32)


@pytest.mark.parametrize("k,ratio,emin,emax", [(0, 1.5, 2.0, 24.0), (1, 1.5, 2.0, 24.0),
                                                (2, 3.0, 2.0, 60.0)])
def test_jfa_config1_maps(tocr, cuda, k, ratio, emin, emax):
    pred = sh.db_map(960, 960, 40, 200, 0x7EC00000, k)
    bm = np.where(pred > np.float32(0.3), 255, 0).astype(np.uint8)
    out, slots = run_chain(tocr.lib(), rk.lib(), bm, pred, 0.6, ratio, emin, emax, cuda)
    assert slots >= 3  # overlapping rectangles merge into few components on some maps
    assert (out["ref"]["expand"].view(np.float32) > 0).sum() >= 2
    assert (out["ref"]["oriented"][:, 5] >= 9).sum() >= 2  # grown regions with pixels
    assert_same(out)


@pytest.mark.parametrize("h,w,seed,density", [(97, 131, 1, 0.35), (256, 300, 2, 0.2),
                                              (33, 1000, 3, 0.5)])
def test_jfa_noise_bitmaps(tocr, cuda, h, w, seed, density):
    bm, prob = noise_bitmap(h, w, seed, density)
    out, slots = run_chain(tocr.lib(), rk.lib(), bm, prob, 0.0, 2.0, 1.0, 9.0, cuda)
    assert slots >= 10
    assert_same(out)


def test_jfa_empty_and_arguments(tocr, cuda):
    L = tocr.lib()
    assert L.tocr_jfa_crack_perimeter(None, None, 4, 4, 0, None, None) == 0
    assert L.tocr_jfa_extract_oriented(None, 4, 4, None, 0, None, None, None) == 0
    assert L.tocr_jfa_crack_perimeter(None, None, 4, 4, 3001, None, None) == 1
    assert L.tocr_jfa_expand_labels(None, None, None, None, 0, 4, None, None, None) == 1


def round_half_away(v):
    return math.floor(v + 0.5) if v >= 0 else -math.floor(-v + 0.5)


def mode2_reference(L, R, bm, prob, dev, box_thresh=0.6, ratio=1.5):
    """run_gpu_ccl_fast on one full-page map with the reference's kernels (the
    labelling is this library's: the reference numbers components in an
    unspecified order)."""
    h, w = bm.shape
    n = h * w
    d_bm, cid, boxes, slots, kept = ccl(L, bm, prob, box_thresh, dev)
    if kept == 0 or slots == 0:
        return [], []
    perim = torch.zeros(KMAX, dtype=torch.int32, device=dev)
    expand = torch.zeros(KMAX, dtype=torch.float32, device=dev)
    lab = torch.empty(n, dtype=torch.int32, device=dev)
    seeds = torch.empty(n, dtype=torch.int32, device=dev)
    alt = torch.empty(n, dtype=torch.int32, device=dev)
    ob = torch.zeros(KMAX * REC_INTS, dtype=torch.int32, device=dev)
    mom = torch.empty(KMAX * 6, dtype=torch.int64, device=dev)
    orient = torch.empty(KMAX * 6, dtype=torch.float32, device=dev)
    assert R.refk_jfa_crack(cid.data_ptr(), d_bm.data_ptr(), w, h, slots, perim.data_ptr(),
                            None) == 0
    assert R.refk_jfa_expand_per_comp(boxes.data_ptr(), perim.data_ptr(), slots, ratio, 2.0, 24.0,
                                      box_thresh, expand.data_ptr(), None) == 0
    assert R.refk_jfa_expand_labels(d_bm.data_ptr(), cid.data_ptr(), expand.data_ptr(),
                                    lab.data_ptr(), w, h, 24.0, seeds.data_ptr(), alt.data_ptr(),
                                    None) == 0
    assert R.refk_jfa_extract_oriented(lab.data_ptr(), w, h, ob.data_ptr(), slots,
                                       mom.data_ptr(), orient.data_ptr(), None) == 0
    torch.cuda.synchronize()
    recs = ob.cpu().numpy().reshape(KMAX, REC_INTS)[:slots]
    pre = boxes.cpu().numpy().reshape(2 * KMAX, REC_INTS)[:slots]
    out, scores = [], []
    for i in range(slots):
        xmin, ymin, xmax, ymax, _, pc = (int(v) for v in recs[i, :6])
        if pc < 9 or xmax - xmin + 1 < 5 or ymax - ymin + 1 < 5:
            continue
        px = recs[i, 6:10].view(np.float32).astype(np.float64).tolist()
        py = recs[i, 10:14].view(np.float32).astype(np.float64).tolist()
        xs, ys = do.order_quad(px, py)
        box = [[min(max(round_half_away(x), 0), w - 1), min(max(round_half_away(y), 0), h - 1)]
               for x, y in zip(xs, ys)]
        rw = int(math.sqrt((box[0][0] - box[1][0]) ** 2 + (box[0][1] - box[1][1]) ** 2))
        rh = int(math.sqrt((box[0][0] - box[3][0]) ** 2 + (box[0][1] - box[3][1]) ** 2))
        if rw <= 3 or rh <= 3:
            continue
        out.append(box)
        ssum = pre[i, 4:5].view(np.float32)[0]
        scores.append(float(ssum / np.float32(pre[i, 5])))
    return out, scores


def test_paddle_det_mode2(tocr, cuda, tmp_path):
    n = 2
    pages = np.stack([sh.make_page(960, 960, 0x7EC00005, 40 + i) for i in range(n)])
    (tmp_path / "pages.bin").write_bytes(pages.tobytes())
    out = subprocess.run([str(mn.build()), "det2", str(tmp_path / "pages.bin"), str(n),
                          str(tmp_path)], capture_output=True, text=True, timeout=600,
                         env=dict(os.environ, GPU_CCL="2"))
    assert out.returncode == 0, out.stderr
    r = json.loads(out.stdout)
    assert r["single_same"] == 1
    for i, page in enumerate(r["pages"]):
        prob = np.fromfile(tmp_path / f"prob{i}.f32", np.float32).reshape(960, 960)
        bm = np.where(prob > np.float32(0.3), 255, 0).astype(np.uint8)
        want, want_scores = mode2_reference(tocr.lib(), rk.lib(), bm, prob, cuda)
        assert len(want) >= 10
        assert page["boxes"] == want
        assert np.allclose(page["scores"], want_scores, rtol=0, atol=1e-6)
