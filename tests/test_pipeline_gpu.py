"""End-to-end page path (config 5) on the GPU, stage by stage:

- stem (det preprocessing fused with the 3x3 s2 conv) against torch fp32;
- ink map against numpy;
- crop transforms on the device against the reference's own
  compute_crop_transform (compiled host header): bit-exact;
- ROI warp against the reference's batch_roi_warp_kernel compiled from its
  sources (fp32), bit-exact after rounding to fp16;
- a small batch through PagePipeline: DB boxes identical to the CPU
  restatement on the same probability map, crops identical to the reference
  kernel, tokens identical to the reference CTC decode of the same logits."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import ctc_oracle as co
from oracle import db_oracle as do

pytestmark = pytest.mark.gpu

REC_MEAN, REC_INV_STD = 0.5, 2.0


@pytest.fixture(autouse=True)
def _no_tf32():
    m, c = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = m, c


def pages(cuda, n, H=960, W=960, first=0):
    from turboocr_b200.pipeline import make_pages
    p = make_pages(n, H, W, first=first, device=cuda)
    torch.cuda.synchronize()
    return p


def test_pages_have_text_lines(cuda):
    p = pages(cuda, 3).cpu().numpy()
    for m in range(3):
        dark_rows = (p[m].min(axis=(1, 2)) == 0).sum()
        assert 100 < dark_rows < 960
        assert set(np.unique(p[m])) <= {0, 255}


@pytest.mark.parametrize("hw", [(960, 960), (37, 51)])
def test_stem_matches_torch(cuda, hw):
    from turboocr_b200 import pipeline as pl
    from turboocr_b200._lib import call, lib
    H, W = hw
    g = torch.Generator(device="cpu").manual_seed(H)
    x = torch.randint(0, 256, (2, H, W, 3), generator=g, dtype=torch.uint8)
    x[0] = pages(cuda, 1, H, W)[0].cpu() if H == 960 else x[0]
    xd = x.to(cuda)
    sw, sb = pl.stem_params(0x7EC00005)
    blob = np.zeros(lib().tocr_stem_params_bytes(), np.uint8)
    call("tocr_stem_pack", sw.ctypes.data, sb.ctypes.data, None, None, blob.ctypes.data, blob.nbytes)
    Ho, Wo = (H - 1) // 2 + 1, (W - 1) // 2 + 1
    out = torch.empty(2, Ho, Wo, 32, dtype=torch.float16, device=cuda)
    call("tocr_stem_f16", xd.data_ptr(), 2, H, W, H * W * 3, blob.ctypes.data,
         out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    mean = torch.tensor([0.485, 0.456, 0.406], dtype=torch.float32, device=cuda)
    inv_std = torch.tensor([1 / 0.229, 1 / 0.224, 1 / 0.225], dtype=torch.float32, device=cuda)
    xn = ((xd.float() * np.float32(1.0 / 255.0) - mean) * inv_std).permute(0, 3, 1, 2)
    ref = torch.nn.functional.conv2d(xn, torch.from_numpy(sw).to(cuda), torch.from_numpy(sb).to(cuda),
                                     stride=2, padding=1)
    ref = torch.nn.functional.hardswish(ref).permute(0, 2, 3, 1)
    torch.cuda.synchronize()
    err = (out.float() - ref).abs() - (2e-3 + 1e-3 * ref.abs())
    assert float(err.max()) <= 0, float((out.float() - ref).abs().max())
    code = C.c_int(-1)  # no bounded wait of the tensor-core stem gave up
    call("tocr_stem_take_error", C.addressof(code))
    assert code.value == 0


def test_ink_map(cuda):
    from turboocr_b200._lib import call
    p = pages(cuda, 2, first=10)
    prob = torch.empty(2, 960, 960, dtype=torch.float32, device=cuda)
    call("tocr_ink_map", p.data_ptr(), 2, 960, 960, 960 * 960 * 3, 12.0, prob.data_ptr(),
         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    pn = p.cpu().numpy().astype(np.float32)
    ink = 1.0 - pn.sum(axis=3) * np.float32(1.0 / 765.0)
    padded = np.pad(ink, ((0, 0), (0, 0), (7, 7)))
    dil = np.max(np.stack([padded[:, :, d:d + 960] for d in range(15)]), axis=0)
    ref = 1.0 / (1.0 + np.exp(-12.0 * (dil - 0.5)))
    assert np.abs(prob.cpu().numpy() - ref).max() < 1e-5


def _ref_crop(box, th=48, mw=320):
    from oracle._loader import load
    L = load("_ref/libcrop_ref.so")
    L.crop_ref_transform.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    b = np.ascontiguousarray(np.asarray(box, np.int32).reshape(8))
    m = np.zeros(9, np.float32)
    cw, v = C.c_int(), C.c_int()
    L.crop_ref_transform(b.ctypes.data, th, mw, m.ctypes.data, C.byref(cw), C.byref(v))
    return m, cw.value, v.value


def _boxes(n, seed, W=960, H=960):
    from test_crop_geom import rotated_boxes
    out = []
    for b in rotated_boxes(n, seed):
        out.append(np.clip(b, 0, [W - 1, H - 1]))
    return np.stack(out).astype(np.int32)


def test_crop_transforms_match_reference(cuda):
    from turboocr_b200._lib import call
    n_pages, max_boxes = 3, 100
    boxes = np.zeros((n_pages, max_boxes, 4, 2), np.int32)
    counts = np.array([100, 37, 0], np.int32)
    allb = _boxes(200, 11)
    boxes[0] = allb[:100]
    boxes[1, :37] = allb[100:137]
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    db, dc = d(boxes), d(counts)
    off = torch.zeros(n_pages + 1, dtype=torch.int32, device=cuda)
    minv = torch.zeros(300, 9, dtype=torch.float32, device=cuda)
    cw = torch.zeros(300, dtype=torch.int32, device=cuda)
    cp = torch.zeros(300, dtype=torch.int32, device=cuda)
    vt = torch.zeros(300, dtype=torch.int32, device=cuda)
    call("tocr_crop_transforms", db.data_ptr(), dc.data_ptr(), n_pages, max_boxes, 48, 320,
         off.data_ptr(), minv.data_ptr(), cw.data_ptr(), cp.data_ptr(), vt.data_ptr(),
         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert off.cpu().tolist() == [0, 100, 137, 137]
    minv, cw, cp, vt = minv.cpu().numpy(), cw.cpu().numpy(), cp.cpu().numpy(), vt.cpu().numpy()
    for c in range(137):
        pg, k = (0, c) if c < 100 else (1, c - 100)
        m, w, v = _ref_crop(boxes[pg, k])
        assert cw[c] == w and vt[c] == v and cp[c] == pg
        assert (minv[c].view(np.uint32) == m.view(np.uint32)).all(), (c, minv[c], m)


def test_roi_warp_matches_reference_kernel(cuda):
    from oracle import ref_kernels as rk
    from turboocr_b200._lib import call
    p = pages(cuda, 1, first=20)
    boxes = _boxes(64, 12)
    ms, ws = zip(*[(_ref_crop(b)[0], _ref_crop(b)[1]) for b in boxes])
    minv = torch.from_numpy(np.stack(ms)).to(cuda)
    cw = torch.tensor(ws, dtype=torch.int32, device=cuda)
    cpage = torch.zeros(64, dtype=torch.int32, device=cuda)
    ncr = torch.tensor([64], dtype=torch.int32, device=cuda)
    mine = torch.empty(64, 3, 48, 320, dtype=torch.float16, device=cuda)
    call("tocr_roi_warp_f16", p.data_ptr(), 960 * 960 * 3, 960, 960, 960 * 3, minv.data_ptr(),
         cw.data_ptr(), cpage.data_ptr(), ncr.data_ptr(), 64, 48, 320, None, None, 1.0 / 255.0,
         mine.data_ptr(), torch.cuda.current_stream().cuda_stream)
    ref = torch.empty(64, 3, 48, 320, dtype=torch.float32, device=cuda)
    L = rk.lib()
    L.refk_roi_warp.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_longlong, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
    assert L.refk_roi_warp(p.data_ptr(), 960, 960, 960 * 3, minv.data_ptr(), cw.data_ptr(),
                           ref.data_ptr(), 64, 48, 320, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(mine, ref.half())


def test_pipeline_small_batch(cuda):
    from turboocr_b200.pipeline import REC_T, REC_V, PagePipeline
    B = 4
    pipe = PagePipeline(cuda, B)
    p = pages(cuda, B, first=40)
    pipe.run(p)
    torch.cuda.synchronize()
    assert pipe.errors() == 0
    res = pipe.results()
    prob = pipe.prob.cpu().numpy()
    n_crops = int(pipe.crop_off[B].item())
    assert n_crops == sum(len(r) for r in res)
    for m in range(B):
        ref = do.db_postprocess(prob[m])
        assert [q for q, *_ in res[m]] == [b for b, _ in ref]
        assert 15 <= len(ref) <= 100, len(ref)
    # crops: reference kernel on page 0's crops
    from oracle import ref_kernels as rk
    k0 = len(res[0])
    ref = torch.empty(k0, 3, 48, 320, dtype=torch.float32, device=cuda)
    L = rk.lib()
    L.refk_roi_warp.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_longlong, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
    assert L.refk_roi_warp(p.data_ptr(), 960, 960, 960 * 3, pipe.minv.data_ptr(),
                           pipe.crop_w.data_ptr(), ref.data_ptr(), k0, 48, 320,
                           torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(pipe.crops[:k0], ref.half())
    # recognition: tokens of a sample of crops against the reference CTC decode
    logits = pipe.logits[:n_crops].cpu().numpy()
    flat = [(m, k) for m in range(B) for k in range(len(res[m]))]
    for c in range(0, n_crops, max(1, n_crops // 12)):
        m, k = flat[c]
        ref_toks, ref_score = co.decode_logits(logits[c], REC_V)
        assert res[m][k][2] == ref_toks
        assert abs(res[m][k][3] - ref_score) <= 1e-3


def test_detection_half_matches_the_full_run(cuda):
    """run(rec=False) (the bench's det_only figure) enqueues the same
    detection stages: boxes, scores, crop transforms and crops identical to
    a full run's, and no recognition output written."""
    from turboocr_b200.pipeline import PagePipeline
    B = 2
    p = pages(cuda, B, first=7)
    full = PagePipeline(cuda, B)
    full.run(p)
    det = PagePipeline(cuda, B)
    det.lengths.fill_(-7)
    det.run(p, rec=False)
    torch.cuda.synchronize()
    assert full.errors() == 0 and det.errors() == 0
    n = int(full.crop_off[B].item())
    assert n > 0 and int(det.crop_off[B].item()) == n
    for a, b in ((full.db.boxes, det.db.boxes), (full.db.scores, det.db.scores),
                 (full.db.counts, det.db.counts), (full.minv[:n], det.minv[:n]),
                 (full.crops[:n], det.crops[:n])):
        assert torch.equal(a, b)
    assert bool((det.lengths == -7).all())
