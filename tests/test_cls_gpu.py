"""The angle classifier (PaddleCls, src/classification/paddle_cls.cpp:43-103)
on the GPU: its network (stem, five DW+PW INT8 blocks, pool + FC + softmax,
synthetic seeded weights) against a torch fp32 restatement with the
dequantised PW weights, and the C++ module (tests/native/modules_test.cpp)
against the same network driven from here: identical scores, the reference's
flip rule (score_180 > score_0 and > 0.9 rotates the corners by two), and the
pipeline's vertical-box gate (ocr_pipeline_runtime.cpp:87-118)."""
import json
import subprocess

import numpy as np
import pytest
import torch

import modules_native as mn
from oracle._crop import crop_transform_full
from oracle import synth_host as sh
from turboocr_b200 import backbone as bb

pytestmark = pytest.mark.gpu

SEED = 0x7EC0C150
BLOCKS = [(32, 64, 1, 0.48), (64, 64, 2, 0.34), (64, 128, 1, 0.34), (128, 128, 2, 0.24),
          (128, 256, 1, 0.24)]
H, W = 80, 160
SCORE_TOL = 3e-2  # softmax probabilities, device (INT8 blocks, fp16 activations) vs fp32


def synth(L, k, scale, n):
    out = np.empty(n, np.float32)
    assert L.tocr_synth_weights(SEED + k, scale, out.ctypes.data, n) == 0
    return out


class Net:
    """The synthetic classifier network: device chain and torch reference."""

    def __init__(self, L, dev):
        self.L, self.dev = L, dev
        self.stem_w = synth(L, 0, 0.53, 32 * 27)
        self.stem_b = synth(L, 1, 0.1, 32)
        self.blocks = []
        for j, (c, co, s, pws) in enumerate(BLOCKS):
            p = bb.BlockParams(wdw=synth(L, 16 + 4 * j, 0.9, c * 9).reshape(c, 3, 3),
                               bdw=synth(L, 17 + 4 * j, 0.1, c),
                               wpw=synth(L, 18 + 4 * j, pws, co * c).reshape(co, c),
                               bpw=synth(L, 19 + 4 * j, 0.1, co))
            self.blocks.append((bb.DwPwBlock(p, bb.KIND_INT8, s, dev), p, s))
        self.head_w = synth(L, 64, 1.0, 2 * 256)
        self.head_b = synth(L, 65, 0.1, 2)
        t = lambda a: torch.from_numpy(a).to(dev)
        self.d = [t(a) for a in (self.stem_w, self.stem_b, self.head_w, self.head_b)]

    def device(self, crops):
        n = crops.shape[0]
        x = torch.empty(n, H // 2, W // 2, 32, dtype=torch.float16, device=self.dev)
        st = torch.cuda.current_stream().cuda_stream
        assert self.L.tocr_cls_stem_f16(crops.data_ptr(), n, H, W, self.d[0].data_ptr(),
                                        self.d[1].data_ptr(), x.data_ptr(), st) == 0
        for blk, _, _ in self.blocks:
            x = blk(x)
        scores = torch.empty(n, 2, dtype=torch.float32, device=self.dev)
        assert self.L.tocr_cls_head_f32(x.data_ptr(), n, x.shape[1] * x.shape[2], 256,
                                        self.d[2].data_ptr(), self.d[3].data_ptr(),
                                        scores.data_ptr(), st) == 0
        torch.cuda.synchronize()
        return scores.cpu().numpy()

    def reference(self, crops):
        F = torch.nn.functional
        x = crops.float()
        w = torch.from_numpy(self.stem_w.reshape(32, 3, 3, 3)).to(self.dev)
        y = F.hardswish(F.conv2d(x, w, torch.from_numpy(self.stem_b).to(self.dev), stride=2,
                                 padding=1))
        y = y.permute(0, 2, 3, 1)
        for blk, p, s in self.blocks:
            y = bb.reference_block(y, p, s, blk.dequantized_pw())
        m = y.mean(dim=(1, 2))
        logits = m @ torch.from_numpy(self.head_w.reshape(2, 256)).to(self.dev).T
        logits = logits + torch.from_numpy(self.head_b).to(self.dev)
        return torch.softmax(logits, dim=1).cpu().numpy()


def crops_of(L, page_dev, boxes, dev):
    n = len(boxes)
    minv = np.zeros((n, 9), np.float32)
    cw = np.zeros(n, np.int32)
    for k, q in enumerate(boxes):
        m, w, _ = crop_transform_full(q, H, W)
        minv[k], cw[k] = m, w
    d_minv, d_cw = torch.from_numpy(minv).to(dev), torch.from_numpy(cw).to(dev)
    page_idx = torch.zeros(n, dtype=torch.int32, device=dev)
    n_dev = torch.tensor([n], dtype=torch.int32, device=dev)
    out = torch.empty(n, 3, H, W, dtype=torch.float16, device=dev)
    assert L.tocr_roi_warp_f16(page_dev.data_ptr(), 0, 960, 960, 960 * 3, d_minv.data_ptr(),
                               d_cw.data_ptr(), page_idx.data_ptr(), n_dev.data_ptr(), n, H, W,
                               None, None, 1.0 / 255.0, out.data_ptr(),
                               torch.cuda.current_stream().cuda_stream) == 0
    return out


def rotated(b):
    return [b[2], b[3], b[0], b[1]]


def vertical(b):
    w = max(abs(b[1][0] - b[0][0]), abs(b[2][0] - b[3][0]))
    h = max(abs(b[3][1] - b[0][1]), abs(b[2][1] - b[1][1]))
    return h * h >= w * w * 225 // 100


@pytest.fixture(scope="module")
def cls_run(tmp_path_factory):
    d = tmp_path_factory.mktemp("cls")
    page = sh.make_page(960, 960, 0x7EC00005, 77)
    (d / "page.bin").write_bytes(page.tobytes())
    out = subprocess.run([str(mn.build()), "cls", str(d / "page.bin"), str(d)],
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    return json.loads(out.stdout), page


def test_cls_network_matches_fp32_reference(tocr, cuda, cls_run):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    r, page = cls_run
    net = Net(tocr.lib(), cuda)
    crops = crops_of(tocr.lib(), torch.from_numpy(page).to(cuda), r["in"], cuda)
    got = net.device(crops)
    want = net.reference(crops)
    assert np.abs(got - want).max() <= SCORE_TOL, np.abs(got - want).max()
    assert np.allclose(got.sum(1), 1.0, atol=1e-6)


def test_paddle_cls_module(tocr, cuda, cls_run):
    r, page = cls_run
    boxes_in, boxes_out, gated = r["in"], r["out"], r["gated"]
    scores = np.array(r["scores"], np.float32)
    assert len(boxes_in) == len(boxes_out) == len(scores) >= 20
    net = Net(tocr.lib(), cuda)
    crops = crops_of(tocr.lib(), torch.from_numpy(page).to(cuda), boxes_in, cuda)
    assert np.array_equal(net.device(crops), scores)  # the module runs the same kernels
    flips = 0
    for b_in, b_out, g, (s0, s180) in zip(boxes_in, boxes_out, gated, scores):
        flip = s180 > s0 and s180 > np.float32(0.9)
        flips += flip
        assert b_out == (rotated(b_in) if flip else b_in)
        assert g == (b_out if vertical(b_in) else b_in)
    assert 0 < flips < len(boxes_in)
    assert sum(vertical(b) for b in boxes_in) >= 12
