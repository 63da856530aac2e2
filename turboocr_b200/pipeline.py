"""End-to-end det+rec page path on one GPU.

Per batch of same-size u8 HWC pages, all on one stream, no host round trip:

  stem      det preprocessing (scale 1) fused with a 3x3 s2 conv 3->32 (+BN, hardswish)
  blocks    8 fused DW3x3+PW1x1 INT8 blocks on tcgen05, channels 32->64->128->256:
            (32,64,s1) (64,64,s2) (64,128,s1) (128,128,s2) (128,128,s1)
            (128,128,s2) (128,128,s1) (128,256,s1)  -> 60x60x256 at 960x960 input
  head      1x1 256->1 + sigmoid (the det head's logit map)
  ink map   the DB probability map of the synthetic run (trained DB heads are
            not available; random-weight backbones produce no text regions)
  DB        tocr_db_postprocess (extract_boxes_from_bitmap on the device)
  crops     compute_crop_transform + batch_roi_warp to 48x320 fp16
  rec       stand-in recognition logits per crop (T=80, V=18385; the rec
            network is out of scope), then the fused CTC decode

The reference runs the same stages in src/pipeline/ocr/ocr_pipeline_run.cpp
(det: paddle_det.cpp, post: det_postprocess.cpp, crops + rec:
paddle_rec.cpp) with TensorRT networks and a host-side crop/CTC loop.
"""
from __future__ import annotations

import numpy as np
import torch

from . import backbone as bb
from ._lib import call, lib, synth
from .kernels import DbPostprocess, _ptr, _stream

SCHEDULE = [(32, 64, 1), (64, 64, 2), (64, 128, 1), (128, 128, 2),
            (128, 128, 1), (128, 128, 2), (128, 128, 1), (128, 256, 1)]
REC_H, REC_W, REC_T, REC_V = 48, 320, 80, 18385
INK_GAIN = 12.0


def stem_params(seed: int):
    """BN-folded 3x3 conv 3->32 (weights N(0, 0.2), BN as backbone._bn)."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.2, (32, 3, 3, 3))
    s, b = bb._bn(rng, 32)
    return (w * s[:, None, None, None]).astype(np.float32), b.astype(np.float32)


def out_hw(h, w, s):
    return (h - 1) // s + 1, (w - 1) // s + 1


class PagePipeline:
    def __init__(self, device, batch: int, H: int = 960, W: int = 960, max_boxes: int = 128,
                 seed: int = 0x7EC00005, point_cap: int = 0, offset_cap: int = 0):
        self.device, self.B, self.H, self.W = device, batch, H, W
        self.max_boxes, self.seed = max_boxes, seed
        L = lib()
        sw, sb = stem_params(seed)
        blob = np.zeros(L.tocr_stem_params_bytes(), np.uint8)
        call("tocr_stem_pack", sw.ctypes.data, sb.ctypes.data, None, None, blob.ctypes.data,
             blob.nbytes)
        self.stem_w, self.stem_b = sw, sb
        self.stem_blob = blob  # host blob: the kernel takes the parameters by value
        self.blocks = []
        h, w = out_hw(H, W, 2)
        self.acts = [torch.empty(batch, h, w, 32, dtype=torch.float16, device=device)]
        for i, (c, co, s) in enumerate(SCHEDULE):
            blk = bb.DwPwBlock(bb.make_block_params(c, co, seed + 1 + i), bb.KIND_INT8, s, device)
            self.blocks.append(blk)
            h, w = out_hw(h, w, s)
            self.acts.append(torch.empty(batch, h, w, co, dtype=torch.float16, device=device))
        rng = np.random.default_rng(seed + 100)
        self.head_w = torch.from_numpy(rng.normal(0, 0.05, 256).astype(np.float32)).to(device)
        self.head_b = float(rng.normal(0, 0.1))
        self.head_map = torch.empty(batch, h, w, dtype=torch.float32, device=device)
        self.prob = torch.empty(batch, H, W, dtype=torch.float32, device=device)
        if point_cap <= 0:
            point_cap = batch * 65536
        if offset_cap <= 0:  # text-line rings: about 1 MB of unclip scratch per page
            offset_cap = batch * 16384
        self.db = DbPostprocess(batch, H, W, device, max_boxes=max_boxes, point_cap=point_cap,
                                offset_cap=offset_cap)
        nc = batch * max_boxes
        self.max_crops = nc
        self.crop_off = torch.zeros(batch + 1, dtype=torch.int32, device=device)
        self.minv = torch.zeros(nc, 9, dtype=torch.float32, device=device)
        self.crop_w = torch.zeros(nc, dtype=torch.int32, device=device)
        self.crop_page = torch.zeros(nc, dtype=torch.int32, device=device)
        self.vertical = torch.zeros(nc, dtype=torch.int32, device=device)
        self.crops = torch.empty(nc, 3, REC_H, REC_W, dtype=torch.float16, device=device)
        self.logits = torch.empty(nc, REC_T, REC_V, dtype=torch.float16, device=device)
        self.tokens = torch.zeros(nc * REC_T, dtype=torch.int32, device=device)
        self.lengths = torch.zeros(nc, dtype=torch.int32, device=device)
        self.line_scores = torch.zeros(nc, dtype=torch.float32, device=device)
        self.step_idx = torch.empty(nc * REC_T, dtype=torch.int32, device=device)
        self.step_prob = torch.empty(nc * REC_T, dtype=torch.float32, device=device)
        # kernels launched per run() (for the bench's gpu_launches count)
        # stem + blocks + head + ink + DB (16 kernels) + crops (2) + warp
        # + stand-in rec logits (2) + CTC (2)
        self.launches_per_run = 1 + len(SCHEDULE) + 1 + 1 + 16 + 2 + 1 + 2 + 2

    def run(self, pages: torch.Tensor, stream=None, rec: bool = True) -> None:
        """Enqueue the whole path for pages u8 [B, H, W, 3] (device). rec=False
        stops after the crops (the detection half: no stand-in rec logits and
        no CTC decode)."""
        B, H, W = self.B, self.H, self.W
        assert pages.shape == (B, H, W, 3) and pages.dtype == torch.uint8
        st = _stream(stream)
        page_stride = H * W * 3
        call("tocr_stem_f16", _ptr(pages), B, H, W, page_stride, self.stem_blob.ctypes.data,
             _ptr(self.acts[0]), st)
        for i, blk in enumerate(self.blocks):
            x, y = self.acts[i], self.acts[i + 1]
            n, h, w, c = x.shape
            call("tocr_dwpw_block", _ptr(x), _ptr(y), n, h, w, blk.C, blk.CO, blk.stride, blk.kind,
                 _ptr(blk.blob), _ptr(blk.err), st)
        last = self.acts[-1]
        call("tocr_head_sigmoid", _ptr(last), last.shape[0] * last.shape[1] * last.shape[2],
             last.shape[3], _ptr(self.head_w), self.head_b, _ptr(self.head_map), st)
        call("tocr_ink_map", _ptr(pages), B, H, W, page_stride, INK_GAIN, _ptr(self.prob), st)
        self.db(self.prob, stream=stream)
        call("tocr_crop_transforms", _ptr(self.db.boxes), _ptr(self.db.counts), B, self.max_boxes,
             REC_H, REC_W, _ptr(self.crop_off), _ptr(self.minv), _ptr(self.crop_w),
             _ptr(self.crop_page), _ptr(self.vertical), st)
        n_crops = self.crop_off[B:]
        call("tocr_roi_warp_f16", _ptr(pages), page_stride, H, W, W * 3, _ptr(self.minv),
             _ptr(self.crop_w), _ptr(self.crop_page), _ptr(n_crops), self.max_crops, REC_H, REC_W,
             None, None, 1.0 / 255.0, _ptr(self.crops), st)
        if not rec:
            return
        synth().tocr_synth_rec_logits(_ptr(self.logits), _ptr(n_crops), self.max_crops, REC_T,
                                      REC_V, self.seed, st)
        call("tocr_ctc_greedy_f16_dev", _ptr(self.logits), _ptr(n_crops), self.max_crops, REC_T,
             REC_V, REC_V, _ptr(self.tokens), _ptr(self.lengths), _ptr(self.line_scores),
             _ptr(self.step_idx), _ptr(self.step_prob), st)

    def errors(self) -> int:
        """Non-zero when a tensor-core kernel of the path gave up a bounded
        wait (DW+PW blocks, stem); synchronises."""
        import ctypes as C
        code = C.c_int(0)
        call("tocr_stem_take_error", C.addressof(code))
        return int(sum(int(b.err.item()) for b in self.blocks)) + int(code.value)

    def results(self):
        """Per page: list of (quad, box score, token ids, line score) (synchronises)."""
        dets = self.db.results()
        off = self.crop_off.cpu().tolist()
        lens = self.lengths.cpu().tolist()
        scs = self.line_scores.cpu().tolist()
        toks = self.tokens.view(self.max_crops, REC_T).cpu()
        out = []
        for p in range(self.B):
            page = []
            for k, (quad, score) in enumerate(dets[p]):
                c = off[p] + k
                page.append((quad, score, toks[c, : lens[c]].tolist(), scs[c]))
            out.append(page)
        return out


def shard(total: int, world: int, rank: int, micro_batch: int = 16) -> tuple[int, int]:
    """Contiguous page shard of one rank: (first page, page count). The job is
    split evenly (rounded up to whole micro-batches); pages are independent,
    so ranks never exchange data (config 5: no cross-GPU reduction)."""
    per = (total + world - 1) // world
    per = (per + micro_batch - 1) // micro_batch * micro_batch
    first = min(total, rank * per)
    return first, max(0, min(per, total - first))


def make_pages(n: int, H: int = 960, W: int = 960, seed: int = 0x7EC00005, first: int = 0,
               device="cuda", stream=None) -> torch.Tensor:
    pages = torch.empty(n, H, W, 3, dtype=torch.uint8, device=device)
    st = _stream(stream)
    rc = synth().tocr_synth_pages(_ptr(pages), n, H, W, seed, first, st)
    if rc != 0:
        raise RuntimeError("tocr_synth_pages failed")
    return pages
