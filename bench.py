"""Benchmark of the B200 det+rec hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W] [--impl b200|reference]

Under torchrun (N > 1) every rank owns one GPU and an independent shard of
the work (pages are independent: no collective on the data path); the timed
region is bracketed by a barrier + device synchronise and the reported time
is the maximum over ranks.

Workloads:
  e2e         config 5 (default, the headline): 4096 960x960 pages split over the
              ranks, det + rec path per page (pipeline.PagePipeline)
  ctc         config 2: 512 lines x 80 steps x 18385-class fp16 logits per GPU
  preprocess  config 3: 256 u8 HWC images (sides 600..2000) -> fp16 960x960 NCHW
  dwpw        config 4: fused DW3x3+PW1x1 block, 32 x 240 x 240 x 128 -> 256, INT8
  db          config 1: DB post-process of 8 fp32 960x960 probability maps
  rec_head    the recognizer's CTC head (K=128 -> 18385 classes) fused with the
              greedy decode on tcgen05, 8192 lines x 80 steps per GPU
  db_head     the det network's DB head (FPN neck + binarisation head) on the
              /4, /8, /16 features of 32 pages of 960x960
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MEASURED = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TFLOPS = 1590.0


def tensor_peak():
    """Dense fp16/bf16 tensor peak: the measured cuBLAS burst figure."""
    if MEASURED.exists():
        try:
            return float(json.loads(MEASURED.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return FALLBACK_TFLOPS, "fallback"


def hbm_peak():
    if MEASURED.exists():
        try:
            return float(json.loads(MEASURED.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- workloads ----
class CtcWorkload:
    """fused CTC greedy decode of fp16 logits."""
    name = "ctc_greedy_512x80x18385_fp16"
    # DRAM read+write bytes per line of ctc_rows_f16_kernel: one ncu capture
    # (dram__bytes_read.sum + dram__bytes_write.sum) of a 64-line case, scaled
    traffic_per_unit = (188_710_912 + 3_741_184) / 64
    traffic_source = "ncu dram__bytes_read/write.sum, 64-line capture scaled per line"
    metric = "lines/sec CTC greedy decode (512x80x18385 fp16 logits)"
    unit = "lines/s"
    dtype = "f16"
    B, T, V = 512, 80, 18385
    default_units = B

    def __init__(self, dev, seed, units=None):
        from turboocr_b200 import kernels as K
        from turboocr_b200._lib import synth
        self.K = K
        self.dev = dev
        if units:
            self.B = units
            self.units_per_step = units
            self.algo_bytes = units * self.T * self.V * 2
        self.x = torch.empty(self.B, self.T, self.V, dtype=torch.float16, device=dev)
        self.plan = torch.empty(self.B * self.T, dtype=torch.int32, device=dev)
        assert synth().tocr_synth_ctc_logits(self.x.data_ptr(), self.plan.data_ptr(), self.B,
                                             self.T, self.V, seed, None) == 0
        self.out = K.CtcOutputs(self.B, self.T, dev)
        torch.cuda.synchronize()

    units_per_step = B
    launches_per_step = 2
    algo_bytes = B * T * V * 2  # logits read once
    l2_note = "inputs 1.51 GB > 126 MB L2 (no flush needed)"

    def step(self):
        self.K.ctc_greedy_f16(self.x, self.V, self.out)

    def dominant_kernel_ms(self, iters=10):
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            self.step()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    # end-to-end: pinned host logits -> H2D -> decode -> D2H of tokens/scores
    def setup_e2e(self):
        self.h_x = torch.empty(self.x.shape, dtype=torch.float16, pin_memory=True)
        self.h_x.copy_(self.x)
        self.h_tok = torch.empty(self.B * self.T, dtype=torch.int32, pin_memory=True)
        self.h_len = torch.empty(self.B, dtype=torch.int32, pin_memory=True)
        self.h_sc = torch.empty(self.B, dtype=torch.float32, pin_memory=True)
        self.h2d = self.h_x.numel() * 2
        self.d2h = self.h_tok.numel() * 4 + self.B * 8

    def e2e_step(self):
        self.x.copy_(self.h_x, non_blocking=True)
        self.K.ctc_greedy_f16(self.x, self.V, self.out)
        self.h_tok.copy_(self.out.tokens, non_blocking=True)
        self.h_len.copy_(self.out.lengths, non_blocking=True)
        self.h_sc.copy_(self.out.scores, non_blocking=True)

class PreprocessWorkload:
    """batched resize/letterbox/normalise to fp16 NCHW."""
    name = "preprocess_256img_600-2000_to_960x960_f16"
    # DRAM bytes per image of preprocess_batch_kernel (32-image ncu capture, scaled;
    # part of the output is still in L2 when that short launch ends)
    traffic_per_unit = (160_950_016 + 131_166_976) / 32
    traffic_source = "ncu dram__bytes_read/write.sum, 32-image capture scaled per image"
    metric = "images/sec batched det preprocessing (256 u8 images -> fp16 960x960 NCHW)"
    unit = "images/s"
    dtype = "f32"
    N, H, W = 256, 960, 960
    default_units = N
    launches_per_step = 1
    l2_note = "inputs 1.3 GB + outputs 1.4 GB > 126 MB L2 (no flush needed)"

    def __init__(self, dev, seed, units=None):
        from turboocr_b200 import kernels as K
        from turboocr_b200._lib import synth
        self.K = K
        if units:
            self.N = units
        lib = synth()
        dims = []
        for i in range(self.N):
            h = 600 + int(lib.tocr_synth_hash(seed, 2000 + i, 0) >> 32) % 1401
            w = 600 + int(lib.tocr_synth_hash(seed, 2000 + i, 1) >> 32) % 1401
            dims.append((h, w))
        self.dims = dims
        sizes = [h * w * 3 for h, w in dims]
        offs = np.concatenate([[0], np.cumsum([(s + 255) // 256 * 256 for s in sizes])])
        self.src = torch.empty(int(offs[-1]), dtype=torch.uint8, device=dev)
        assert lib.tocr_synth_fill_u8(self.src.data_ptr(), self.src.numel(), seed, 3, None) == 0
        base = self.src.data_ptr()
        content = [det_resize_max960(h, w) for h, w in dims]
        self.content = content
        self.meta = K.PreprocessMeta([base + int(o) for o in offs[:-1]], [w * 3 for _, w in dims],
                                     dims, content, dev)
        self.out = torch.empty(self.N, 3, self.H, self.W, dtype=torch.float16, device=dev)
        self.units_per_step = self.N
        self.algo_bytes = touched_source_bytes(dims, content) + self.N * 3 * self.H * self.W * 2
        self.offs = offs
        torch.cuda.synchronize()

    def step(self):
        self.K.preprocess_batch(self.meta, self.out)

    def dominant_kernel_ms(self, iters=10):
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            self.step()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    def setup_e2e(self):
        self.h_src = torch.empty(self.src.numel(), dtype=torch.uint8, pin_memory=True)
        self.h_src.copy_(self.src)
        self.h_out = torch.empty(self.out.shape, dtype=torch.float16, pin_memory=True)
        self.h2d = int(sum(h * w * 3 for h, w in self.dims))
        self.d2h = self.h_out.numel() * 2

    def e2e_step(self):
        self.src.copy_(self.h_src, non_blocking=True)
        self.K.preprocess_batch(self.meta, self.out)
        self.h_out.copy_(self.out, non_blocking=True)

class DwPwWorkload:
    """fused DW3x3 + PW1x1 block, INT8 PW weights on tcgen05."""
    name = "dwpw_block_32x128x240x240_to_256_int8"
    # DRAM bytes per image of dwpw_kernel (8-image ncu capture, scaled; part of
    # the output is still in L2 when that short launch ends)
    traffic_per_unit = (118_064_128 + 177_737_728) / 8
    traffic_source = "ncu dram__bytes_read/write.sum, 8-image capture scaled per image"
    metric = "images/sec fused dw3x3+pw1x1 block (32x128x240x240 fp16 -> 256ch, INT8 PW)"
    unit = "images/s"
    dtype = "i8 (PW on tcgen05 kind::i8, DW fp16x2)"
    N, H, W, C, CO = 32, 240, 240, 128, 256
    default_units = N
    launches_per_step = 1
    l2_note = "input 472 MB + output 944 MB per step > 126 MB L2 (no flush needed)"
    kind = 0

    def __init__(self, dev, seed, units=None):
        from turboocr_b200 import backbone as bb
        if units:
            self.N = units
        self.bb = bb
        self.params = bb.make_block_params(self.C, self.CO, 0x7EC00004)
        self.blk = bb.DwPwBlock(self.params, self.kind, 1, dev)
        g = torch.Generator(device=dev).manual_seed(seed)
        self.x = torch.randn(self.N, self.H, self.W, self.C, generator=g, device=dev).to(torch.float16)
        self.y = torch.empty(self.N, self.H, self.W, self.CO, dtype=torch.float16, device=dev)
        self.units_per_step = self.N
        px = self.N * self.H * self.W
        self.algo_bytes = px * self.C * 2 + px * self.CO * 2 + self.blk.blob.numel()
        self.algo_flops = 2 * px * self.C * (9 + self.CO)
        torch.cuda.synchronize()

    def step(self):
        self.blk(self.x, self.y)

    def dominant_kernel_ms(self, iters=10):
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            self.step()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    def setup_e2e(self):
        self.h_x = torch.empty(self.x.shape, dtype=torch.float16, pin_memory=True)
        self.h_x.copy_(self.x)
        self.h_y = torch.empty(self.y.shape, dtype=torch.float16, pin_memory=True)
        self.h2d = self.h_x.numel() * 2
        self.d2h = self.h_y.numel() * 2

    def e2e_step(self):
        self.x.copy_(self.h_x, non_blocking=True)
        self.blk(self.x, self.y)
        self.h_y.copy_(self.y, non_blocking=True)

class RecHeadWorkload:
    """The recognizer's CTC head (fp16 features [lines*80][128] x weights
    [18385][128] + bias) fused with the greedy decode on tcgen05
    (tocr_rec_head_ctc_f16): the logits are formed and reduced on the SM."""
    name = "rec_head_ctc_8192x80_k128_v18385"
    metric = "lines/sec recognizer CTC head + greedy decode (80 steps, K=128, V=18385)"
    unit = "lines/s"
    dtype = "f16 operands, f32 accumulate (tcgen05 kind::f16)"
    bound = "tensor"
    B, T, K, V = 8192, 80, 128, 18385
    default_units = B
    launches_per_step = 2
    l2_note = "features 168 MB per step > 126 MB L2 (no flush needed); weights 4.7 MB stay in L2"
    dominant = "rec_head_kernel + ctc_collapse_kernel per launch"

    def __init__(self, dev, seed, units=None):
        L = __import__("turboocr_b200").lib()
        self.L = L
        if units:
            self.B = units
        rows = self.B * self.T
        g = torch.Generator(device=dev).manual_seed(seed)
        self.feat = torch.randn(rows, self.K, generator=g, device=dev).to(torch.float16)
        self.w = (torch.randn(self.V, self.K, generator=g, device=dev) *
                  (3.0 / self.K ** 0.5)).to(torch.float16)
        self.bias = torch.randn(self.V, generator=g, device=dev) * 0.5
        self.toks = torch.empty(rows, dtype=torch.int32, device=dev)
        self.lens = torch.empty(self.B, dtype=torch.int32, device=dev)
        self.sc = torch.empty(self.B, dtype=torch.float32, device=dev)
        self.sidx = torch.empty(rows, dtype=torch.int32, device=dev)
        self.sprob = torch.empty(rows, dtype=torch.float32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.units_per_step = self.B
        self.algo_bytes = rows * self.K * 2 + self.V * self.K * 2 + self.V * 4 + rows * 4 + self.B * 8
        self.algo_flops = 2 * rows * self.K * self.V
        torch.cuda.synchronize()

    def step(self):
        st = self.L.tocr_rec_head_ctc_f16(
            self.feat.data_ptr(), self.B, self.T, self.K, self.w.data_ptr(), self.bias.data_ptr(),
            self.V, self.V - 2, self.toks.data_ptr(), self.lens.data_ptr(), self.sc.data_ptr(),
            self.sidx.data_ptr(), self.sprob.data_ptr(), self.err.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
        assert st == 0, self.L.tocr_last_error_string()

    def dominant_kernel_ms(self, iters=10):
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            self.step()
        e1.record(s)
        torch.cuda.synchronize()
        assert int(self.err.item()) == 0
        return e0.elapsed_time(e1) / iters

    def setup_e2e(self):
        self.h_feat = torch.empty(self.feat.shape, dtype=torch.float16, pin_memory=True)
        self.h_feat.copy_(self.feat)
        self.h_tok = torch.empty(self.toks.shape, dtype=torch.int32, pin_memory=True)
        self.h_len = torch.empty(self.B, dtype=torch.int32, pin_memory=True)
        self.h_sc = torch.empty(self.B, dtype=torch.float32, pin_memory=True)
        self.h2d = self.h_feat.numel() * 2
        self.d2h = self.h_tok.numel() * 4 + self.B * 8

    def e2e_step(self):
        self.feat.copy_(self.h_feat, non_blocking=True)
        self.step()
        self.h_tok.copy_(self.toks, non_blocking=True)
        self.h_len.copy_(self.lens, non_blocking=True)
        self.h_sc.copy_(self.sc, non_blocking=True)


class DbHeadWorkload:
    """The det network's DB head (FPN neck over the /4, /8, /16 backbone
    levels + binarisation head, turboocr_b200/dbhead.py) on 32 pages of
    960x960: features c2 [32][240][240][128], c3 [32][120][120][128],
    c4 [32][60][60][256] fp16 -> probability maps [32][960][960] fp32."""
    name = "db_head_32x960x960"
    metric = "pages/sec DB head (FPN + binarisation head, 960x960 pages)"
    unit = "pages/s"
    dtype = "f16 operands, f32 accumulate (tcgen05 kind::f16); fp32 probability map"
    N = 32
    default_units = N
    launches_per_step = 9
    bound = "tensor"
    l2_note = "features 648 MB + maps 118 MB per step > 126 MB L2 (no flush needed)"
    dominant = ("the 9 launches of one DB head pass (achieved = useful flops of its 7 "
                "tensor-core convolutions / the pass time)")

    def __init__(self, dev, seed, units=None):
        from turboocr_b200 import dbhead
        if units:
            self.N = units
        n = self.N
        g = torch.Generator(device=dev).manual_seed(seed)
        mk = lambda *s: torch.randn(*s, generator=g, device=dev).to(torch.float16)
        self.c2, self.c3, self.c4 = mk(n, 240, 240, 128), mk(n, 120, 120, 128), mk(n, 60, 60, 256)
        self.head = dbhead.DbHead(dev)
        self.units_per_step = n
        feat = sum(t.numel() * 2 for t in (self.c2, self.c3, self.c4))
        self.algo_bytes = feat + n * 960 * 960 * 4  # features read once, map written once
        # useful multiply-adds of the tensor-core convolutions (unpadded K, N)
        px4, px8, px16 = 240 * 240, 120 * 120, 60 * 60
        self.algo_flops = 2 * n * (px16 * 256 * 96 + px8 * 128 * 96 + px4 * 128 * 96 +
                                   (px16 + px8 + px4) * 864 * 24 + px4 * 648 * 24)
        self.head(self.c2, self.c3, self.c4)
        torch.cuda.synchronize()

    def step(self):
        self.head(self.c2, self.c3, self.c4)

    def dominant_kernel_ms(self, iters=10):
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            self.step()
        e1.record(s)
        torch.cuda.synchronize()
        assert int(self.head.err.item()) == 0
        return e0.elapsed_time(e1) / iters

    def setup_e2e(self):
        self.h_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in
                     (self.c2, self.c3, self.c4)]
        for h, d in zip(self.h_in, (self.c2, self.c3, self.c4)):
            h.copy_(d)
        self.h_prob = torch.empty((self.N, 960, 960), dtype=torch.float32, pin_memory=True)
        self.h2d = sum(t.numel() * 2 for t in self.h_in)
        self.d2h = self.h_prob.numel() * 4

    def e2e_step(self):
        for h, d in zip(self.h_in, (self.c2, self.c3, self.c4)):
            d.copy_(h, non_blocking=True)
        prob = self.head(self.c2, self.c3, self.c4)
        self.h_prob.copy_(prob, non_blocking=True)


class PngWorkload:
    """PNG decode to device BGR (turboocr_b200/decode.py, csrc/png.cu): 512
    document pages of 1240x1754 (A4 at 150 dpi) as OpenCV's PNG writer
    encodes them (turboocr_b200/pagegen.py), one batch per step. A file's
    DEFLATE stream is decoded by one serial chain (two warps), so a batch
    needs several files per SM to fill the GPU: 512 keeps about 3.5 on each
    of the 148 SMs; the 64-page batch is reported beside it. Device arm: the
    compressed files resident in HBM -> BGR u8 pages; e2e: host bytes ->
    pinned staging -> H2D -> decode -> per-page status back."""
    name = "png_decode_512xA4"
    metric = "pages/sec PNG decode to device BGR (1240x1754 document pages)"
    unit = "pages/s"
    dtype = "u8 (DEFLATE + PNG filters, integer)"
    N = 512
    default_units = N
    launches_per_step = 3
    bound = "hbm"
    l2_note = ("per step: 189 MB of files, 3.4 GB of scanlines and 3.3 GB of pixels "
               "written and read once > 126 MB L2 (no flush needed)")
    dominant = ("the 3 launches of one decode (parse, inflate, unfilter); achieved = files "
                "read + pixels written per decode / its time")

    def __init__(self, dev, seed, units=None):
        from turboocr_b200 import decode as D, pagegen
        if units:
            self.N = units
        self.files = pagegen.png_pages(self.N, seed)
        self.dec = D.PngBatchDecoder(dev)
        out = self.dec.decode(self.files)  # sizes the buffers, checks the statuses
        assert all(s == D.PNG_OK for s in out.status), out.status
        jobs, ok, self.nsrc, self.nscr, self.ndst = self.dec.plan(self.files)
        self.d_in = self.dec._bufs["d_src"]
        self.jo = (self.nsrc + 15) & ~15
        self.units_per_step = self.N
        self.algo_bytes = self.nsrc + sum(int(j["height"]) * 3 * int(j["width"]) for j in jobs)
        self.status = torch.zeros(self.N, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()

    def step(self):
        from turboocr_b200._lib import call
        s = torch.cuda.current_stream()
        call("tocr_png_decode_batch", self.d_in.data_ptr(), self.d_in.data_ptr() + self.jo,
             self.N, self.dec._bufs["dst"].data_ptr(), self.dec._bufs["scratch"].data_ptr(),
             self.status.data_ptr(), s.cuda_stream)

    def dominant_kernel_ms(self, iters=5):
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            self.step()
        e1.record(s)
        torch.cuda.synchronize()
        assert int((self.status != 0).sum()) == 0
        return e0.elapsed_time(e1) / iters

    def setup_e2e(self):
        self.h2d = self.nsrc + self.N * 48
        self.d2h = self.N * 4

    def e2e_step(self):
        self.dec.decode(self.files)


def det_resize_max960(h, w):
    """compute_det_resize with {"max", 960, 960} (det_config.h:58-81), as the
    library computes it (config 3's DET_LIMIT_TYPE=max, 960, 960)."""
    from turboocr_b200.det_config import DetResizeParams, compute_det_resize
    return compute_det_resize(h, w, DetResizeParams("max", 960, 960))


def touched_source_bytes(dims, content):
    """Exact distinct source bytes the bilinear taps touch (preprocess_kernels.cu:19-54)."""
    total = 0
    for (h, w), (ch, cw) in zip(dims, content):
        def taps(n_src, n_dst):
            s = np.float32(n_src) / np.float32(n_dst)
            d = np.arange(n_dst, dtype=np.float32)
            sx = (d + np.float32(0.5)) * s - np.float32(0.5)
            x0 = np.floor(sx).astype(np.int64)
            x1 = np.clip(x0 + 1, 0, n_src - 1)
            x0 = np.clip(x0, 0, n_src - 1)
            return len(np.union1d(x0, x1))
        total += taps(h, ch) * taps(w, cw) * 3
    return total


class DbWorkload:
    """DB post-process of 8 fp32 probability maps 960x960
    (40-200 rotated text rectangles each), threshold 0.3, box_thresh 0.6,
    unclip 1.5, fused on the device (tocr_db_postprocess). --units sets the
    batch (the survey's sweep: 8 / 64 / 512)."""
    name = "db_postprocess_8x960x960"
    metric = "maps/sec DB post-process (960x960 fp32 probability maps)"
    unit = "maps/s"
    dtype = "f32 map / int geometry"
    N, H, W = 8, 960, 960
    default_units = N
    launches_per_step = 16
    l2_note = ("8 maps = 29.5 MB < L2: every step first writes a 256 MB buffer to flush L2 "
               "(inside the timed step; the roofline time excludes it)")

    def __init__(self, dev, seed, units=None):
        from turboocr_b200._lib import synth
        from turboocr_b200.kernels import DbPostprocess
        if units:
            self.N = units
        self.units_per_step = self.N
        maps = np.zeros((self.N, self.H, self.W), np.float32)
        for i in range(self.N):
            synth().tocr_synth_db_map_host(maps[i].ctypes.data, self.H, self.W, 40, 200, seed, i)
        self.host_maps = maps
        self.maps = torch.from_numpy(maps).to(dev)
        self.db = DbPostprocess(self.N, self.H, self.W, dev, max_boxes=512)
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.algo_bytes = self.N * self.H * self.W * 4  # every map read once
        torch.cuda.synchronize()

    def step(self):
        self.flush.fill_(1)      # evict the maps from L2 (126 MB) between steps
        self.db(self.maps)

    def dominant_kernel_ms(self, iters=10):
        """The whole DB stage of one batch (L2 flushed before each)."""
        s = torch.cuda.current_stream()
        t = 0.0
        for _ in range(iters):
            self.flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            self.db(self.maps)
            e1.record(s)
            torch.cuda.synchronize()
            t += e0.elapsed_time(e1)
        self.dominant = "tocr_db_postprocess (16 launches) per batch"
        return t / iters

    def setup_e2e(self):
        self.h_maps = torch.empty(self.maps.shape, dtype=torch.float32, pin_memory=True)
        self.h_maps.copy_(self.maps)
        d = self.db
        self.h_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                      for t in (d.boxes, d.scores, d.counts)]
        self.h2d = self.h_maps.numel() * 4
        self.d2h = sum(t.numel() * t.element_size() for t in self.h_out)

    def e2e_step(self):
        self.maps.copy_(self.h_maps, non_blocking=True)
        self.db(self.maps)
        for h, d in zip(self.h_out, (self.db.boxes, self.db.scores, self.db.counts)):
            h.copy_(d, non_blocking=True)

class E2eWorkload:
    """BASELINE config 5 (the headline metric): 4096 synthetic 960x960 pages
    through preprocess + stem -> 8 INT8 DW+PW blocks -> head -> DB -> crops
    48x320 -> CTC (T=80, V=18385), split contiguously over the ranks (strong
    scaling: the job is 4096 pages in total). One step = this rank's whole
    shard, in micro-batches of 32 pages (turboocr_b200.pipeline.PagePipeline)."""
    name = "e2e_4096pages_960x960_det_rec"
    metric = "pages/sec det+rec hot path (960x960)"
    unit = "pages/s"
    dtype = "i8 (DW+PW blocks) / f16 activations / f32 DB map"
    scaling = "strong"
    TOTAL, MB = 4096, 32
    # pipelines (one stream each) that overlap consecutive micro-batches:
    # measured 7507 / 7646 / 7728 / 7752 / 7762 pages/s for 2 / 3 / 4 / 6 / 8;
    # each holds about 13 GB (mostly the stand-in logits of 4096 crop slots)
    NP = 6
    # DRAM bytes of the dominant launch (the CTC decode of pages 0..31's crops),
    # from one ncu capture of that launch (dram__bytes_read.sum + write.sum)
    traffic_per_launch = 5_026_007_296 + 3_558_912
    traffic_source = "ncu dram__bytes_read/write.sum of that launch"
    l2_note = "pages 2.76 MB each, >= 1.4 GB of input per rank per step > 126 MB L2 (no flush needed)"
    world = 1
    rank = 0

    def __init__(self, dev, seed, units=None):
        from turboocr_b200 import pipeline as pl
        self.pl = pl
        self.dev = dev
        if units:
            first, per = self.rank * units, units
        else:
            first, per = pl.shard(self.TOTAL, self.world, self.rank, self.MB)
        self.n_pages = max(self.MB, (per + self.MB - 1) // self.MB * self.MB)
        self.units_per_step = self.n_pages
        self.n_mb = self.n_pages // self.MB
        # NP pipelines on NP streams: consecutive micro-batches overlap, so the
        # latency-bound DB and crop stages of one run beside the streaming
        # stages of the other
        self.pipes = [pl.PagePipeline(dev, self.MB) for _ in range(self.NP)]
        self.pipe = self.pipes[0]
        self.streams = [torch.cuda.Stream(dev) for _ in range(self.NP)]
        self.pages = torch.empty(self.n_pages, 960, 960, 3, dtype=torch.uint8, device=dev)
        from turboocr_b200._lib import synth
        for i in range(0, self.n_pages, 256):
            n = min(256, self.n_pages - i)
            assert synth().tocr_synth_pages(self.pages[i].data_ptr(), n, 960, 960, 0x7EC00005,
                                            first + i, None) == 0
        torch.cuda.synchronize()
        self.launches_per_step = self.n_mb * self.pipes[0].launches_per_run
        self.algo_bytes = None  # set by dominant_kernel_ms (depends on the crop count)

    def _fork(self):
        cur = torch.cuda.current_stream()
        ev = torch.cuda.Event()
        ev.record(cur)
        for st in self.streams:
            st.wait_event(ev)

    def _join(self):
        cur = torch.cuda.current_stream()
        for st in self.streams:
            ev = torch.cuda.Event()
            ev.record(st)
            cur.wait_event(ev)

    def step(self):
        self._fork()
        for i in range(self.n_mb):
            k = i % self.NP
            with torch.cuda.stream(self.streams[k]):
                self.pipes[k].run(self.pages[i * self.MB:(i + 1) * self.MB])
        self._join()

    def dominant_kernel_ms(self, iters=10):
        """The CTC decode of one micro-batch's crops (tocr_ctc_greedy_f16_dev:
        the logits read is the largest single stream of the path)."""
        from turboocr_b200._lib import call
        p = self.pipe
        p.run(self.pages[:self.MB])
        torch.cuda.synchronize()
        n_crops = int(p.crop_off[self.MB].item())
        self.algo_bytes = n_crops * self.pl.REC_T * self.pl.REC_V * 2
        self.dominant = "ctc_rows_f16_kernel (+ collapse) over one micro-batch's crops"
        s = torch.cuda.current_stream()
        nc = p.crop_off[self.MB:]

        def once():
            call("tocr_ctc_greedy_f16_dev", p.logits.data_ptr(), nc.data_ptr(), p.max_crops,
                 self.pl.REC_T, self.pl.REC_V, self.pl.REC_V, p.tokens.data_ptr(),
                 p.lengths.data_ptr(), p.line_scores.data_ptr(), p.step_idx.data_ptr(),
                 p.step_prob.data_ptr(), s.cuda_stream)
        once()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(iters):
            once()
        e1.record(s)
        torch.cuda.synchronize()
        self.crops_per_page = n_crops / self.MB
        return e0.elapsed_time(e1) / iters

    def det_only_pages_per_s(self, reps=2):
        """The same shard through the detection half only (stem, blocks, head,
        ink map, DB, crop transforms, ROI warp; no stand-in rec logits and no
        CTC decode), device-timed like the headline."""
        def det_step():
            self._fork()
            for i in range(self.n_mb):
                k = i % self.NP
                with torch.cuda.stream(self.streams[k]):
                    self.pipes[k].run(self.pages[i * self.MB:(i + 1) * self.MB], rec=False)
            self._join()
        det_step()
        torch.cuda.synchronize()
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            det_step()
        e1.record(s)
        torch.cuda.synchronize()
        return self.n_pages * reps / (e0.elapsed_time(e1) / 1e3)

    def path_bytes_per_page(self):
        """Algorithmic HBM bytes of the whole path per page: stem in/out, every
        block's input and output, the DB map written and read, crops written,
        stand-in logits written and read by the decode."""
        b = 960 * 960 * 3 + 480 * 480 * 32 * 2
        h, w = 480, 480
        for c, co, st in self.pl.SCHEDULE:
            ho, wo = (h - 1) // st + 1, (w - 1) // st + 1
            b += h * w * c * 2 + ho * wo * co * 2
            h, w = ho, wo
        b += 960 * 960 * 3 + 2 * 960 * 960 * 4          # ink map: page read, map write + read
        crops = getattr(self, "crops_per_page", 58.0)
        b += crops * (3 * self.pl.REC_H * self.pl.REC_W * 2 + 2 * self.pl.REC_T * self.pl.REC_V * 2)
        return b

    # end-to-end: pinned host pages -> H2D per micro-batch -> path -> D2H of
    # boxes, scores, counts, tokens, line scores; each stream copies
    # its own micro-batch in and its results out, so copies overlap the other
    # stream's compute
    def setup_e2e(self):
        self.n_host = min(self.n_pages, 256)
        self.h_pages = torch.empty(self.n_host, 960, 960, 3, dtype=torch.uint8, pin_memory=True)
        self.h_pages.copy_(self.pages[:self.n_host])
        self.stage = [torch.empty(self.MB, 960, 960, 3, dtype=torch.uint8, device=self.dev)
                      for _ in range(self.NP)]
        self.h_out = []
        for p in self.pipes:
            self.h_out.append([torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                               for t in (p.db.boxes, p.db.scores, p.db.counts, p.tokens,
                                         p.lengths, p.line_scores)])
        self.h2d = self.n_pages * 960 * 960 * 3
        per_mb = sum(t.numel() * t.element_size() for t in self.h_out[0])
        self.d2h = self.n_mb * per_mb

    def e2e_step(self):
        self._fork()
        for i in range(self.n_mb):
            k = i % self.NP
            p = self.pipes[k]
            with torch.cuda.stream(self.streams[k]):
                j = (i * self.MB) % self.n_host
                src = self.h_pages[j:j + self.MB] if j + self.MB <= self.n_host else self.h_pages[:self.MB]
                self.stage[k].copy_(src, non_blocking=True)
                p.run(self.stage[k])
                for h, d in zip(self.h_out[k], (p.db.boxes, p.db.scores, p.db.counts, p.tokens,
                                                p.lengths, p.line_scores)):
                    h.copy_(d, non_blocking=True)
        self._join()

def workload_config(Wl, world: int, units: int) -> dict:
    """The `config` object of both arms (computed without a GPU, so the
    reference arm prints the same one)."""
    cfg = {"workload": Wl.name, "l2": Wl.l2_note,
           "parallelism": f"dp{world} (independent shards)"}
    if Wl is E2eWorkload:
        per = -(-Wl.TOTAL // world)
        per = -(-per // Wl.MB) * Wl.MB
        cfg.update({
            "pages_total": Wl.TOTAL, "pages_per_gpu": units or per, "micro_batch": Wl.MB,
            "backbone": "stem 3->32 s2; " + ", ".join(f"{c}->{co} s{st}" for c, co, st in
                                                     E2E_SCHEDULE),
            "rec": "stand-in logits 80 x 18385 per crop (rec network out of scope)"})
    else:
        cfg["units_per_gpu_per_step"] = units or Wl.default_units
    return cfg


E2E_SCHEDULE = [(32, 64, 1), (64, 64, 2), (64, 128, 1), (128, 128, 2),
                (128, 128, 1), (128, 128, 2), (128, 128, 1), (128, 256, 1)]

WORKLOADS = {"db": DbWorkload, "ctc": CtcWorkload, "preprocess": PreprocessWorkload,
             "dwpw": DwPwWorkload, "rec_head": RecHeadWorkload, "db_head": DbHeadWorkload,
             "png": PngWorkload, "e2e": E2eWorkload}
SEEDS = {"db": 0, "ctc": 1, "preprocess": 2, "dwpw": 3, "e2e": 5, "rec_head": 6, "db_head": 7,
         "png": 8}


# ------------------------------------------------------------------ main ----
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="e2e", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--units", type=int, default=0,
                    help="override the per-GPU units per step (small profiling cases)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    Wl = WORKLOADS[args.workload]
    cores = len(os.sched_getaffinity(0))

    config = workload_config(Wl, world, args.units)
    if args.impl == "reference":
        # The reference's CPU implementation of the path on this host's cores,
        # rank 0 only; no GPU and none of this repository's libraries.
        if rank != 0:
            return
        from oracle.cpu_baselines import BASELINES
        vals, desc = BASELINES[args.workload](cores, args.warmup + args.steps)
        v = statistics.median(vals[args.warmup:])
        units = desc.pop("units_per_step")
        print(json.dumps({"impl": "reference", "metric": Wl.metric, "value": v, "unit": Wl.unit,
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": 1e3 * units / v,
                          "higher_is_better": True, "scaling": getattr(Wl, "scaling", "weak"),
                          "vs_baseline": None, "dtype": Wl.dtype,
                          "data": "synthetic (seeded generator, BASELINE config shapes)",
                          "config": config,
                          "cpu_baseline": dict(desc, value=v, unit=Wl.unit),
                          "e2e": {"value": v, "unit": Wl.unit, "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    seed = 0x7EC00000 + SEEDS[args.workload] + 1000 * rank
    Wl.world, Wl.rank = world, rank
    wl = Wl(dev, seed, args.units)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        wl.step()
    e1.record(s)
    torch.cuda.synchronize()
    barrier()
    ms_total = e0.elapsed_time(e1)
    clk = clocks.stop()

    # end-to-end through the public API with pinned host buffers
    wl.setup_e2e()
    for _ in range(2):
        wl.e2e_step()
    torch.cuda.synchronize()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(s)
    n_e2e = max(3, min(args.steps, 10))
    for _ in range(n_e2e):
        wl.e2e_step()
    e3.record(s)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = e2.elapsed_time(e3) / n_e2e

    kernel_ms = wl.dominant_kernel_ms()
    t = torch.tensor([ms_total, ms_e2e, kernel_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, ms_e2e, kernel_ms = t.tolist()

    if rank == 0:
        ms_step = ms_total / args.steps
        value = wl.units_per_step * world / (ms_step / 1e3)
        peak, peak_kind = hbm_peak()
        achieved = wl.algo_bytes / (kernel_ms / 1e3) / 1e9
        tensor_bound = getattr(Wl, "bound", "hbm") == "tensor"
        if tensor_bound:
            peak, peak_kind = tensor_peak()
            achieved = wl.algo_flops / (kernel_ms / 1e3) / 1e12
        line = {
            "metric": Wl.metric, "value": value, "unit": Wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": getattr(Wl, "scaling", "weak"),
            "vs_baseline": None,
            "dtype": Wl.dtype, "data": "synthetic (seeded generator, BASELINE config shapes)",
            "config": config,
            "gpu_launches": wl.launches_per_step * args.steps,
            "e2e": {"value": wl.units_per_step * world / (ms_e2e / 1e3), "unit": Wl.unit,
                    "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h},
            "roofline": {"bound": "tensor" if tensor_bound else "hbm", "achieved": achieved,
                         "peak": peak, "unit": "TFLOP/s" if tensor_bound else "GB/s",
                         "frac": achieved / peak,
                         "traffic": getattr(Wl, "traffic_per_launch", None) or
                                    (getattr(Wl, "traffic_per_unit", 0) * wl.units_per_step or None),
                         "traffic_source": getattr(Wl, "traffic_source", None),
                         "peak_source": f"{peak_kind} " + ("bf16_tflops" if tensor_bound
                                                            else "hbm_gbs"),
                         "algorithmic_bytes_per_launch": wl.algo_bytes},
            "clocks": clk,
        }
        if hasattr(wl, "dominant"):
            line["roofline"]["kernel"] = wl.dominant
        if args.workload == "db" and not args.units and world == 1:
            # the survey's batch sweep: one call over 64 and 512 maps (the
            # call's latency is the longest union sweep, more maps run beside it)
            sweep = {"8": value}
            for n in (64, 512):
                big = Wl(dev, seed + n, n)
                big.step()
                torch.cuda.synchronize()
                sweep[str(n)] = n / (big.dominant_kernel_ms(iters=2) / 1e3)
                del big
                torch.cuda.empty_cache()
            line["batch_sweep_maps_per_s"] = sweep
            line["latency_ms_batch8"] = kernel_ms
        if args.workload == "png" and not args.units and world == 1:
            # a 64-page batch (one file per SM on fewer than half of the SMs)
            small = Wl(dev, seed + 64, 64)
            small.step()
            torch.cuda.synchronize()
            ms64 = small.dominant_kernel_ms(iters=3)
            line["batch_sweep_pages_per_s"] = {"64": 64 / (ms64 / 1e3), str(Wl.N): value}
            line["latency_ms_batch64"] = ms64
            del small
            torch.cuda.empty_cache()
        if args.workload == "e2e":
            line["crops_per_page"] = round(wl.crops_per_page, 2)
            bpp = wl.path_bytes_per_page()
            ach = bpp * value / world / 1e9
            line["roofline_path"] = {"bound": "hbm", "bytes_per_page": bpp,
                                     "achieved": ach, "peak": peak, "unit": "GB/s",
                                     "frac": ach / peak,
                                     "note": "algorithmic bytes of every stage per page x pages/s per GPU"}
            if world == 1:
                line["det_only"] = {
                    "value": wl.det_only_pages_per_s(), "unit": "pages/s",
                    "stages": "preprocess+stem, 8 DW+PW blocks, head, ink map, DB, crop "
                              "transforms, ROI warp (no stand-in rec logits, no CTC)"}
        if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
            from oracle.cpu_baselines import BASELINES
            vals, desc = BASELINES[args.workload](cores, 2)
            desc.pop("units_per_step")
            line["cpu_baseline"] = dict(desc, value=vals[-1], unit=Wl.unit)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
