"""ORACLE-side CPU path of the end-to-end page workload,
used only as bench.py's reference arm and cpu_baseline. It loads none of
this repository's native libraries: inputs come from oracle/synth_host.py
(numpy restatements of the seeded generators), every stage runs on the host.

Per page, the stages of the reference's CPU backend (src/pipeline/ocr/
cpu_ocr_pipeline.cpp:92,116), with the networks that are absent here
replaced the same way the device path replaces them:

  preprocess  cv2.resize (INTER_LINEAR) + per-channel normalise to fp32 CHW,
              src/detection/cpu_paddle_det.cpp:53-94
  backbone    stem 3x3 s2 3->32 and the 8 DW3x3+PW1x1 blocks in torch fp32
              with the device path's random-init weights (same seeds); the
              reference runs its det network in ONNX Runtime, absent here
  prob map    the synthetic run's DB map (ink map of the page)
  DB          extract_boxes_from_bitmap restated over cv2 + the reference's
              Clipper (oracle/db_oracle.py, det_postprocess.cpp:145-222)
  crops       cv2.warpPerspective with the reference's compute_crop_transform
              (src/recognition/cpu_paddle_rec.cpp:80-85)
  CTC         the reference's own ctc_decode.cpp (ctc_greedy_decode_raw) on
              fp32 rows; the stand-in logits are made before the timed region

Throughput: one single-threaded worker process per host core, each owning
its own pages; a step is every worker processing its pages once, timed from
the first worker's start to the last worker's end.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import time

import numpy as np

PAGE_SEED = 0x7EC00005
SCHEDULE = [(32, 64, 1), (64, 64, 2), (64, 128, 1), (128, 128, 2),
            (128, 128, 1), (128, 128, 2), (128, 128, 1), (128, 256, 1)]
REC_H, REC_W, REC_T, REC_V = 48, 320, 80, 18385
BN_EPS = 1e-5
DET_MEAN = np.array([0.485, 0.456, 0.406], np.float32)
DET_INV_STD = (1.0 / np.array([0.229, 0.224, 0.225], np.float32)).astype(np.float32)


def _bn(rng, n):
    g = rng.uniform(0.5, 1.5, n)
    b = rng.normal(0.0, 0.1, n)
    mu = rng.normal(0.0, 0.1, n)
    var = rng.uniform(0.5, 1.5, n)
    s = g / np.sqrt(var + BN_EPS)
    return s, b - mu * s


def network_params(seed: int = PAGE_SEED):
    """The device pipeline's random-init weights, drawn with the same seeds
    and order: stem (seed), block i (seed + 1 + i), head (seed + 100)."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.2, (32, 3, 3, 3))
    s, b = _bn(rng, 32)
    stem = ((w * s[:, None, None, None]).astype(np.float32), b.astype(np.float32))
    blocks = []
    for i, (c, co, st) in enumerate(SCHEDULE):
        r = np.random.default_rng(seed + 1 + i)
        wdw = r.normal(0.0, 0.05, (c, 3, 3))
        wpw = r.normal(0.0, 0.05, (co, c))
        s1, b1 = _bn(r, c)
        s2, b2 = _bn(r, co)
        blocks.append(((wdw * s1[:, None, None]).astype(np.float32), b1.astype(np.float32),
                       (wpw * s2[:, None]).astype(np.float32), b2.astype(np.float32), st))
    r = np.random.default_rng(seed + 100)
    head = (r.normal(0, 0.05, 256).astype(np.float32), float(r.normal(0, 0.1)))
    return stem, blocks, head


class PageWork:
    """One page's inputs, prepared before the timed region."""

    def __init__(self, page_index: int, seed: int = PAGE_SEED):
        from . import db_oracle as do
        from . import synth_host as sh
        self.page = sh.make_page(960, 960, seed, page_index)
        n_crops = len(do.db_postprocess(sh.ink_map(self.page)))
        self.n_crops = n_crops
        self.logits = sh.rec_logits(n_crops, REC_T, REC_V, seed, 0, dtype=np.float32)


class CpuPath:
    def __init__(self, seed: int = PAGE_SEED):
        import torch
        stem, blocks, head = network_params(seed)
        t = torch.from_numpy
        self.stem = (t(stem[0]), t(stem[1]))
        self.blocks = [(t(a).unsqueeze(1), t(b), t(c)[:, :, None, None], t(d), st)
                       for a, b, c, d, st in blocks]
        self.head = (t(head[0])[None, :, None, None], head[1])

    def backbone(self, x):
        import torch
        F = torch.nn.functional
        with torch.no_grad():
            y = F.hardswish(F.conv2d(torch.from_numpy(x), *self.stem, stride=2, padding=1))
            for wd, bd, wp, bp, st in self.blocks:
                y = F.hardswish(F.conv2d(y, wd, bd, stride=st, padding=1, groups=wd.shape[0]))
                y = F.hardswish(F.conv2d(y, wp, bp))
            return torch.sigmoid(F.conv2d(y, self.head[0]) + self.head[1])

    def run_page(self, w: PageWork, times: dict) -> int:
        import cv2
        from . import ctc_oracle as co
        from . import db_oracle as do
        from . import synth_host as sh
        from ._crop import crop_transform
        t0 = time.perf_counter()
        r = cv2.resize(w.page, (960, 960), interpolation=cv2.INTER_LINEAR)
        x = ((r.astype(np.float32) * np.float32(1 / 255.0) - DET_MEAN) * DET_INV_STD)
        x = np.ascontiguousarray(x.transpose(2, 0, 1)[None])
        t1 = time.perf_counter()
        self.backbone(x)
        t2 = time.perf_counter()
        dets = do.db_postprocess(sh.ink_map(w.page))
        t3 = time.perf_counter()
        for quad, _ in dets:
            m = crop_transform(quad, REC_H, REC_W)
            cv2.warpPerspective(w.page, m.reshape(3, 3), (REC_W, REC_H),
                                flags=cv2.INTER_LINEAR | cv2.WARP_INVERSE_MAP,
                                borderMode=cv2.BORDER_REPLICATE)
        t4 = time.perf_counter()
        n = min(len(dets), w.n_crops)
        if n:
            co.ref_decode_batch(w.logits[:n], REC_V, 1, simd=True)
        t5 = time.perf_counter()
        for k, v in (("preprocess", t1 - t0), ("backbone", t2 - t1), ("db", t3 - t2),
                     ("crops", t4 - t3), ("ctc", t5 - t4)):
            times[k] = times.get(k, 0.0) + v
        return len(dets)


_THREAD_VARS = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")


def _worker(pages, n_steps, seed, start, results):
    import cv2
    import torch
    torch.set_num_threads(1)
    cv2.setNumThreads(1)
    path = CpuPath(seed)
    works = [PageWork(p, seed) for p in pages]
    path.run_page(works[0], {})          # first-call costs outside the timed steps
    start.wait()
    for step in range(n_steps):
        start.wait()
        times: dict = {}
        t0 = time.perf_counter()
        for w in works:
            path.run_page(w, times)
        t1 = time.perf_counter()
        results.put((step, t0, t1, len(works), times))


def run_throughput(n_steps: int, workers: int, pages_per_worker: int = 1,
                   seed: int = PAGE_SEED, first_page: int = 0):
    """Runs n_steps steps; returns per step (pages/s, stage seconds summed
    over the workers, pages). CLOCK_MONOTONIC (perf_counter) is shared by the
    processes, so the step time is max(end) - min(start) over workers."""
    ctx = mp.get_context("spawn")
    # single-threaded workers: the thread pools of numpy/torch are sized at
    # import, so the limits go into the environment the children inherit
    saved = {k: os.environ.get(k) for k in _THREAD_VARS}
    os.environ.update({k: "1" for k in _THREAD_VARS})
    start = ctx.Barrier(workers + 1)
    results = ctx.Queue()
    procs = []
    for k in range(workers):
        pages = [first_page + k * pages_per_worker + j for j in range(pages_per_worker)]
        p = ctx.Process(target=_worker, args=(pages, n_steps, seed, start, results), daemon=True)
        p.start()
        procs.append(p)
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    out = []
    try:
        start.wait(timeout=600)
        for step in range(n_steps):
            start.wait(timeout=600)
            rows = [results.get(timeout=600) for _ in range(workers)]
            t0 = min(r[1] for r in rows)
            t1 = max(r[2] for r in rows)
            pages = sum(r[3] for r in rows)
            times: dict = {}
            for r in rows:
                for k, v in r[4].items():
                    times[k] = times.get(k, 0.0) + v
            out.append((pages / (t1 - t0), times, pages))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    return out
