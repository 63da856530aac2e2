"""ORACLE-side CPU baselines of the five BASELINE configs, for bench.py's
reference arm (`--impl reference`) and its `cpu_baseline` key only. Nothing
here loads this repository's native libraries or touches a GPU: inputs are
made on the host by oracle/synth_host.py, the work runs on the host cores.

Each function runs `n_steps` bounded samples of its workload and returns
(list of per-step values in the workload's unit, a dict describing the
sample: kind, cores, units_per_step, sample).
"""
from __future__ import annotations

import multiprocessing as mp
import time

import numpy as np

from . import synth_host as sh

SEED = 0x7EC00000


def e2e(cores: int, n_steps: int, pages_per_worker: int = 1):
    """Config 5: one single-threaded worker process per core, each with its
    own pages (oracle/cpu_path.py); a step = every worker's pages once."""
    from . import cpu_path as cp
    rows = cp.run_throughput(n_steps, cores, pages_per_worker)
    pages = rows[0][2]
    stage = {}
    for _, times, p in rows:
        for k, v in times.items():
            stage[k] = stage.get(k, 0.0) + v / p / len(rows)
    return [r[0] for r in rows], {
        "kind": "port", "cores": cores, "units_per_step": pages,
        "sample": f"{pages} pages per step ({pages_per_worker} per worker process x {cores} "
                  "single-threaded processes); stage s/page/core: " +
                  ", ".join(f"{k} {v:.3f}" for k, v in stage.items()) +
                  "; CTC = the reference's ctc_decode.cpp, DB = cv2 + the reference's Clipper, "
                  "backbone = torch fp32 (ORT absent)"}


def ctc(cores: int, n_steps: int, lines: int = 0):
    """Config 2: the reference's ctc_decode.cpp (ctc_greedy_decode_raw, SIMD_CTC=1)
    plus the max-softmax beside it, on fp32 rows, lines over `cores` threads."""
    from . import ctc_oracle as co
    T, V = 80, 18385
    n = lines or max(2 * cores, 16)
    x = sh.ctc_logits(n, T, V, SEED + 1, dtype=np.float32)
    co.ref_decode_batch(x[:cores], V, cores, simd=True)
    vals = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        co.ref_decode_batch(x, V, cores, simd=True)
        vals.append(n / (time.perf_counter() - t0))
    return vals, {"kind": "reference", "cores": cores, "units_per_step": n,
                  "sample": f"{n} lines of 80 x 18385 per step (config-2 generator on the host), "
                            "fp32 rows, std::thread over lines"}


def _pre_images(n: int):
    """The first n images of the config-3 batch, as the device generator lays
    them out (one byte stream, each image at a 256-byte aligned offset)."""
    seed = SEED + 2
    dims = sh.preprocess_dims(n, seed)
    sizes = [h * w * 3 for h, w in dims]
    offs = np.concatenate([[0], np.cumsum([(s + 255) // 256 * 256 for s in sizes])])
    buf = sh.fill_u8(int(offs[-1]), seed, 3)
    return dims, [buf[int(offs[i]):int(offs[i]) + sizes[i]].reshape(h, w, 3)
                  for i, (h, w) in enumerate(dims)]


def round32_floor(v: float) -> int:
    """det_config.h:50-52: std::round (half away from zero) of v / 32, x32, floor 32."""
    q = v / 32.0
    f = np.floor(q)
    r = f + 1.0 if q - f >= 0.5 else f
    return max(int(r) * 32, 32)


def det_resize_max(h: int, w: int, L: int = 960, max_side: int = 960):
    """compute_det_resize with {"max", L, max_side} (det_config.h:58-81)."""
    ratio = np.float32(1.0)
    if max(h, w) > L:
        ratio = np.float32(np.float32(L) / np.float32(max(h, w)))
    rh = round32_floor(float(np.float32(np.float32(h) * ratio)))
    rw = round32_floor(float(np.float32(np.float32(w) * ratio)))
    lo = max(rh, rw)
    if lo > max_side:
        rs = max_side / lo
        rh, rw = round32_floor(rh * rs), round32_floor(rw * rs)
    return rh, rw


def preprocess(cores: int, n_steps: int, n_images: int = 0):
    """Config 3: cpu_paddle_det.cpp:53-94 restated with cv2 (INTER_LINEAR
    resize, normalise, letterbox into 960x960 fp16), images over threads."""
    import cv2
    from concurrent.futures import ThreadPoolExecutor
    cv2.setNumThreads(1)
    n = n_images or max(2 * cores, 16)
    dims, imgs = _pre_images(n)
    content = [det_resize_max(h, w) for h, w in dims]
    mean = np.array([0.485, 0.456, 0.406], np.float32)
    istd = 1.0 / np.array([0.229, 0.224, 0.225], np.float32)
    pad = ((0 - mean) * istd).astype(np.float16)[:, None, None]

    def one(i):
        ch, cw = content[i]
        r = cv2.resize(imgs[i], (cw, ch), interpolation=cv2.INTER_LINEAR)
        f = (r.astype(np.float32) * np.float32(1 / 255.0) - mean) * istd
        canvas = np.empty((3, 960, 960), np.float16)
        canvas[:] = pad
        canvas[:, :ch, :cw] = f.transpose(2, 0, 1)
        return canvas

    vals = []
    with ThreadPoolExecutor(cores) as ex:
        list(ex.map(one, range(min(n, cores))))
        for _ in range(n_steps):
            t0 = time.perf_counter()
            list(ex.map(one, range(n)))
            vals.append(n / (time.perf_counter() - t0))
    return vals, {"kind": "port", "cores": cores, "units_per_step": n,
                  "sample": f"{n} images per step (sides 600..2000), cv2 {cv2.__version__} "
                            "resize + normalise + letterbox, threads over images"}


def dwpw(cores: int, n_steps: int, images: int = 1):
    """Config 4: the block (DW3x3 + hardswish, PW1x1 + hardswish, BN folded)
    in torch fp32 on the host (mkldnn), all threads."""
    import torch
    torch.set_num_threads(cores)
    rng = np.random.default_rng(SEED + 4)
    C, CO = 128, 256
    wdw = rng.normal(0, 0.05, (C, 1, 3, 3)).astype(np.float32)
    bdw = rng.normal(0, 0.1, C).astype(np.float32)
    wpw = rng.normal(0, 0.05, (CO, C, 1, 1)).astype(np.float32)
    bpw = rng.normal(0, 0.1, CO).astype(np.float32)
    x = torch.from_numpy(rng.standard_normal((images, C, 240, 240), dtype=np.float32))
    F = torch.nn.functional
    t = [torch.from_numpy(a) for a in (wdw, bdw, wpw, bpw)]

    def block():
        with torch.no_grad():
            y = F.hardswish(F.conv2d(x, t[0], t[1], padding=1, groups=C))
            return F.hardswish(F.conv2d(y, t[2], t[3]))

    block()
    vals = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        block()
        vals.append(images / (time.perf_counter() - t0))
    return vals, {"kind": "port", "cores": cores, "units_per_step": images,
                  "sample": f"{images} image(s) of 128x240x240 per step, torch {torch.__version__} "
                            f"fp32, {cores} threads"}


def _db_one(m):
    from . import db_oracle as do
    return len(do.db_postprocess(m))


def db(cores: int, n_steps: int, maps: int = 8):
    """Config 1: the cv2 + reference-Clipper restatement of
    extract_boxes_from_bitmap, one process per map over the host cores."""
    from concurrent.futures import ProcessPoolExecutor
    host = [sh.db_map(960, 960, 40, 200, SEED, i) for i in range(maps)]
    vals = []
    with ProcessPoolExecutor(min(cores, maps), mp_context=mp.get_context("spawn")) as ex:
        list(ex.map(_db_one, host[:min(cores, maps)]))
        for _ in range(n_steps):
            t0 = time.perf_counter()
            list(ex.map(_db_one, host))
            vals.append(maps / (time.perf_counter() - t0))
    return vals, {"kind": "port", "cores": min(cores, maps), "units_per_step": maps,
                  "sample": f"{maps} maps per step, one process per map (cv2 + reference Clipper)"}


def rec_head(cores: int, n_steps: int, lines: int = 0):
    """The recognizer head + decode on the host: torch fp32 (all threads) for
    logits = features @ W^T + bias, argmax and max softmax probability per
    step, then the reference collapse (oracle/ctc_oracle.py). The reference
    runs this layer inside TensorRT, so the baseline is this restatement."""
    import torch
    from . import ctc_oracle as co
    T, K, V = 80, 128, 18385
    n = lines or max(4 * cores, 32)
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(SEED + 6)
    feat = torch.randn(n * T, K, generator=g).to(torch.float16).float()
    w = (torch.randn(V, K, generator=g) * (3.0 / K ** 0.5)).to(torch.float16).float()
    b = torch.randn(V, generator=g) * 0.5

    def once():
        logits = feat @ w.T + b
        m, idx = logits.max(dim=1)
        p = 1.0 / torch.exp(logits - m[:, None]).sum(dim=1)
        idx, p = idx.numpy(), p.numpy().astype(np.float32)
        for line in range(n):
            co.collapse(idx[line * T:(line + 1) * T].tolist(), p[line * T:(line + 1) * T], V - 2)

    once()
    vals = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        once()
        vals.append(n / (time.perf_counter() - t0))
    return vals, {"kind": "port", "cores": cores, "units_per_step": n,
                  "sample": f"{n} lines x 80 steps per step, K=128, V=18385: torch fp32 GEMM "
                            "+ argmax + softmax max on all threads, then the reference collapse"}


def db_head(cores: int, n_steps: int, pages: int = 1):
    """The DB head on the host: the fp32 torch restatement of the network
    (turboocr_b200/dbhead.py reference), all threads; weights drawn by the
    same formula as tocr_synth_weights (restated in numpy here, so no product
    library is loaded)."""
    import torch
    torch.set_num_threads(cores)
    M64 = (1 << 64) - 1

    def synth(seed, scale, n):
        i = np.arange(1, n + 1, dtype=np.uint64)
        with np.errstate(over="ignore"):
            z = np.uint64(seed) + i * np.uint64(0x9E3779B97F4A7C15)
            z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
            z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
            z ^= z >> np.uint64(31)
        u = (z >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)
        return np.float32(scale) * (np.float32(2.0) * u - np.float32(1.0))

    shapes = {"lat4": (0, (96, 256, 1, 1), 0.108), "lat3": (1, (96, 128, 1, 1), 0.153),
              "lat2": (2, (96, 128, 1, 1), 0.153), "p4": (3, (24, 96, 3, 3), 0.059),
              "p3": (4, (24, 96, 3, 3), 0.059), "p2": (5, (24, 96, 3, 3), 0.059),
              "head": (6, (24, 72, 3, 3), 0.068), "b1": (7, (24,), 0.1),
              "up1": (8, (24, 24, 2, 2), 0.354), "b2": (9, (24,), 0.1),
              "up2": (10, (24, 1, 2, 2), 0.354), "b3": (11, (1,), 0.1)}
    w = {k: synth(0x7EC0DB00 + s, sc, int(np.prod(sh))).reshape(sh)
         for k, (s, sh, sc) in shapes.items()}
    g = torch.Generator().manual_seed(SEED + 7)
    c2 = torch.randn(pages, 240, 240, 128, generator=g).to(torch.float16)
    c3 = torch.randn(pages, 120, 120, 128, generator=g).to(torch.float16)
    c4 = torch.randn(pages, 60, 60, 256, generator=g).to(torch.float16)
    F = torch.nn.functional

    def once():  # the same network as turboocr_b200.dbhead.reference
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
        x2, x3, x4 = (c.permute(0, 3, 1, 2).float() for c in (c2, c3, c4))
        up = lambda x, s: F.interpolate(x, scale_factor=s, mode="nearest")
        in4 = F.conv2d(x4, t(w["lat4"]))
        out3 = F.conv2d(x3, t(w["lat3"])) + up(in4, 2)
        out2 = F.conv2d(x2, t(w["lat2"])) + up(out3, 2)
        fuse = torch.cat([up(F.conv2d(in4, t(w["p4"]), padding=1), 4),
                          up(F.conv2d(out3, t(w["p3"]), padding=1), 2),
                          F.conv2d(out2, t(w["p2"]), padding=1)], dim=1)
        h1 = F.relu(F.conv2d(fuse, t(w["head"]), t(w["b1"]), padding=1))
        h2 = F.relu(F.conv_transpose2d(h1, t(w["up1"]), t(w["b2"]), stride=2))
        return torch.sigmoid(F.conv_transpose2d(h2, t(w["up2"]), t(w["b3"]), stride=2))

    once()
    vals = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        once()
        vals.append(pages / (time.perf_counter() - t0))
    return vals, {"kind": "port", "cores": cores, "units_per_step": pages,
                  "sample": f"{pages} page(s) per step: the fp32 torch restatement of the DB head "
                            "on all threads (the reference runs it in TensorRT/ORT)"}


def _pagegen():
    """turboocr_b200/pagegen.py loaded by path (numpy + cv2 only), so that the
    package and its native library stay unloaded."""
    import importlib.util
    from pathlib import Path
    path = Path(__file__).resolve().parents[1] / "turboocr_b200" / "pagegen.py"
    spec = importlib.util.spec_from_file_location("_tocr_pagegen", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def png(cores: int, n_steps: int, pages: int = 64):
    """PNG decode as the reference does it (FastPngDecoder::decode: its
    vendored Wuffs, compiled in place, to BGR), the bench's 64 A4 pages
    spread over `cores` threads (the C decode releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    from . import png_oracle as po
    files = _pagegen().png_pages(pages, SEED + 8)
    vals = []
    with ThreadPoolExecutor(max_workers=cores) as ex:
        list(ex.map(po.wuffs_decode, files[:cores]))
        for _ in range(n_steps):
            t0 = time.perf_counter()
            outs = list(ex.map(po.wuffs_decode, files))
            vals.append(pages / (time.perf_counter() - t0))
            assert all(o[0] is not None for o in outs)
    return vals, {"kind": "reference", "cores": cores, "units_per_step": pages,
                  "sample": f"{pages} A4 pages of 1240x1754 (OpenCV-encoded PNG) per step, the "
                            "reference's Wuffs decode to BGR, one page per thread task"}


BASELINES = {"e2e": e2e, "ctc": ctc, "preprocess": preprocess, "dwpw": dwpw, "db": db,
             "rec_head": rec_head, "db_head": db_head, "png": png}
