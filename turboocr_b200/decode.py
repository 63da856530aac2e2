"""PNG files to device images (the reference's GpuImage: BGR u8 HWC rows
`step` bytes apart) over the C-ABI of turboocr_b200/csrc/png.cu.

The reference decodes on the host (src/decode/fast_png_decoder.cpp:48-128,
Wuffs; 16-bit files through cv::imdecode) and uploads the BGR pixels
(src/pipeline/ocr/ocr_pipeline_runtime.cpp:120-147). Here the compressed
files go to HBM and the pixels are made there; the per-side and pixel-area
caps are the reference's (include/turbo_ocr/decode/image_config.h:13-38,
env MAX_IMAGE_DIM and MAX_IMAGE_PIXELS_MP)."""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import call, lib

PNG_OK = 0
STATUS_NAMES = {
    0: "ok", 1: "bad header", 2: "bad chunk", 3: "bad checksum", 4: "missing palette",
    5: "bad zlib header", 6: "bad deflate data", 7: "too much data", 8: "not enough data",
    9: "bad filter", 10: "size mismatch", 11: "unsupported dimension", 12: "timeout",
    -1: "rejected on the host (not a PNG, malformed IHDR or over the size caps)",
}

JOB_DTYPE = np.dtype([("src_off", "<u8"), ("src_len", "<u8"), ("dst_off", "<u8"),
                      ("dst_pitch", "<u8"), ("scratch_off", "<u8"), ("width", "<i4"),
                      ("height", "<i4")])
assert JOB_DTYPE.itemsize == 48


class PngInfo(C.Structure):
    _fields_ = [("width", C.c_int32), ("height", C.c_int32), ("bit_depth", C.c_int32),
                ("color_type", C.c_int32), ("interlace", C.c_int32), ("reserved", C.c_int32),
                ("raw_bytes", C.c_uint64), ("scratch_bytes", C.c_uint64)]


def _env_int(name: str, default: int, lo: int, hi: int) -> int:
    """env::env_int (include/turbo_ocr/common/env_utils.h:35-45): unset,
    empty or malformed -> default; out of range -> clamped."""
    v = os.environ.get(name)
    if not v:
        return default
    try:
        x = int(v, 10)
    except ValueError:
        return default
    return min(max(x, lo), hi)


def max_image_dim() -> int:
    return _env_int("MAX_IMAGE_DIM", 16384, 64, 65535)


def max_image_pixels() -> int:
    return _env_int("MAX_IMAGE_PIXELS_MP", 128, 1, 4096) * 1000000


def is_png(data: bytes) -> bool:
    """FastPngDecoder::is_png (fast_png_decoder.h:18-21)."""
    return len(data) >= 8 and data[0] == 0x89 and data[1:4] == b"PNG"


def peek(data: bytes, max_dim: int | None = None, max_pixels: int | None = None) -> PngInfo | None:
    """The IHDR of one file and the scratch it needs, or None when it is not a
    PNG, the IHDR is malformed or the caps reject it."""
    info = PngInfo()
    buf = (C.c_uint8 * len(data)).from_buffer_copy(data) if data else None
    rc = lib().tocr_png_peek(buf, len(data), max_image_dim() if max_dim is None else max_dim,
                             max_image_pixels() if max_pixels is None else max_pixels,
                             C.byref(info))
    return info if rc == 0 else None


def _a16(v: int) -> int:
    return (v + 15) & ~15


@dataclass
class DecodedBatch:
    images: list[torch.Tensor | None]  # [h, w, 3] uint8 views into `dst` (row pitch `pitches`)
    status: list[int]
    pitches: list[int]
    dst: torch.Tensor


class PngBatchDecoder:
    """Decodes lists of PNG files on one device. Device buffers (files,
    scratch, pixels) and the pinned staging grow on demand and are reused;
    decode() returns views into them, valid until the next call."""

    def __init__(self, device: torch.device | str = "cuda"):
        self.dev = torch.device(device)
        self._bufs: dict[str, torch.Tensor] = {}

    def _buf(self, name: str, nbytes: int, pinned: bool = False) -> torch.Tensor:
        b = self._bufs.get(name)
        if b is None or b.numel() < nbytes:
            n = max(nbytes, 16)
            b = (torch.empty(n, dtype=torch.uint8, pin_memory=True) if pinned
                 else torch.empty(n, dtype=torch.uint8, device=self.dev))
            self._bufs[name] = b
        return b

    def plan(self, files: list[bytes]):
        """Host layout of one batch: the jobs, the host-rejected files and the
        byte totals (files, scratch, pixels)."""
        jobs = np.zeros(len(files), JOB_DTYPE)
        ok = []
        src = scr = dst = 0
        for i, f in enumerate(files):
            info = peek(f)
            if info is None:
                continue
            pitch = _a16(3 * info.width)
            jobs[i] = (src, len(f), dst, pitch, scr, info.width, info.height)
            ok.append(i)
            src += len(f)
            scr += _a16(info.scratch_bytes)
            dst += pitch * info.height
        return jobs, ok, src, scr, dst

    def decode(self, files: list[bytes], stream: torch.cuda.Stream | None = None) -> DecodedBatch:
        s = stream if stream is not None else torch.cuda.current_stream(self.dev)
        jobs, ok, nsrc, nscr, ndst = self.plan(files)
        status = [-1] * len(files)
        images: list[torch.Tensor | None] = [None] * len(files)
        pitches = [0] * len(files)
        dst = self._buf("dst", ndst)
        if not ok:
            return DecodedBatch(images, status, pitches, dst)
        sel = jobs[ok]
        host = self._buf("h_src", nsrc + sel.nbytes, pinned=True)
        hv = host.numpy()
        for j, i in enumerate(ok):
            o = int(sel[j]["src_off"])
            hv[o:o + len(files[i])] = np.frombuffer(files[i], np.uint8)
        hv[nsrc:nsrc + sel.nbytes] = np.frombuffer(sel.tobytes(), np.uint8)
        d_in = self._buf("d_src", _a16(nsrc) + sel.nbytes)
        scratch = self._buf("scratch", nscr)
        d_status = self._buf("status", 4 * len(ok)).view(torch.int32)
        h_status = self._buf("h_status", 4 * len(ok), pinned=True).view(torch.int32)
        with torch.cuda.stream(s):
            d_in[:nsrc].copy_(host[:nsrc], non_blocking=True)
            jo = _a16(nsrc)
            d_in[jo:jo + sel.nbytes].copy_(host[nsrc:nsrc + sel.nbytes], non_blocking=True)
            call("tocr_png_decode_batch", d_in.data_ptr(), d_in.data_ptr() + jo, len(ok),
                 dst.data_ptr(), scratch.data_ptr(), d_status.data_ptr(), s.cuda_stream)
            h_status[:len(ok)].copy_(d_status[:len(ok)], non_blocking=True)
        s.synchronize()
        for j, i in enumerate(ok):
            st = int(h_status[j])
            status[i] = st
            w, h, pitch = int(sel[j]["width"]), int(sel[j]["height"]), int(sel[j]["dst_pitch"])
            pitches[i] = pitch
            if st == PNG_OK:
                o = int(sel[j]["dst_off"])
                images[i] = dst[o:o + pitch * h].view(h, pitch)[:, :3 * w].view(h, w, 3)
        return DecodedBatch(images, status, pitches, dst)
