"""The DB head of the detection network on the device (FPN neck over three
backbone levels + the binarisation head), over the C-ABI of
turboocr_b200/csrc/dbhead.cu. The reference runs PP-OCR's DBFPN + DBHead
inside TensorRT; its trained weights are not available, so the weights here
are drawn by tocr_synth_weights from seed 0x7EC0DB00 + k (uniform, scaled to
keep the activation variance near one), with the BatchNorms of the head
already folded into the convolutions:

  lat4 [96][256] (k=0), lat3 [96][128] (k=1), lat2 [96][128] (k=2)   1x1, no bias
  p4, p3, p2 [24][96][3][3] (k=3, 4, 5)                              3x3, no bias
  head conv [24][72][3][3] (k=6) + b1 [24] (k=7), ReLU
  convT1 [24][24][2][2] (k=8) + b2 [24] (k=9), ReLU
  convT2 [24][1][2][2] (k=10) + b3 (k=11), sigmoid
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import call, lib

SEED = 0x7EC0DB00
SHAPES = {  # name: (k, shape, scale)
    "lat4": (0, (96, 256, 1, 1), 0.108), "lat3": (1, (96, 128, 1, 1), 0.153),
    "lat2": (2, (96, 128, 1, 1), 0.153),
    "p4": (3, (24, 96, 3, 3), 0.059), "p3": (4, (24, 96, 3, 3), 0.059),
    "p2": (5, (24, 96, 3, 3), 0.059),
    "head": (6, (24, 72, 3, 3), 0.068), "b1": (7, (24,), 0.1),
    "up1": (8, (24, 24, 2, 2), 0.354), "b2": (9, (24,), 0.1),
    "up2": (10, (24, 1, 2, 2), 0.354), "b3": (11, (1,), 0.1),
}


def synth_weights() -> dict[str, np.ndarray]:
    L = lib()
    out = {}
    for name, (k, shape, scale) in SHAPES.items():
        a = np.empty(int(np.prod(shape)), np.float32)
        assert L.tocr_synth_weights(SEED + k, scale, a.ctypes.data, a.size) == 0
        out[name] = a.reshape(shape)
    return out


def _pack(w: np.ndarray) -> np.ndarray:
    cout, cin, k, _ = w.shape
    L = lib()
    n = L.tocr_conv_tc_packed_bytes(cin, cout, k)
    blob = np.zeros(n, np.uint8)
    w = np.ascontiguousarray(w, np.float32)
    call("tocr_conv_tc_pack", cin, cout, k, w.ctypes.data, blob.ctypes.data, C.c_size_t(n))
    return blob


class DbHead:
    """c2 [n][h][w][128], c3 [n][h/2][w/2][128], c4 [n][h/4][w/4][256] fp16
    NHWC (levels /4, /8, /16 of the page) -> probability map [n][4h][4w] fp32."""

    def __init__(self, device, weights: dict[str, np.ndarray] | None = None):
        self.dev = device
        self.w = weights or synth_weights()
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
        self.blobs = {k: t(_pack(self.w[k])) for k in ("lat4", "lat3", "lat2", "p4", "p3", "p2",
                                                       "head")}
        self.b1 = t(self.w["b1"])
        self.up1 = t(self.w["up1"])
        self.b2 = t(self.w["b2"])
        self.up2 = t(self.w["up2"])
        self.b3 = float(self.w["b3"][0])
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.bufs = {}

    def _buf(self, name, shape, dtype=torch.float16):
        b = self.bufs.get(name)
        if b is None or tuple(b.shape) != tuple(shape):
            b = torch.empty(shape, dtype=dtype, device=self.dev)
            self.bufs[name] = b
        return b

    def _conv(self, x, blob, cout, k, out, bias=None, relu=False, up=None, stream=None):
        n, h, w, cin = x.shape
        s = stream if stream is not None else torch.cuda.current_stream()
        call("tocr_conv_tc_f16", x.data_ptr(), n, h, w, cin, cout, k, blob.data_ptr(),
             bias.data_ptr() if bias is not None else None, int(relu),
             up.data_ptr() if up is not None else None, out.data_ptr(), self.err.data_ptr(),
             s.cuda_stream)
        return out

    def __call__(self, c2, c3, c4, stream=None):
        n, h, w, _ = c2.shape
        s = stream if stream is not None else torch.cuda.current_stream()
        in4 = self._conv(c4, self.blobs["lat4"], 96, 1, self._buf("in4", (n, h // 4, w // 4, 96)),
                         stream=s)
        out3 = self._conv(c3, self.blobs["lat3"], 96, 1, self._buf("out3", (n, h // 2, w // 2, 96)),
                          up=in4, stream=s)
        out2 = self._conv(c2, self.blobs["lat2"], 96, 1, self._buf("out2", (n, h, w, 96)),
                          up=out3, stream=s)
        p4 = self._conv(in4, self.blobs["p4"], 24, 3, self._buf("p4", (n, h // 4, w // 4, 24)),
                        stream=s)
        p3 = self._conv(out3, self.blobs["p3"], 24, 3, self._buf("p3", (n, h // 2, w // 2, 24)),
                        stream=s)
        p2 = self._conv(out2, self.blobs["p2"], 24, 3, self._buf("p2", (n, h, w, 24)), stream=s)
        fuse = self._buf("fuse", (n, h, w, 72))
        call("tocr_fpn_concat_f16", p4.data_ptr(), p3.data_ptr(), p2.data_ptr(), n, h, w,
             fuse.data_ptr(), s.cuda_stream)
        h1 = self._conv(fuse, self.blobs["head"], 24, 3, self._buf("h1", (n, h, w, 24)),
                        bias=self.b1, relu=True, stream=s)
        prob = self._buf("prob", (n, 4 * h, 4 * w), torch.float32)
        call("tocr_db_head_up_f32", h1.data_ptr(), n, h, w, self.up1.data_ptr(), self.b2.data_ptr(),
             self.up2.data_ptr(), C.c_float(self.b3), prob.data_ptr(), s.cuda_stream)
        return prob


def reference(w: dict[str, np.ndarray], c2, c3, c4):
    """fp32 torch restatement (NCHW) of the same network; returns (h1 NHWC, prob)."""
    F = torch.nn.functional
    dev = c2.device
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    x2, x3, x4 = (c.permute(0, 3, 1, 2).float() for c in (c2, c3, c4))
    up = lambda x, s: F.interpolate(x, scale_factor=s, mode="nearest")
    in4 = F.conv2d(x4, t(w["lat4"]))
    out3 = F.conv2d(x3, t(w["lat3"])) + up(in4, 2)
    out2 = F.conv2d(x2, t(w["lat2"])) + up(out3, 2)
    p4 = F.conv2d(in4, t(w["p4"]), padding=1)
    p3 = F.conv2d(out3, t(w["p3"]), padding=1)
    p2 = F.conv2d(out2, t(w["p2"]), padding=1)
    fuse = torch.cat([up(p4, 4), up(p3, 2), p2], dim=1)
    h1 = F.relu(F.conv2d(fuse, t(w["head"]), t(w["b1"]), padding=1))
    h2 = F.relu(F.conv_transpose2d(h1, t(w["up1"]), t(w["b2"]), stride=2))
    h3 = F.conv_transpose2d(h2, t(w["up2"]), t(w["b3"]), stride=2)
    return h1.permute(0, 2, 3, 1), torch.sigmoid(h3)[:, 0]
