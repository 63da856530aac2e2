"""Fused depthwise-separable conv blocks (subsystem 2) on top of the C-ABI.

``DwPwBlock`` owns one packed parameter blob on the device and runs
tocr_dwpw_block. ``make_block_params`` draws the synthetic block of
BASELINE config 4 (the weights of the reference's trained backbone are not
available): DW w ~ N(0, 0.05), PW w ~ N(0, 0.05), BatchNorm gamma ~ U[.5,1.5],
beta ~ N(0,.1), mean ~ N(0,.1), var ~ U[.5,1.5], folded into the convs.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import call, lib

KIND_INT8, KIND_FP8 = 0, 1
BN_EPS = 1e-5


@dataclass
class BlockParams:
    """BN-folded fp32 parameters of one block."""
    wdw: np.ndarray   # [C, 3, 3]
    bdw: np.ndarray   # [C]
    wpw: np.ndarray   # [CO, C]
    bpw: np.ndarray   # [CO]

    @property
    def C(self):
        return self.wdw.shape[0]

    @property
    def CO(self):
        return self.wpw.shape[0]


def _bn(rng, n):
    g = rng.uniform(0.5, 1.5, n)
    b = rng.normal(0.0, 0.1, n)
    mu = rng.normal(0.0, 0.1, n)
    var = rng.uniform(0.5, 1.5, n)
    s = g / np.sqrt(var + BN_EPS)
    return s, b - mu * s


def make_block_params(C_in: int, C_out: int, seed: int) -> BlockParams:
    rng = np.random.default_rng(seed)
    wdw = rng.normal(0.0, 0.05, (C_in, 3, 3))
    wpw = rng.normal(0.0, 0.05, (C_out, C_in))
    s1, b1 = _bn(rng, C_in)
    s2, b2 = _bn(rng, C_out)
    return BlockParams(wdw=(wdw * s1[:, None, None]).astype(np.float32),
                       bdw=b1.astype(np.float32),
                       wpw=(wpw * s2[:, None]).astype(np.float32),
                       bpw=b2.astype(np.float32))


def pack(params: BlockParams, kind: int) -> np.ndarray:
    """Host blob for tocr_dwpw_block (quantised PW weights, fp16 DW weights)."""
    L = lib()
    n = L.tocr_dwpw_packed_bytes(params.C, params.CO)
    out = np.zeros(n, dtype=np.uint8)
    arrs = [np.ascontiguousarray(a, dtype=np.float32)
            for a in (params.wdw, params.bdw, params.wpw, params.bpw)]
    call("tocr_dwpw_pack", params.C, params.CO, kind, *[a.ctypes.data for a in arrs],
         out.ctypes.data, C.c_size_t(n))
    return out


def dequant_pw(blob: np.ndarray, C_in: int, C_out: int, kind: int) -> np.ndarray:
    w = np.empty((C_out, C_in), dtype=np.float32)
    call("tocr_dwpw_dequant_pw", blob.ctypes.data, C_in, C_out, kind, w.ctypes.data)
    return w


class DwPwBlock:
    """One fused DW3x3 + PW1x1 block; activations fp16 NHWC on the device."""

    def __init__(self, params: BlockParams, kind: int, stride: int, device):
        self.params, self.kind, self.stride = params, kind, stride
        self.C, self.CO = params.C, params.CO
        self.blob_host = pack(params, kind)
        self.blob = torch.from_numpy(self.blob_host).to(device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    def out_shape(self, x: torch.Tensor):
        N, H, W, _ = x.shape
        return (N, (H - 1) // self.stride + 1, (W - 1) // self.stride + 1, self.CO)

    def __call__(self, x: torch.Tensor, y: torch.Tensor | None = None, stream=None):
        assert x.dtype == torch.float16 and x.is_contiguous() and x.shape[-1] == self.C
        if y is None:
            y = torch.empty(self.out_shape(x), dtype=torch.float16, device=x.device)
        N, H, W, _ = x.shape
        s = stream if stream is not None else torch.cuda.current_stream()
        call("tocr_dwpw_block", x.data_ptr(), y.data_ptr(), N, H, W, self.C, self.CO, self.stride,
             self.kind, self.blob.data_ptr(), self.err.data_ptr(), s.cuda_stream)
        return y

    def dequantized_pw(self) -> np.ndarray:
        return dequant_pw(self.blob_host, self.C, self.CO, self.kind)


def reference_block(x_nhwc: torch.Tensor, params: BlockParams, stride: int,
                    wpw: np.ndarray | None = None) -> torch.Tensor:
    """fp32 torch reference of one block (NHWC fp32 out): DW conv (groups=C)
    + bias, hardswish, 1x1 conv with `wpw` (default: the unquantised weights)
    + bias, hardswish. TF32 is disabled by the caller's context."""
    dev = x_nhwc.device
    x = x_nhwc.permute(0, 3, 1, 2).float()
    wd = torch.from_numpy(params.wdw).to(dev).unsqueeze(1)
    bd = torch.from_numpy(params.bdw).to(dev)
    y1 = torch.nn.functional.hardswish(
        torch.nn.functional.conv2d(x, wd, bd, stride=stride, padding=1, groups=params.C))
    w = torch.from_numpy(params.wpw if wpw is None else wpw).to(dev)
    y2 = torch.einsum("nchw,oc->nhwo", y1, w) + torch.from_numpy(params.bpw).to(dev)
    return torch.nn.functional.hardswish(y2)
