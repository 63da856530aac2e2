"""Host-side packing of the fused-block parameters (no GPU): quantisation
matches a numpy restatement, the 128B-swizzled layout round-trips, and
unsupported shapes are rejected."""
import numpy as np
import pytest
import torch

from turboocr_b200 import backbone as bb


@pytest.mark.parametrize("C,CO", [(128, 256), (64, 64), (32, 64), (256, 256)])
def test_int8_pack_roundtrip(C, CO):
    p = bb.make_block_params(C, CO, 3)
    blob = bb.pack(p, bb.KIND_INT8)
    w = bb.dequant_pw(blob, C, CO, bb.KIND_INT8)
    scale = np.abs(p.wpw).max(axis=1, keepdims=True) / np.float32(127)
    q = np.clip(np.rint(p.wpw / scale), -127, 127)
    np.testing.assert_allclose(w, (q * scale).astype(np.float32), rtol=1e-6, atol=1e-9)


def test_fp8_pack_matches_torch_e4m3():
    C, CO = 128, 256
    p = bb.make_block_params(C, CO, 4)
    blob = bb.pack(p, bb.KIND_FP8)
    w = bb.dequant_pw(blob, C, CO, bb.KIND_FP8)
    scale = np.abs(p.wpw).max(axis=1, keepdims=True) / np.float32(448)
    e = torch.from_numpy((p.wpw / scale).astype(np.float32)).to(torch.float8_e4m3fn).float()
    np.testing.assert_allclose(w, (e.numpy() * scale).astype(np.float32), rtol=1e-6, atol=1e-9)


def test_swizzle_layout():
    """Byte (co, c) of the B image sits at row co, 16B chunk (c/16) ^ (co%8)."""
    C, CO = 128, 64
    p = bb.make_block_params(C, CO, 5)
    blob = bb.pack(p, bb.KIND_INT8)
    scale = np.abs(p.wpw).max(axis=1, keepdims=True) / np.float32(127)
    q = np.clip(np.rint(p.wpw / scale), -127, 127).astype(np.int8)
    img = blob[: CO * 128].view(np.int8).reshape(CO, 8, 16)
    for co in (0, 1, 7, 8, 63):
        for c in (0, 15, 16, 77, 127):
            assert img[co, (c // 16) ^ (co % 8), c % 16] == q[co, c]


def test_rejects_unsupported_shapes():
    import turboocr_b200 as t
    p = bb.make_block_params(48, 64, 1)
    with pytest.raises(t.InvalidArgument):
        bb.pack(p, bb.KIND_INT8)
