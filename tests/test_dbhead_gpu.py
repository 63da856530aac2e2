"""The DB head (FPN neck + binarisation head, turboocr_b200/dbhead.py over
csrc/dbhead.cu) against an fp32 torch restatement of the same network with
the same weights: the head's last hidden map (24 channels at /4) normwise and
the probability map elementwise. The device runs fp16 operands (weights and
stored activations) with fp32 accumulation, so the bounds are those of fp16
rounding carried through five convolutions."""
import numpy as np
import pytest
import torch

from turboocr_b200 import dbhead

pytestmark = pytest.mark.gpu

H1_TOL = 2e-2   # normwise relative, per image
PROB_TOL = 1e-2  # absolute, probabilities


@pytest.mark.parametrize("n,h,w", [(2, 64, 64), (1, 48, 80), (3, 32, 160)])
def test_db_head_matches_fp32_reference(tocr, cuda, n, h, w):
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator().manual_seed(n * 1000 + h + w)
    c2 = torch.randn(n, h, w, 128, generator=g).to(torch.float16).to(cuda)
    c3 = torch.randn(n, h // 2, w // 2, 128, generator=g).to(torch.float16).to(cuda)
    c4 = torch.randn(n, h // 4, w // 4, 256, generator=g).to(torch.float16).to(cuda)
    head = dbhead.DbHead(cuda)
    prob = head(c2, c3, c4)
    torch.cuda.synchronize()
    assert int(head.err.item()) == 0
    h1_ref, prob_ref = dbhead.reference(head.w, c2, c3, c4)
    h1 = head.bufs["h1"].float()
    for i in range(n):
        rel = (h1[i] - h1_ref[i]).norm() / h1_ref[i].norm()
        assert rel <= H1_TOL, (i, float(rel))
    d = (prob - prob_ref).abs().max().item()
    assert d <= PROB_TOL, d
    assert prob.shape == (n, 4 * h, 4 * w)
    p = prob.cpu().numpy()
    assert 1e-3 < p.std() and p.min() >= 0 and p.max() <= 1


def test_conv_tc_rejects_unsupported_shapes(tocr):
    L = tocr.lib()
    assert L.tocr_conv_tc_f16(None, 1, 8, 8, 64, 24, 3, None, None, 0, None, None, None,
                              None) == 1
    assert L.tocr_conv_tc_packed_bytes(96, 24, 3) == 9 * 2 * 32 * 128
