"""The allocation-free CTC entry (tocr_ctc_greedy_f16_noalloc, scratch in a
static device array) against the caller-buffer entry tocr_ctc_greedy_f16:
two calls in a row on different inputs must both reproduce the existing
entry's outputs exactly, and sizes beyond the static scratch are refused.
Collected last on purpose (file name), so it also runs after every other
GPU test in the same process."""
import pytest
import torch

from turboocr_b200 import kernels as K
from turboocr_b200._lib import InvalidArgument, call

pytestmark = pytest.mark.gpu

MAX_STEPS = 1 << 20


def noalloc(logits, num_labels):
    B, T, V = logits.shape
    tokens = torch.full((B * T,), -7, dtype=torch.int32, device=logits.device)
    lengths = torch.full((B,), -7, dtype=torch.int32, device=logits.device)
    scores = torch.full((B,), -7.0, dtype=torch.float32, device=logits.device)
    call("tocr_ctc_greedy_f16_noalloc", logits.data_ptr(), B, T, V, num_labels,
         tokens.data_ptr(), lengths.data_ptr(), scores.data_ptr(),
         torch.cuda.current_stream().cuda_stream)
    return tokens, lengths, scores


def existing(logits, num_labels):
    B, T, V = logits.shape
    out = K.CtcOutputs(B, T, logits.device)
    K.ctc_greedy_f16(logits, num_labels, out)
    return out.tokens, out.lengths, out.scores


def same(a, b):
    ta, la, sa = a
    tb, lb, sb = b
    assert torch.equal(la, lb)
    B = la.numel()
    T = ta.numel() // B
    for r in range(B):
        n = int(la[r])
        assert torch.equal(ta[r * T: r * T + n], tb[r * T: r * T + n]), r
    assert torch.equal(sa, sb)


def test_noalloc_matches_existing_entry_twice(cuda):
    g = torch.Generator(device="cuda").manual_seed(1234)
    V, labels = 18385, 18384
    a = (torch.randn(512, 80, V, generator=g, device=cuda) * 4).half()
    b = (torch.randn(37, 25, V, generator=g, device=cuda) * 4).half()
    a[:, ::3, 0] += 30.0      # blank runs so lines collapse
    r1 = noalloc(a, labels)
    r2 = noalloc(b, labels)
    torch.cuda.synchronize()
    same(r1, existing(a, labels))
    same(r2, existing(b, labels))
    torch.cuda.synchronize()


def test_noalloc_limit(cuda):
    x = torch.zeros(1, 1, 8, dtype=torch.float16, device=cuda)
    t = torch.zeros(1, dtype=torch.int32, device=cuda)
    with pytest.raises(InvalidArgument, match="exceeds the static scratch"):
        call("tocr_ctc_greedy_f16_noalloc", x.data_ptr(), MAX_STEPS + 1, 1, 8, 8,
             t.data_ptr(), t.data_ptr(), t.data_ptr(), torch.cuda.current_stream().cuda_stream)
    # exactly at the limit is accepted
    big = torch.zeros(MAX_STEPS, 1, 8, dtype=torch.float16, device=cuda)
    big[:, 0, 3] = 1.0
    toks, lens, scores = noalloc(big, 8)
    ref = existing(big, 8)
    torch.cuda.synchronize()
    same((toks, lens, scores), ref)
