"""Subsystem 4 parity on the GPU: the fused fp16 CTC decode (C-ABI
tocr_ctc_greedy_f16) against the reference's own ctc_decode.cpp fed with
the softmax of the same logits. Token indices must match exactly; the line
confidence (mean max-softmax) within 1e-3."""
import numpy as np
import pytest
import torch

from oracle import ctc_oracle as co

pytestmark = pytest.mark.gpu

SCORE_TOL = 1e-3


def run_gpu(tocr, logits_f16: torch.Tensor, num_labels: int):
    from turboocr_b200 import kernels as K
    B, T, V = logits_f16.shape
    out = K.CtcOutputs(B, T, logits_f16.device)
    K.ctc_greedy_f16(logits_f16, num_labels, out)
    torch.cuda.synchronize()
    return K.ctc_results(out), out


def check_lines(tocr, logits_f16, num_labels, lines=None):
    res, out = run_gpu(tocr, logits_f16, num_labels)
    host = logits_f16.cpu().numpy()
    B = host.shape[0]
    lines = range(B) if lines is None else lines
    for b in lines:
        ref_toks, ref_score = co.decode_logits(host[b], num_labels)
        toks, score = res[b]
        assert toks == ref_toks, f"line {b}"
        assert abs(score - ref_score) <= SCORE_TOL, (b, score, ref_score)
    return res, out


@pytest.mark.parametrize("V", [1, 2, 7, 8, 9, 31, 255, 1000, 18385])
def test_random_small(tocr, cuda, V):
    g = torch.Generator(device="cpu").manual_seed(V)
    B, T = 5, 23
    x = (torch.randn(B, T, V, generator=g) * 4).to(torch.float16).to(cuda)
    check_lines(tocr, x, V)


def test_ties_take_lowest_index(tocr, cuda):
    B, T, V = 3, 16, 777
    x = torch.full((B, T, V), -5.0, dtype=torch.float16)
    for t in range(T):
        for b in range(B):
            # equal maxima at several indices, across chunk and lane boundaries
            for j in (3 + t + b, 300 + t, 776 - t):
                x[b, t, j] = 7.0
    x = x.to(cuda)
    res, out = check_lines(tocr, x, V)
    idx = out.step_idx.view(B, T).cpu()
    for b in range(B):
        for t in range(T):
            assert int(idx[b, t]) == 3 + t + b


def test_blank_and_label_range(tocr, cuda):
    B, T, V = 4, 40, 300
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(B, T, V, generator=g)).to(torch.float16)
    x[0] = -3.0
    x[0, :, 0] = 5.0           # all blank -> empty, score 0
    x[1, ::2, 250] = 9.0       # indices beyond num_labels are dropped
    x = x.to(cuda)
    res, _ = check_lines(tocr, x, num_labels=200)
    assert res[0] == ([], 0.0)


@pytest.mark.parametrize("offset", [1, 2, 3, 5, 7])
def test_misaligned_rows(tocr, cuda, offset):
    B, T, V = 2, 9, 1001
    g = torch.Generator().manual_seed(offset)
    base = (torch.randn(B * T * V + 16, generator=g) * 3).to(torch.float16).to(cuda)
    x = base[offset:offset + B * T * V].view(B, T, V)
    res, out = run_gpu(tocr, x, V)
    host = x.cpu().numpy()
    for b in range(B):
        assert res[b][0] == co.decode_logits(host[b], V)[0]


def test_zero_steps(tocr, cuda):
    from turboocr_b200 import kernels as K
    x = torch.empty(3, 0, 50, dtype=torch.float16, device=cuda)
    out = K.CtcOutputs(3, 0, cuda)
    K.ctc_greedy_f16(x, 50, out)
    assert K.ctc_results(out) == [([], 0.0)] * 3


def test_config2_full_size(tocr, cuda):
    """BASELINE config 2 at full size: 512 x 80 x 18385 fp16 logits from the
    seeded generator. Planted steps must decode to their planted index on
    every line; 24 lines are compared in full against the oracle."""
    from turboocr_b200._lib import synth
    B, T, V = 512, 80, 18385
    x = torch.empty(B, T, V, dtype=torch.float16, device=cuda)
    plan = torch.empty(B * T, dtype=torch.int32, device=cuda)
    assert synth().tocr_synth_ctc_logits(x.data_ptr(), plan.data_ptr(), B, T, V,
                                         0x7EC00001, None) == 0
    res, out = run_gpu(tocr, x, V)
    plan = plan.view(B, T).cpu()
    idx = out.step_idx.view(B, T).cpu()
    planted = plan >= 0
    assert torch.equal(idx[planted], plan[planted])
    host = x[:24].cpu().numpy()
    for b in range(24):
        ref_toks, ref_score = co.decode_logits(host[b], V)
        assert res[b][0] == ref_toks
        assert abs(res[b][1] - ref_score) <= SCORE_TOL


def test_argmax_f32_matches_reference_contract(tocr, cuda):
    from turboocr_b200 import kernels as K
    g = torch.Generator().manual_seed(11)
    B, T, V = 4, 30, 6907
    x = torch.rand(B, T, V, generator=g)
    x[0, 0, 100] = 2.0
    x[0, 0, 200] = 2.0
    xd = x.to(cuda)
    idx = torch.empty(B * T, dtype=torch.int32, device=cuda)
    val = torch.empty(B * T, dtype=torch.float32, device=cuda)
    K.cuda_argmax(xd, idx, val)
    torch.cuda.synchronize()
    flat = x.view(B * T, V).numpy()
    assert np.array_equal(idx.cpu().numpy(), flat.argmax(axis=1))
    assert np.array_equal(val.cpu().numpy(), flat.max(axis=1))
    assert int(idx[0]) == 100


def test_argmax_bit_exact_vs_reference_kernel(tocr, cuda):
    from oracle import ref_kernels as rk
    from turboocr_b200 import kernels as K
    g = torch.Generator().manual_seed(12)
    B, T, V = 8, 40, 18385
    x = torch.rand(B, T, V, generator=g)
    x[1, 3, 5] = x[1, 3, 4000] = 5.0  # tie
    xd = x.to(cuda)
    i1 = torch.empty(B * T, dtype=torch.int32, device=cuda)
    v1 = torch.empty(B * T, dtype=torch.float32, device=cuda)
    i2, v2 = torch.empty_like(i1), torch.empty_like(v1)
    K.cuda_argmax(xd, i1, v1)
    rk.argmax(xd, i2, v2)
    torch.cuda.synchronize()
    assert torch.equal(i1, i2) and torch.equal(v1, v2)
