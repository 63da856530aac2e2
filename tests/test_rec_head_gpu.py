"""The fused recognizer head (tocr_rec_head_ctc_f16): logits formed on the
tensor cores and reduced in place, against a torch fp32 restatement of the
same layer (logits = features @ W^T + bias, TF32 off) followed by the
reference decode rule: per step the argmax (lowest index on ties) and
p = 1 / sum exp(l - l_max), then the greedy collapse of ctc_decode.cpp:25-88
(restated in oracle/ctc_oracle.py). Argmax indices must be equal wherever
the reference's top two logits differ by more than the fp32 summation-order
noise; within that margin either of the two is accepted."""
import numpy as np
import pytest
import torch

from oracle import ctc_oracle as co

pytestmark = pytest.mark.gpu

GAP = 1e-3     # logit margin above which the argmax must match exactly
P_RTOL = 1e-4  # max-softmax probability


def run_head(L, feat, w, bias, B, T, num_labels, dev):
    K, V = feat.shape[1], w.shape[0]
    rows = B * T
    toks = torch.zeros(rows, dtype=torch.int32, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    sc = torch.zeros(B, dtype=torch.float32, device=dev)
    sidx = torch.full((rows,), -1, dtype=torch.int32, device=dev)
    sprob = torch.full((rows,), -1.0, dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = L.tocr_rec_head_ctc_f16(feat.data_ptr(), B, T, K, w.data_ptr(), bias.data_ptr(), V,
                                 num_labels, toks.data_ptr(), lens.data_ptr(), sc.data_ptr(),
                                 sidx.data_ptr(), sprob.data_ptr(), err.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.tocr_last_error_string()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return (sidx.cpu().numpy(), sprob.cpu().numpy(), toks.cpu().numpy().reshape(B, T),
            lens.cpu().numpy(), sc.cpu().numpy())


def reference(feat, w, bias):
    torch.backends.cuda.matmul.allow_tf32 = False
    logits = feat.float() @ w.float().T + bias
    top2, i2 = torch.topk(logits, 2, dim=1)
    m = top2[:, :1]
    p = 1.0 / torch.exp(logits - m).sum(dim=1)
    first = (logits == m).float().argmax(dim=1)  # lowest index of the maximum
    return (first.cpu().numpy().astype(np.int32), i2[:, 1].cpu().numpy(),
            (top2[:, 0] - top2[:, 1]).cpu().numpy(), p.cpu().numpy())


def make_case(B, T, K, V, seed, dev, gain=3.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    feat = torch.randn(B * T, K, generator=g).to(torch.float16)
    w = (torch.randn(V, K, generator=g) * (gain / K ** 0.5)).to(torch.float16)
    bias = (torch.randn(V, generator=g) * 0.5).float()
    # plant a clear winner on some steps so lines have tokens and blanks
    tok = torch.randint(0, V, (B * T,), generator=g)
    plant = torch.rand(B * T, generator=g) < 0.5
    feat_f = feat.float()
    for r in torch.nonzero(plant).flatten().tolist():
        feat_f[r] = w[tok[r]].float() * (4.0 * K ** 0.5 / gain)
    feat = feat_f.clamp(-60000, 60000).to(torch.float16)
    return feat.to(dev), w.to(dev), bias.to(dev)


@pytest.mark.parametrize("B,T,K,V", [(32, 80, 128, 18385), (7, 25, 64, 5000), (3, 20, 128, 300)])
def test_rec_head_matches_fp32_reference(tocr, cuda, B, T, K, V):
    feat, w, bias = make_case(B, T, K, V, 100 + K + V, cuda)
    num_labels = V - 2
    sidx, sprob, toks, lens, sc = run_head(tocr.lib(), feat, w, bias, B, T, num_labels, cuda)
    ridx, rsecond, gap, rp = reference(feat, w, bias)
    sure = gap > GAP
    assert sure.mean() > 0.95
    assert np.array_equal(sidx[sure], ridx[sure])
    near = ~sure
    assert np.all((sidx[near] == ridx[near]) | (sidx[near] == rsecond[near]))
    assert np.allclose(sprob, rp, rtol=P_RTOL, atol=0)
    # collapse of the device steps: the reference rule on the same (idx, p)
    for b in range(B):
        want, want_score = co.collapse(sidx[b * T:(b + 1) * T].tolist(),
                                       sprob[b * T:(b + 1) * T], num_labels)
        assert lens[b] == len(want) and toks[b, :lens[b]].tolist() == want
        assert abs(sc[b] - want_score) <= 1e-6
    assert lens.sum() > 0


def test_rec_head_arguments(tocr):
    L = tocr.lib()
    args = [None, 1, 4, 96, None, None, 10, 8] + [None] * 6 + [None]
    assert L.tocr_rec_head_ctc_f16(*args) == 1  # K must be 64 or 128
    args[3] = 128
    assert L.tocr_rec_head_ctc_f16(*args) == 1  # null pointers
    args[1] = 0
    assert L.tocr_rec_head_ctc_f16(*args) == 0  # empty batch
