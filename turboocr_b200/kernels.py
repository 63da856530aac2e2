"""Tensor-level wrappers with the reference kernel names
(turbo_ocr::kernels::cuda_*, include/turbo_ocr/kernels/kernels.h in TurboOCR)
plus the fused B200 entries. Arguments are CUDA torch tensors; work is
enqueued on torch's current stream (or ``stream=``) and returns immediately.
Caller-owned outputs are passed in, as in the reference (no allocation in
the call); convenience allocators are provided separately.
"""
from __future__ import annotations

import torch

from ._lib import call


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("tensor must live on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def _stream(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream if hasattr(s, "cuda_stream") else int(s)


# ---- subsystem 4 ------------------------------------------------------------

def cuda_argmax(probs: torch.Tensor, out_idx: torch.Tensor, out_val: torch.Tensor,
                stream=None) -> None:
    """reduce_kernels.cu:85-93 — probs fp32 [B, T, V] -> idx int32 [B*T], max fp32 [B*T]."""
    B, T, V = probs.shape
    assert probs.dtype == torch.float32 and out_idx.dtype == torch.int32
    call("tocr_argmax_f32", _ptr(probs), _ptr(out_idx), _ptr(out_val), B, T, V, _stream(stream))


class CtcOutputs:
    """Caller-owned output buffers of ctc_greedy_f16 for a [B, T] problem."""

    def __init__(self, batch: int, seq_len: int, device):
        self.tokens = torch.empty(batch * seq_len, dtype=torch.int32, device=device)
        self.lengths = torch.empty(batch, dtype=torch.int32, device=device)
        self.scores = torch.empty(batch, dtype=torch.float32, device=device)
        self.step_idx = torch.empty(batch * seq_len, dtype=torch.int32, device=device)
        self.step_prob = torch.empty(batch * seq_len, dtype=torch.float32, device=device)
        self.batch, self.seq_len = batch, seq_len


def ctc_greedy_f16(logits: torch.Tensor, num_labels: int, out: CtcOutputs, stream=None) -> None:
    """Fused argmax + softmax-max + collapse on fp16 logits [B, T, V]."""
    B, T, V = logits.shape
    assert logits.dtype == torch.float16
    assert out.batch >= B and out.seq_len == T
    call("tocr_ctc_greedy_f16", _ptr(logits), B, T, V, num_labels, _ptr(out.tokens),
         _ptr(out.lengths), _ptr(out.scores), _ptr(out.step_idx), _ptr(out.step_prob),
         _stream(stream))


def ctc_results(out: CtcOutputs, batch: int | None = None) -> list[tuple[list[int], float]]:
    """Host copy of (token list, score) per line (synchronises the stream)."""
    B = out.batch if batch is None else batch
    toks = out.tokens[: B * out.seq_len].view(B, out.seq_len).cpu()
    lens = out.lengths[:B].cpu()
    sc = out.scores[:B].cpu()
    return [(toks[b, : int(lens[b])].tolist(), float(sc[b])) for b in range(B)]


# ---- subsystem 1 ------------------------------------------------------------

class PreprocessMeta:
    """Device-side per-image descriptor arrays of a preprocessing batch
    (the d_src_* / d_dst_* arrays of preprocess_kernels.cu:180-201)."""

    def __init__(self, ptrs, steps, src_hw, dst_hw, device):
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.steps = torch.tensor(steps, dtype=torch.int32, device=device)
        self.src_h = torch.tensor([h for h, _ in src_hw], dtype=torch.int32, device=device)
        self.src_w = torch.tensor([w for _, w in src_hw], dtype=torch.int32, device=device)
        self.dst_h = torch.tensor([h for h, _ in dst_hw], dtype=torch.int32, device=device)
        self.dst_w = torch.tensor([w for _, w in dst_hw], dtype=torch.int32, device=device)
        self.n = len(ptrs)


def preprocess_batch(meta: PreprocessMeta, out: torch.Tensor, mean=None, inv_std=None,
                     stream=None) -> None:
    """Batched resize+letterbox+normalise into out [B, 3, H, W] (fp16 or fp32)."""
    B, C, H, W = out.shape
    assert C == 3 and B == meta.n
    import ctypes
    m = (ctypes.c_float * 3)(*mean) if mean is not None else None
    s = (ctypes.c_float * 3)(*inv_std) if inv_std is not None else None
    fn = "tocr_preprocess_batch_f16" if out.dtype == torch.float16 else "tocr_preprocess_batch_f32"
    call(fn, _ptr(meta.ptrs), _ptr(meta.steps), _ptr(meta.src_h), _ptr(meta.src_w),
         _ptr(meta.dst_h), _ptr(meta.dst_w), _ptr(out), W, H, B,
         ctypes.cast(m, ctypes.c_void_p) if m is not None else None,
         ctypes.cast(s, ctypes.c_void_p) if s is not None else None, _stream(stream))


def cuda_batch_threshold_to_u8(src: torch.Tensor, dst: torch.Tensor, w: int, h: int,
                               batch: int, thresh: float, stream=None) -> None:
    call("tocr_threshold_u8", _ptr(src), _ptr(dst), w, h, batch, float(thresh), _stream(stream))
