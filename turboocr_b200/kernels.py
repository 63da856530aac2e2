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


# ---- subsystem 3 ------------------------------------------------------------

DB_STATUS_BITS = {1: "point pool full", 2: "border walk exceeded its bound",
                  4: "geometry scratch pool full", 8: "more boxes than max_boxes (truncated)",
                  16: "union sweep out of bounds (raw offset ring used)"}


class DbPostprocess:
    """Device DB post-process for batches of [n_maps, h, w] fp32 maps
    (extract_boxes_from_bitmap, src/detection/det_postprocess.cpp:145-222,
    with the threshold fused). Owns its workspace and output buffers; the
    defaults are the reference's (thresh 0.3, box_thresh 0.6, unclip 1.5,
    kMinBoxSide 3, kMinUnclippedSide 5 — paddle_det.h:62-63)."""

    def __init__(self, n_maps: int, h: int, w: int, device, max_boxes: int = 1000,
                 thresh: float = 0.3, box_thresh: float = 0.6, unclip_ratio: float = 1.5,
                 min_box_side: float = 3.0, min_unclipped_side: float = 5.0,
                 point_cap: int = 0, offset_cap: int = 0):
        from ._lib import lib
        self.n_maps, self.h, self.w, self.max_boxes = n_maps, h, w, max_boxes
        self.params = (thresh, box_thresh, unclip_ratio, min_box_side, min_unclipped_side)
        self.caps = (point_cap, offset_cap)
        nbytes = lib().tocr_db_workspace_bytes(n_maps, h, w, point_cap, offset_cap)
        self.workspace = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        off = (-self.workspace.data_ptr()) % 256
        self.ws_ptr, self.ws_bytes = self.workspace.data_ptr() + off, nbytes
        self.boxes = torch.zeros(n_maps, max_boxes, 4, 2, dtype=torch.int32, device=device)
        self.scores = torch.zeros(n_maps, max_boxes, dtype=torch.float32, device=device)
        self.counts = torch.zeros(n_maps, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)

    def __call__(self, pred: torch.Tensor, geometry: torch.Tensor | None = None,
                 stream=None) -> None:
        n, h, w = pred.shape
        assert pred.dtype == torch.float32 and (h, w) == (self.h, self.w) and n <= self.n_maps
        call("tocr_db_postprocess", _ptr(pred), n, h, w, _ptr(geometry), *self.params,
             *self.caps, self.ws_ptr, self.ws_bytes, _ptr(self.boxes), _ptr(self.scores),
             _ptr(self.counts), self.max_boxes, _ptr(self.status), _stream(stream))

    def results(self, n: int | None = None) -> list[list[tuple[list[list[int]], float]]]:
        """Per map: [(quad [[x, y] * 4], score)] in contour order (synchronises)."""
        st = int(self.status.item())
        if st & 23:
            msgs = [m for b, m in DB_STATUS_BITS.items() if st & b]
            raise RuntimeError("tocr_db_postprocess: " + ", ".join(msgs))
        n = self.n_maps if n is None else n
        counts = self.counts[:n].cpu().tolist()
        boxes = self.boxes[:n].cpu()
        scores = self.scores[:n].cpu()
        return [[(boxes[m, k].tolist(), float(scores[m, k])) for k in range(counts[m])]
                for m in range(n)]


def db_components(pred: torch.Tensor, thresh: float = 0.3, stream=None, shortcuts: bool = True):
    """(labels int32 [n, h, w], bitmap u8 [n, h, w]) of the labelling stage
    (with the background-tile shortcuts of the full DB stage by default)."""
    from ._lib import lib
    n, h, w = pred.shape
    labels = torch.empty(n, h, w, dtype=torch.int32, device=pred.device)
    bitmap = torch.empty(n, h, w, dtype=torch.uint8, device=pred.device)
    scratch = None
    if shortcuts:
        scratch = torch.empty(lib().tocr_db_components_scratch_bytes(n, h, w), dtype=torch.uint8,
                              device=pred.device)
    call("tocr_db_components", _ptr(pred), n, h, w, thresh, _ptr(labels), _ptr(bitmap),
         _ptr(scratch), _stream(stream))
    return labels, bitmap
