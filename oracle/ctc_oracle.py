"""ORACLE (test infrastructure only) for subsystem 4, CTC greedy decode.

* ``ref_decode_raw`` / ``ref_decode`` run the reference's own
  src/recognition/ctc_decode.cpp (ctc_greedy_decode_raw :69-92,
  ctc_greedy_decode :25-48), compiled unchanged into oracle/_ref/.
* ``collapse`` is a plain-Python restatement of the same collapse rule
  (ctc_decode.cpp:25-48), pinned against the reference's known-answer tests
  (tests/recognition/test_ctc_decode.cpp:14-88) in tests/test_oracle_ctc.py.
* ``softmax_probs`` turns fp16 logits into the fp32 probabilities a PP-OCR
  recognition head emits, so that the reference decode sees probs and its
  score is the mean max-softmax of the emitted steps.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._loader import load

_P = C.POINTER


def _lib(simd: bool) -> C.CDLL:
    name = "_ref/libctc_ref_simd.so" if simd else "_ref/libctc_ref_scalar.so"
    lib = load(name)
    if not getattr(lib, "_tocr_ready", False):
        lib.ctc_ref_init.argtypes = [C.c_int]
        lib.ctc_ref_init(1 if simd else 0)
        lib.ctc_ref_decode_raw.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                           _P(C.c_float)]
        lib.ctc_ref_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                       _P(C.c_float)]
        lib.ctc_ref_decode_batch.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                             C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        lib._tocr_ready = True
    return lib


def ref_decode_raw(probs: np.ndarray, num_labels: int, simd: bool = False):
    """Reference ctc_greedy_decode_raw on fp32 probs [T, V] -> (tokens, score)."""
    probs = np.ascontiguousarray(probs, dtype=np.float32)
    T, V = probs.shape
    toks = np.zeros(max(T, 1), dtype=np.int32)
    sc = C.c_float()
    n = _lib(simd).ctc_ref_decode_raw(probs.ctypes.data, T, V, num_labels, toks.ctypes.data,
                                      C.byref(sc))
    return toks[:n].tolist(), sc.value


def ref_decode(indices, scores, num_labels: int):
    """Reference ctc_greedy_decode on per-step (index, score) -> (tokens, score)."""
    idx = np.ascontiguousarray(indices, dtype=np.int32)
    s = np.ascontiguousarray(scores, dtype=np.float32)
    toks = np.zeros(max(len(idx), 1), dtype=np.int32)
    sc = C.c_float()
    n = _lib(False).ctc_ref_decode(idx.ctypes.data if len(idx) else None,
                                   s.ctypes.data if len(s) else None, len(idx), num_labels,
                                   toks.ctypes.data, C.byref(sc))
    return toks[:n].tolist(), sc.value


def ref_decode_batch(logits_f32: np.ndarray, num_labels: int, n_threads: int, simd: bool):
    """CPU baseline: reference decode_raw over [B, T, V] plus the per-step
    softmax maximum, lines spread over n_threads std::threads."""
    B, T, V = logits_f32.shape
    toks = np.zeros((B, T), dtype=np.int32)
    lens = np.zeros(B, dtype=np.int32)
    sc = np.zeros(B, dtype=np.float32)
    _lib(simd).ctc_ref_decode_batch(logits_f32.ctypes.data, B, T, V, num_labels, n_threads,
                                    toks.ctypes.data, lens.ctypes.data, sc.ctypes.data)
    return toks, lens, sc


def collapse(indices, scores, num_labels: int):
    """Restatement of ctc_decode.cpp:25-48: emit idx when idx != last,
    idx != 0 and idx < num_labels; score = fp32 sequential mean."""
    out, total, last = [], np.float32(0.0), -1
    for i, idx in enumerate(indices):
        idx = int(idx)
        if idx != last and idx != 0 and idx < num_labels:
            out.append(idx)
            total = np.float32(total + np.float32(scores[i]))
        last = idx
    score = np.float32(total / np.float32(len(out))) if out else np.float32(0.0)
    return out, float(score)


def softmax_probs(logits_f16: np.ndarray) -> np.ndarray:
    """fp32 softmax over the last axis, computed in float64."""
    x = logits_f16.astype(np.float64)
    x = x - x.max(axis=-1, keepdims=True)
    e = np.exp(x)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def decode_logits(logits_f16: np.ndarray, num_labels: int, simd: bool = False):
    """Oracle for one line of fp16 logits [T, V]: (tokens, mean max-softmax)."""
    return ref_decode_raw(softmax_probs(logits_f16), num_labels, simd)
