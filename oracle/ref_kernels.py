"""ORACLE (test infrastructure only): the reference's own CUDA kernels
(src/kernels/preprocess_kernels.cu, src/kernels/reduce_kernels.cu,
src/kernels/jfa.cu) compiled
unchanged into oracle/_ref/libref_kernels.so. GPU tests use them to pin the
fp32 arithmetic of the B200 kernels bit for bit."""
from __future__ import annotations

import ctypes as C

from ._loader import load


def lib():
    L = load("_ref/libref_kernels.so")
    if not getattr(L, "_tocr_ready", False):
        L.refk_batch_preprocess.argtypes = [C.c_void_p] * 7 + [C.c_int] * 3 + [C.c_void_p]
        L.refk_argmax.argtypes = [C.c_void_p] * 3 + [C.c_int] * 3 + [C.c_void_p]
        L.refk_threshold.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                     C.c_float, C.c_void_p]
        L.refk_roi_warp.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_longlong, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                    C.c_void_p]
        L.refk_fused_single.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_longlong, C.c_void_p,
                                        C.c_int, C.c_int, C.c_void_p]
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        L.refk_jfa_crack.argtypes = [vp, vp, i, i, i, vp, vp]
        L.refk_jfa_expand_per_comp.argtypes = [vp, vp, i, f, f, f, f, vp, vp]
        L.refk_jfa_expand_labels.argtypes = [vp, vp, vp, vp, i, i, f, vp, vp, vp]
        L.refk_jfa_extract_bboxes.argtypes = [vp, i, i, vp, i, vp]
        L.refk_jfa_extract_oriented.argtypes = [vp, i, i, vp, i, vp, vp, vp]
        L._tocr_ready = True
    return L


def batch_preprocess(meta, out_f32, stream=0):
    """cuda_batch_fused_resize_normalize_det on the same descriptor arrays."""
    B, _, H, W = out_f32.shape
    st = lib().refk_batch_preprocess(meta.ptrs.data_ptr(), meta.steps.data_ptr(),
                                     meta.src_h.data_ptr(), meta.src_w.data_ptr(),
                                     meta.dst_h.data_ptr(), meta.dst_w.data_ptr(),
                                     out_f32.data_ptr(), W, H, B, stream)
    assert st == 0


def argmax(probs, idx, val, stream=0):
    B, T, V = probs.shape
    assert lib().refk_argmax(probs.data_ptr(), idx.data_ptr(), val.data_ptr(), B, T, V,
                             stream) == 0


def threshold(src, dst, w, h, batch, t, stream=0):
    assert lib().refk_threshold(src.data_ptr(), dst.data_ptr(), w, h, batch, t, stream) == 0
