"""ctypes binding of the C-ABI (include/tocr_capi.h).

The product library is loaded from this package directory only. If it is
missing the import fails loudly: there is no CPU fallback on this path.
Status codes are mapped to the reference's exception types
(include/turbo_ocr/common/errors.h in TurboOCR): OcrError, CudaError,
InferenceError, TimeoutError.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent

TOCR_OK = 0
TOCR_ERR_INVALID = 1
TOCR_ERR_CUDA = 2
TOCR_ERR_OVERFLOW = 3
TOCR_ERR_TIMEOUT = 4
TOCR_ERR_INJECTED = 5


class OcrError(RuntimeError):
    """Base of the reference's error hierarchy."""


class CudaError(OcrError):
    pass


class InferenceError(OcrError):
    pass


class TimeoutError(OcrError):  # noqa: A001 - mirrors turbo_ocr::TimeoutError
    pass


class InvalidArgument(CudaError, ValueError):
    """TOCR_ERR_INVALID / TOCR_ERR_OVERFLOW (the reference raises CudaError
    with cudaErrorInvalidValue for these, reduce_kernels.cu:140-142)."""


_vp = C.c_void_p
_i = C.c_int
_f = C.c_float
_ll = C.c_longlong
_u64 = C.c_uint64

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "tocr_last_error_string": (C.c_char_p, []),
    "tocr_version": (_i, []),
    "tocr_debug_inject_error": (None, [_i, _i]),
    "tocr_debug_db_shared_columns": (None, [_i]),
    "tocr_argmax_f32": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "tocr_ctc_greedy_f16": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "tocr_ctc_greedy_f16_noalloc": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "tocr_preprocess_batch_f16": (_i, [_vp] * 7 + [_i, _i, _i, _vp, _vp, _vp]),
    "tocr_preprocess_batch_f32": (_i, [_vp] * 7 + [_i, _i, _i, _vp, _vp, _vp]),
    "tocr_threshold_u8": (_i, [_vp, _vp, _i, _i, _i, _f, _vp]),
    "tocr_dwpw_block": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "tocr_dwpw_packed_bytes": (C.c_size_t, [_i, _i]),
    "tocr_dwpw_pack": (_i, [_i, _i, _i, _vp, _vp, _vp, _vp, _vp, C.c_size_t]),
    "tocr_dwpw_dequant_pw": (_i, [_vp, _i, _i, _i, _vp]),
    "tocr_db_workspace_bytes": (C.c_size_t, [_i, _i, _i, _ll, _ll]),
    "tocr_db_postprocess": (_i, [_vp, _i, _i, _i, _vp, _f, _f, _f, _f, _f, _ll, _ll, _vp,
                                 C.c_size_t, _vp, _vp, _vp, _i, _vp, _vp]),
    "tocr_db_components_scratch_bytes": (C.c_size_t, [_i, _i, _i]),
    "tocr_db_components": (_i, [_vp, _i, _i, _i, _f, _vp, _vp, _vp, _vp]),
    "tocr_stem_params_bytes": (C.c_size_t, []),
    "tocr_stem_pack": (_i, [_vp, _vp, _vp, _vp, _vp, C.c_size_t]),
    "tocr_stem_take_error": (_i, [_vp]),
    "tocr_stem_f16": (_i, [_vp, _i, _i, _i, _ll, _vp, _vp, _vp]),
    "tocr_ink_map": (_i, [_vp, _i, _i, _i, _ll, _f, _vp, _vp]),
    "tocr_head_sigmoid": (_i, [_vp, _ll, _i, _vp, _f, _vp, _vp]),
    "tocr_crop_transforms": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "tocr_roi_warp_f16": (_i, [_vp, _ll, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _f,
                               _vp, _vp]),
    "tocr_ctc_greedy_f16_dev": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "tocr_preprocess_one_f32": (_i, [_vp, _i, _i, _i, _vp, _i, _i, _vp, _vp, _vp]),
    "tocr_preprocess_one_f16": (_i, [_vp, _i, _i, _i, _vp, _i, _i, _vp, _vp, _vp]),
    "tocr_roi_warp_f32": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _i, _vp, _vp, _f, _vp, _vp]),
    "tocr_det_standin_prob_f32": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _f, _vp, _vp]),
    "tocr_rec_standin_logits_f16": (_i, [_vp, _vp, _i, _i, _i, _u64, _vp]),
    "tocr_gpu_ccl_detect": (_i, [_vp, _vp, _i, _i, _f, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _vp]),
    "tocr_jfa_crack_perimeter": (_i, [_vp, _vp, _i, _i, _i, _vp, _vp]),
    "tocr_jfa_expand_per_comp": (_i, [_vp, _vp, _i, _f, _f, _f, _f, _vp, _vp]),
    "tocr_jfa_expand_labels": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "tocr_jfa_extract_bboxes": (_i, [_vp, _i, _i, _vp, _i, _vp]),
    "tocr_jfa_extract_oriented": (_i, [_vp, _i, _i, _vp, _i, _vp, _vp, _vp]),
    "tocr_rec_head_ctc_f16": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp,
                                   _vp, _vp]),
    "tocr_conv_tc_packed_bytes": (C.c_size_t, [_i, _i, _i]),
    "tocr_conv_tc_pack": (_i, [_i, _i, _i, _vp, _vp, C.c_size_t]),
    "tocr_conv_tc_f16": (_i, [_vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _i, _vp, _vp, _vp, _vp]),
    "tocr_fpn_concat_f16": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "tocr_db_head_up_f32": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _f, _vp, _vp]),
    "tocr_cls_stem_f16": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "tocr_cls_head_f32": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "tocr_synth_weights": (_i, [_u64, _f, _vp, _ll]),
    "tocr_png_peek": (_i, [_vp, C.c_size_t, _i, _ll, _vp]),
    "tocr_png_decode_batch": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp]),
    "tocr_compute_det_resize": (_i, [_i, _i, _i, _i, _i, _vp, _vp]),
    "tocr_read_det_resize": (_i, [_vp, _vp, _vp]),
    "tocr_effective_det_max_side": (_i, [_i]),
    "tocr_read_db_params": (_i, [_vp, _vp, _vp]),
}

SYNTH_SIGNATURES: dict[str, tuple] = {
    "tocr_synth_hash": (_u64, [_u64, _u64, _u64]),
    "tocr_synth_fill_u8": (_i, [_vp, _ll, _u64, _u64, _vp]),
    "tocr_synth_normal_f16": (_i, [_vp, _ll, _f, _u64, _u64, _vp]),
    "tocr_synth_ctc_logits": (_i, [_vp, _vp, _i, _i, _i, _u64, _vp]),
    "tocr_synth_db_map_host": (_i, [_vp, _i, _i, _i, _i, _u64, _u64]),
    "tocr_synth_pages": (_i, [_vp, _i, _i, _i, _u64, _ll, _vp]),
    "tocr_synth_rec_logits": (_i, [_vp, _vp, _i, _i, _i, _u64, _vp]),
}


def _load(name: str, sigs: dict) -> C.CDLL:
    path = PKG / name
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m turboocr_b200.build` "
            "(the B200 path has no CPU fallback)")
    lib = C.CDLL(str(path))
    for fn, (res, args) in sigs.items():
        f = getattr(lib, fn)
        f.restype = res
        f.argtypes = args
    return lib


_LIB: C.CDLL | None = None
_SYNTH: C.CDLL | None = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _load("libtocr_b200.so", SIGNATURES)
    return _LIB


def synth() -> C.CDLL:
    global _SYNTH
    if _SYNTH is None:
        _SYNTH = _load("libtocr_synth.so", SYNTH_SIGNATURES)
    return _SYNTH


def last_error() -> str:
    return lib().tocr_last_error_string().decode()


def check(status: int, where: str) -> None:
    """Raise the reference exception matching a C-ABI status."""
    if status == TOCR_OK:
        return
    msg = f"{where}: {last_error()}"
    if status in (TOCR_ERR_INVALID, TOCR_ERR_OVERFLOW):
        raise InvalidArgument(msg)
    if status == TOCR_ERR_TIMEOUT:
        raise TimeoutError(msg)
    if status == TOCR_ERR_INJECTED:
        raise InferenceError(msg)
    raise CudaError(msg)


def call(fn: str, *args) -> None:
    check(getattr(lib(), fn)(*args), fn)
