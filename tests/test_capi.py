"""C-ABI library: loads, exports every symbol tocr_capi.h declares, validates
arguments and honours host-side fault injection — all without a GPU."""
import ctypes as C
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "tocr_capi.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TOCR_API\s+[\w\s\*]+?\b(tocr_\w+)\s*\(", text)))


def test_header_declares_entries():
    syms = declared_symbols()
    assert "tocr_ctc_greedy_f16" in syms and "tocr_preprocess_batch_f16" in syms
    assert len(syms) >= 8


def test_library_exports_every_declared_symbol(tocr):
    lib = tocr.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_bindings_cover_header(tocr):
    from turboocr_b200._lib import SIGNATURES
    assert set(declared_symbols()) <= set(SIGNATURES)


def test_version(tocr):
    assert tocr.lib().tocr_version() >= 0x000100


def test_invalid_arguments_rejected_without_gpu(tocr):
    lib = tocr.lib()
    st = lib.tocr_ctc_greedy_f16(None, -1, 80, 100, 100, None, None, None, None, None, None)
    assert st == 1  # TOCR_ERR_INVALID
    assert "bad sizes" in tocr._lib.last_error()
    st = lib.tocr_preprocess_batch_f16(None, None, None, None, None, None, None, 961, 960, 4,
                                       None, None, None)
    assert st == 1
    assert "multiple of 8" in tocr._lib.last_error()
    with pytest.raises(tocr.InvalidArgument):
        tocr.check(lib.tocr_argmax_f32(None, None, None, 1, 1, 0, None), "tocr_argmax_f32")


def test_empty_problems_are_noops(tocr):
    lib = tocr.lib()
    assert lib.tocr_ctc_greedy_f16(None, 0, 80, 100, 100, None, None, None, None, None, None) == 0
    assert lib.tocr_threshold_u8(None, None, 0, 0, 0, 0.3, None) == 0
    assert lib.tocr_preprocess_batch_f16(None, None, None, None, None, None, None, 960, 960, 0,
                                         None, None, None) == 0


def test_fault_injection_surfaces_as_inference_error(tocr):
    lib = tocr.lib()
    lib.tocr_debug_inject_error(5, 2)
    try:
        for _ in range(2):
            st = lib.tocr_threshold_u8(None, None, 4, 4, 1, 0.3, None)
            assert st == 5
            with pytest.raises(tocr.InferenceError):
                tocr.check(st, "tocr_threshold_u8")
        # injection consumed: the next call validates normally (null pointer)
        assert lib.tocr_threshold_u8(None, None, 4, 4, 1, 0.3, None) == 1
    finally:
        lib.tocr_debug_inject_error(0, 0)


def test_geometry_and_page_entries_reject_bad_arguments_without_gpu(tocr):
    """Argument checks of the DB, stem, crop and warp entries run before any
    CUDA call."""
    import ctypes as C
    lib = tocr.lib()
    # DB: a map taller than the geometry's coordinate range, too wide for
    # the box-score masks, a workspace that is too small
    st = lib.tocr_db_postprocess(C.c_void_p(1), 1, 1 << 19, 8, None, 0.3, 0.6, 1.5, 3.0, 5.0,
                                 0, 0, C.c_void_p(256), 1 << 30, C.c_void_p(1), C.c_void_p(1),
                                 C.c_void_p(1), 10, C.c_void_p(1), None)
    assert st == 1 and "too large" in tocr._lib.last_error()
    st = lib.tocr_db_postprocess(C.c_void_p(1), 1, 64, 5000, None, 0.3, 0.6, 1.5, 3.0, 5.0,
                                 0, 0, C.c_void_p(256), 1 << 30, C.c_void_p(1), C.c_void_p(1),
                                 C.c_void_p(1), 10, C.c_void_p(1), None)
    assert st == 1 and "width" in tocr._lib.last_error()
    need = lib.tocr_db_workspace_bytes(2, 96, 128, 0, 0)
    assert need > 0
    st = lib.tocr_db_postprocess(C.c_void_p(1), 2, 96, 128, None, 0.3, 0.6, 1.5, 3.0, 5.0,
                                 0, 0, C.c_void_p(256), need - 1, C.c_void_p(1), C.c_void_p(1),
                                 C.c_void_p(1), 10, C.c_void_p(1), None)
    assert st == 1 and "workspace" in tocr._lib.last_error()
    # a bigger scratch pool needs a bigger workspace; zero maps is a no-op
    assert lib.tocr_db_workspace_bytes(2, 96, 128, 0, 1 << 20) > need
    assert lib.tocr_db_postprocess(None, 0, 96, 128, None, 0.3, 0.6, 1.5, 3.0, 5.0, 0, 0, None,
                                   0, None, None, None, 10, None, None) == 0
    # stem, ink map, ROI warp, crop transforms
    assert lib.tocr_stem_f16(None, -1, 960, 960, 0, None, None, None) == 1
    assert lib.tocr_stem_f16(None, 0, 960, 960, 0, None, None, None) == 0
    assert lib.tocr_stem_take_error(None) == 1
    assert lib.tocr_ink_map(None, 1, 0, 960, 0, 12.0, None, None) == 1
    assert lib.tocr_roi_warp_f16(None, 0, 960, 960, 2880, None, None, None, None, -1, 48, 320,
                                 None, None, 1.0, None, None) == 1
    assert lib.tocr_roi_warp_f16(None, 0, 960, 960, 2880, None, None, None, None, 0, 48, 320,
                                 None, None, 1.0, None, None) == 0
    small = bytearray(8)
    buf = (C.c_char * len(small)).from_buffer(small)
    assert lib.tocr_stem_pack(None, None, None, None, buf, 8) == 1
