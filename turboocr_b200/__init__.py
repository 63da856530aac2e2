"""B200-native TurboOCR det+rec hot path.

Host-side mirror of the reference's kernel and module entry points over the
C-ABI library ``libtocr_b200.so`` (include/tocr_capi.h). Device memory,
streams and process groups come from PyTorch; every byte of the hot path is
computed by this package's CUDA kernels.
"""
from ._lib import (  # noqa: F401
    CudaError,
    InferenceError,
    InvalidArgument,
    OcrError,
    TimeoutError,
    check,
    lib,
    synth,
)
from . import kernels  # noqa: F401
