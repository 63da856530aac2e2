"""Build the in-tree shared libraries of the B200 path.

``libtocr_b200.so``  — every CUDA kernel, the C-ABI (include/tocr_capi.h)
                       and the C++ shims that re-expose the reference
                       signatures (include/turbo_ocr/...).
``libtocr_synth.so`` — the seeded synthetic-input generators used by the
                       tests and bench.py (not part of the product path).

Everything is compiled for sm_100a only. Objects go to turboocr_b200/_build/,
libraries next to this file, so a snapshot of the repository carries them.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++20", "-Xcompiler", "-fPIC", "-Xcompiler",
          "-fvisibility=hidden", f"-I{INCLUDE}", f"-I{CSRC}"]

LIBS = {
    "libtocr_b200.so": ["capi_common.cu", "ctc.cu", "preprocess.cu", "threshold.cu", "dwpw.cu",
                        "db.cu", "pagekernels.cu", "crop.cu", "jfa.cu", "cls.cu", "rec_head.cu", "dbhead.cu",
                        "png.cu"],
    "libtocr_synth.so": ["synth.cu"],
}
# C++ host sources (reference-signature shims), built into libtocr_b200.so.
HOST_SOURCES = {
    "libtocr_b200.so": ["shim_kernels.cpp", "shim_ctc.cpp", "det_config_capi.cpp", "modules.cpp"],
}
HEADERS = sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.rglob("*.h")))


def _newest_header() -> float:
    return max((h.stat().st_mtime for h in HEADERS), default=0.0)


# Per-file extra flags. db.cu and crop.cu must not contract multiply-adds:
# they reproduce the floating-point operation order of OpenCV, Clipper and
# the reference's host geometry (explicit fma() where those contract).
EXTRA = {"db.cu": ["-fmad=false"], "crop.cu": ["-fmad=false"],
         "modules.cpp": ["-Xcompiler", "-ffp-contract=off"]}


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    flags = list(COMMON) + EXTRA.get(src.name, [])
    if src.suffix == ".cu":
        flags += ARCH
    else:
        flags += ["-x", "c++"]
    cmd = [NVCC, *flags, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")


def build(verbose: bool = False, force: bool = False) -> list[Path]:
    """Compile (incrementally) and link every library; return their paths."""
    BUILD.mkdir(exist_ok=True)
    hdr_time = _newest_header()
    out = []
    jobs = []
    for lib, cu in LIBS.items():
        for name in cu + HOST_SOURCES.get(lib, []):
            src = CSRC / name
            obj = BUILD / (name + ".o")
            if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
                jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(lambda j: _compile(j[0], j[1], verbose), jobs))
    for lib, cu in LIBS.items():
        objs = [BUILD / (n + ".o") for n in cu + HOST_SOURCES.get(lib, [])]
        target = PKG / lib
        if force or not target.exists() or target.stat().st_mtime < max(o.stat().st_mtime for o in objs):
            cmd = [NVCC, *ARCH, "-shared", "-o", str(target), *map(str, objs)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"link failed for {lib}:\n{r.stdout}\n{r.stderr}")
        out.append(target)
    return out


def ptxas_report(name: str) -> str:
    """`-Xptxas -v` register/shared-memory report of one .cu file."""
    cmd = [NVCC, *COMMON, *ARCH, "-Xptxas", "-v", "-c", str(CSRC / name), "-o", os.devnull]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.stdout + r.stderr


if __name__ == "__main__":
    force = "--force" in sys.argv
    if "--ptxas" in sys.argv:
        print(ptxas_report(sys.argv[sys.argv.index("--ptxas") + 1]))
    else:
        for p in build(verbose=True, force=force):
            print("built", p)
