"""Builds tests/native/modules_test.cpp, a C++ caller of libtocr_b200.so
compiled with g++ against include/ only (as reference-side code would be)."""
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "native" / "modules_test.cpp"
OUT = ROOT / "tests" / "native" / "_build" / "modules_test"
LIB = ROOT / "turboocr_b200"
CUDA = Path("/usr/local/cuda")


def build() -> Path:
    OUT.parent.mkdir(exist_ok=True)
    headers = list((ROOT / "include").rglob("*.h"))
    newest = max([SRC.stat().st_mtime, (LIB / "libtocr_b200.so").stat().st_mtime] +
                 [h.stat().st_mtime for h in headers])
    if not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = ["g++", "-std=c++20", "-O2", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}",
               str(SRC), "-o", str(OUT), f"-L{LIB}", "-ltocr_b200", f"-Wl,-rpath,{LIB}",
               f"-L{CUDA / 'lib64'}", "-lcudart", f"-Wl,-rpath,{CUDA / 'lib64'}"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(r.stdout + r.stderr)
    return OUT
