"""The reference's own Catch2 unit tests for the path, compiled in place from
the reference tree against THIS repository's headers (include/) and linked
to libtocr_b200.so, as a reference maintainer would build them after the
swap: tests/common/test_box.cpp, tests/common/test_perspective.cpp,
tests/recognition/test_ctc_decode.cpp and tests/recognition/test_rec_geometry.cpp
with third_party/catch2. No reference header is on the include path, so
every declaration they use comes from include/turbo_ocr/. Host-only (no
GPU); skipped where the reference tree is absent (the GPU box)."""
import subprocess
from pathlib import Path

import pytest

from oracle._loader import REF

ROOT = Path(__file__).resolve().parents[1]
OUT = ROOT / "tests" / "native" / "_build" / "reference_unit_tests"
LIB = ROOT / "turboocr_b200"
CUDA = Path("/usr/local/cuda")
SUITES = ["tests/common/test_box.cpp", "tests/common/test_perspective.cpp",
          "tests/recognition/test_ctc_decode.cpp", "tests/recognition/test_rec_geometry.cpp"]


def build():
    catch = REF / "third_party" / "catch2"
    srcs = [REF / s for s in SUITES] + [catch / "catch_amalgamated.cpp"]
    headers = list((ROOT / "include").rglob("*.h"))
    newest = max([p.stat().st_mtime for p in srcs + headers] +
                 [(LIB / "libtocr_b200.so").stat().st_mtime])
    if OUT.exists() and OUT.stat().st_mtime >= newest:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    objs = []
    for s in srcs:
        o = OUT.parent / (s.stem + ".ref.o")
        if not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime,
                                                      max(h.stat().st_mtime for h in headers)):
            r = subprocess.run(["g++", "-std=c++20", "-O1", "-c", str(s), f"-I{catch}",
                                f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}", "-o", str(o)],
                               capture_output=True, text=True)
            assert r.returncode == 0, r.stderr[-4000:]
        objs.append(str(o))
    r = subprocess.run(["g++", "-o", str(OUT), *objs, f"-L{LIB}", "-ltocr_b200",
                        f"-Wl,-rpath,{LIB}", f"-L{CUDA / 'lib64'}", "-lcudart",
                        f"-Wl,-rpath,{CUDA / 'lib64'}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return OUT


@pytest.mark.skipif(not (REF / "third_party" / "catch2").exists(),
                    reason="reference tree absent (only the build container has it)")
def test_reference_unit_tests_pass_against_this_library():
    exe = build()
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "All tests passed" in r.stdout
    n = int(r.stdout.split("in ")[-1].split(" test cases")[0])
    assert n >= 28
