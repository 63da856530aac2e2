"""Loads the oracle's shared libraries, building them when the reference tree
is available (in the build container); on a GPU box the prebuilt files that
travelled with the snapshot are used."""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _reference_root() -> Path:
    """The reference checkout: $TOCR_REFERENCE, else BASELINE.json's
    reference_path. It exists only where the oracle is built, not on a GPU
    box (which uses the prebuilt files)."""
    env = os.environ.get("TOCR_REFERENCE")
    if env:
        return Path(env)
    try:
        return Path(json.loads((HERE.parent / "BASELINE.json").read_text())["reference_path"])
    except (OSError, KeyError, ValueError):
        return HERE / "_no_reference"


REF = _reference_root()


def build(verbose: bool = False) -> None:
    targets = ["own"] + (["ref"] if REF.exists() else [])
    r = subprocess.run(["make", "-C", str(HERE), f"REF={REF}", *targets],
                       capture_output=True, text=True)
    if verbose or r.returncode != 0:
        print(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed")


_cache: dict[str, C.CDLL] = {}


def load(rel: str) -> C.CDLL:
    if rel in _cache:
        return _cache[rel]
    path = HERE / rel
    if not path.exists():
        build()
    if not path.exists():
        raise FileNotFoundError(f"{path} not built (needs the reference tree for _ref/)")
    lib = C.CDLL(str(path), mode=os.RTLD_LOCAL | os.RTLD_NOW)
    _cache[rel] = lib
    return lib
