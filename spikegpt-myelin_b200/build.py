"""Build recipe for libspikegpt_wkv.so (sm_100a), in-tree.

    python spikegpt-myelin_b200/build.py          # builds lib/libspikegpt_wkv.so

nvcc cross-compiles for sm_100a without a GPU. The shared library is placed in
``spikegpt-myelin_b200/lib/`` so that it travels with the source tree; the
Python package loads it from there.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
LIB_DIR = PKG_ROOT / "lib"
LIB = LIB_DIR / "libspikegpt_wkv.so"
SOURCES = [CSRC / "wkv_capi.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + [REPO_ROOT / "include" / "spikegpt_wkv.h"]

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def build(force: bool = False, verbose: bool = False) -> Path:
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    if not force and LIB.exists():
        newest = max(p.stat().st_mtime for p in DEPS)
        if LIB.stat().st_mtime >= newest:
            return LIB
    tmp = LIB.with_name(LIB.name + f".tmp{os.getpid()}")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(REPO_ROOT / "include"), "-I", str(CSRC)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [*map(str, SOURCES), "-o", str(tmp)]
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
