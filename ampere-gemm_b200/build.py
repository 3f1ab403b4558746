"""Ahead-of-time build of the native GEMM library for sm_100a.

Produces ``tensorcore_gemm/_lib/libb200gemm.so`` next to the Python package,
in-tree, so a snapshot of the repository carries the built library with it.
The reference JIT-compiled its kernels on first call with load_inline and an
arch taken from whatever GPU was present (tensorcore_gemm/cuda_compile.py:47-62,
157-269); this library is compiled once, explicitly for sm_100a, and needs no
GPU to build.

Usage:  python ampere-gemm_b200/build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
LIB_DIR = PKG_ROOT / "tensorcore_gemm" / "_lib"
LIB_PATH = LIB_DIR / "libb200gemm.so"
HEADERS = [REPO_ROOT / "include" / "b200_gemm.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xptxas", "-v",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xcompiler", "-fvisibility=hidden",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the B200 GEMM library cannot be built")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + HEADERS


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/b200_gemm.cu into the in-tree shared library."""
    if not force and not needs_build():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "b200_gemm.cu")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    (LIB_DIR / "build.log").write_text(" ".join(cmd) + "\n" + log)
    if proc.returncode != 0:
        sys.stderr.write(log)
        raise RuntimeError(f"nvcc failed building {LIB_PATH.name} (exit {proc.returncode})")
    if verbose:
        sys.stdout.write(log)
    tmp.replace(LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
