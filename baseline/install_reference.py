"""Install the unmodified reference package into baseline/_ref (offline).

    python baseline/install_reference.py [--force]

Runs `pip install --no-index --no-build-isolation --no-deps --find-links
/opt/wheelhouse --target baseline/_ref` on a copy of the reference source tree
(pip's build writes into the tree it builds from, and the original is
read-only).  `--no-deps` because the reference's only hard dependency besides
setuptools, `modal`, is its cloud runner and is not in the wheelhouse.

The reference's pyproject declares no package data, so the wheel carries only
its .py modules; its `gemm.py` and `cublas_gemm.py` read their CUDA sources
(`gemm.cu`, `cublas_gemm.cu`, ...) from beside themselves
(tensorcore_gemm/cublas_gemm.py:9-10).  Those source files are copied, as
they are, next to the installed modules so the installed package can run
its own GPU comparator through its own JIT path (cuda_compile.compile_cuda).
Nothing here is committed: baseline/_ref is git-ignored.
"""
from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"
REFERENCE = Path("/root/reference")
WHEELHOUSE = Path("/opt/wheelhouse")


def installed() -> bool:
    pkg = TARGET / "tensorcore_gemm"
    return (pkg / "__init__.py").exists() and (pkg / "cublas_gemm.cu").exists()


def install(force: bool = False) -> bool:
    """Returns True when baseline/_ref holds the reference package afterwards."""
    if installed() and not force:
        return True
    if not (REFERENCE / "pyproject.toml").exists():
        return installed()
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "reference"
        shutil.copytree(REFERENCE, src, ignore=shutil.ignore_patterns(".git", "results", "plots"))
        if TARGET.exists():
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", str(WHEELHOUSE), "--target", str(TARGET), str(src)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            return False
        pkg_src = src / "src" / "tensorcore_gemm"
        for f in sorted(pkg_src.iterdir()):
            if f.suffix in (".cu", ".cuh"):
                shutil.copy2(f, TARGET / "tensorcore_gemm" / f.name)
    return installed()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ok = install(force=ap.parse_args().force)
    print("baseline/_ref:", "installed" if ok else "NOT installed")
    sys.exit(0 if ok else 1)
