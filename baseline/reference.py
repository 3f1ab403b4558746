"""Loads the unmodified reference package from baseline/_ref.

The package is imported under its own module name prefix
(`_reference_tensorcore_gemm`) so it never shadows this repository's
`tensorcore_gemm`.  Only the benchmark's reference arm and comparators and
the GPU cross-check tests use it; the product path never does.
"""
from __future__ import annotations

import importlib
import importlib.util
import sys
from pathlib import Path

REF_DIR = Path(__file__).resolve().parent / "_ref"
MODULE_NAME = "_reference_tensorcore_gemm"


def load_package():
    """The reference's `tensorcore_gemm` package, or None if it is not installed."""
    if MODULE_NAME in sys.modules:
        return sys.modules[MODULE_NAME]
    init = REF_DIR / "tensorcore_gemm" / "__init__.py"
    if not init.exists():
        return None
    spec = importlib.util.spec_from_file_location(MODULE_NAME, init, submodule_search_locations=[str(init.parent)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def cublas_module():
    """The reference's cuBLAS comparator module (tensorcore_gemm/cublas_gemm.py), or None."""
    pkg = load_package()
    if pkg is None or not (REF_DIR / "tensorcore_gemm" / "cublas_gemm.cu").exists():
        return None
    return importlib.import_module(MODULE_NAME + ".cublas_gemm")
