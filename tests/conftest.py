"""Shared test setup: import paths, the `gpu` marker, built libraries."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_DIR = REPO / "ampere-gemm_b200"
for p in (str(REPO), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def native_lib():
    """Build (if stale and nvcc is present) and load libb200gemm.so."""
    import build as pkg_build  # ampere-gemm_b200/build.py
    from tensorcore_gemm import _native

    if pkg_build.needs_build():
        try:
            pkg_build.build()
        except RuntimeError:
            if not _native.LIB_PATH.exists():
                raise
    return _native.load()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test scheduled without a visible CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"GPU tests need an sm_100 device, found capability major {major}")
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda:0")
