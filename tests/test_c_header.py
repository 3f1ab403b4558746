"""CPU: the public header is plain C and the library links from a C program.

A C99 translation unit includes include/b200_gemm.h with every warning an
error, links against libb200gemm.so, and calls the host-only entry points
(version, launch plan, argument validation) -- no GPU needed.
"""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
LIB_DIR = REPO / "ampere-gemm_b200" / "tensorcore_gemm" / "_lib"

C_SOURCE = r"""
#include <stdio.h>
#include <string.h>
#include "b200_gemm.h"

int main(void) {
  int variant = -1, ranges = -1;
  if (b200_gemm_version() < 100) return 1;
  if (b200_gemm_plan(65536, 8192, 8192, 148, &variant, &ranges) != B200_OK) return 2;
  if (variant != B200_VARIANT_PAIR_WIDE || ranges != 1) return 3;
  if (b200_gemm_plan(4096, 4096, 16384, 148, &variant, &ranges) != B200_OK) return 4;
  if (variant != B200_VARIANT_PAIR || ranges != 2) return 5;
  /* argument checks run before any CUDA call */
  if (b200_gemm_f16(NULL, NULL, NULL, -1, 8, 8, 8, 8, 8, B200_B_ROW_MAJOR, NULL) != B200_ERR_INVALID_ARGUMENT) return 6;
  if (b200_kmeans_workspace_size(1024, 256) <= 0) return 7;
  if (strlen(b200_gemm_strerror(B200_ERR_MISALIGNED)) == 0) return 8;
  printf("ok %d\n", b200_gemm_version());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_is_c99_and_links(native_lib, tmp_path):
    src = tmp_path / "abi.c"
    src.write_text(C_SOURCE)
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{REPO / 'include'}",
                    str(src), "-o", str(exe), f"-L{LIB_DIR}", "-lb200gemm", f"-Wl,-rpath,{LIB_DIR}"],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert out.stdout.startswith("ok ")
