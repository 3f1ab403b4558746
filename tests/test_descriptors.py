"""CPU: bit packing of the tcgen05 shared-memory and instruction descriptors,
checked against values worked out by hand from the PTX ISA field tables."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
CSRC = REPO / "ampere-gemm_b200" / "csrc"

PROGRAM = r"""
#include <cstdio>
#include "umma_desc.h"
using namespace b200;
int main() {
  std::printf("%llx\n", (unsigned long long)make_desc_kmajor_sw128(0x400));
  std::printf("%llx\n", (unsigned long long)make_desc_kmajor_sw128(0x1a420));
  std::printf("%llx\n", (unsigned long long)make_desc_mnmajor_sw128(0x2000, 8192));
  std::printf("%x\n", make_idesc_f16_f32(128, 256, Major::kK, Major::kK));
  std::printf("%x\n", make_idesc_f16_f32(128, 256, Major::kK, Major::kMN));
  std::printf("%x\n", make_idesc_f16_f32(256, 256, Major::kK, Major::kMN));
  std::printf("%x\n", make_idesc_f16_f32(128, 64, Major::kMN, Major::kK));
  std::printf("%llx\n", (unsigned long long)make_smem_desc(0x3fff0, 0x3fff0, 0x3fff0, SmemSwizzle::kNone));
  return 0;
}
"""


def _hand_smem(addr, lbo, sbo, swz):
    return ((addr >> 4) & 0x3FFF) | (((lbo >> 4) & 0x3FFF) << 16) | (((sbo >> 4) & 0x3FFF) << 32) | (1 << 46) | (swz << 61)


def _hand_idesc(m, n, a_mn, b_mn):
    # D=f32 at bit 4, A/B f16 (0), a_major bit 15, b_major bit 16, N>>3 at 17, M>>4 at 24.
    return (1 << 4) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) | ((m >> 4) << 24)


@pytest.fixture(scope="module")
def values(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.fail("no host C++ compiler for the descriptor test")
    d = tmp_path_factory.mktemp("desc")
    (d / "t.cpp").write_text(PROGRAM)
    subprocess.run([cxx, "-std=c++17", "-O1", f"-I{CSRC}", "-o", str(d / "t"), str(d / "t.cpp")], check=True)
    out = subprocess.run([str(d / "t")], check=True, capture_output=True, text=True).stdout.split()
    return [int(x, 16) for x in out]


def test_kmajor_sw128(values):
    assert values[0] == _hand_smem(0x400, 16, 1024, 2)
    assert values[0] == 0x4000_4040_0001_0040
    assert values[1] == _hand_smem(0x1A420, 16, 1024, 2)


def test_mnmajor_sw128(values):
    assert values[2] == _hand_smem(0x2000, 8192, 1024, 2)


def test_instruction_descriptors(values):
    assert values[3] == _hand_idesc(128, 256, 0, 0) == 0x08400010
    assert values[4] == _hand_idesc(128, 256, 0, 1) == 0x08410010
    assert values[5] == _hand_idesc(256, 256, 0, 1)
    assert values[6] == _hand_idesc(128, 64, 1, 0)


def test_field_masking(values):
    assert values[7] == _hand_smem(0x3FFF0, 0x3FFF0, 0x3FFF0, 0)
