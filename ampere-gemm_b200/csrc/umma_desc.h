// Bit packing of the two 64/32-bit words a tcgen05.mma instruction reads:
// the shared-memory matrix descriptor and the instruction descriptor for
// kind::f16.  Plain C++ (host and device) so host-side unit tests can check
// every field against values computed by hand from the PTX ISA tables.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define B200_HD constexpr __host__ __device__ __forceinline__
#else
#define B200_HD constexpr inline
#endif

namespace b200 {

// Shared-memory swizzle codes of the sm_100 matrix descriptor (bits 61..63).
enum class SmemSwizzle : uint32_t { kNone = 0, kSw128Base32 = 1, kSw128 = 2, kSw64 = 4, kSw32 = 6 };

// Shared-memory matrix descriptor:
//   bits  0..13  start address >> 4
//   bits 16..29  leading-dimension byte offset >> 4
//   bits 32..45  stride-dimension byte offset >> 4
//   bits 46..47  descriptor version (1 on sm_100)
//   bits 49..51  base offset (0: every swizzle atom starts 1024-byte aligned)
//   bit  52      LBO mode (0: relative byte offset)
//   bits 61..63  swizzle mode
B200_HD uint64_t make_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes, SmemSwizzle sw) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(static_cast<uint32_t>(sw) & 0x7u) << 61;
  return d;
}

// Operand major-ness as the MMA sees it: K-major means the reduction index is
// the contiguous one (A row-major, or B stored N x K); MN-major means the
// M (for A) or N (for B) index is contiguous (B stored row-major K x N).
enum class Major : uint32_t { kK = 0, kMN = 1 };

// Instruction descriptor for tcgen05.mma kind::f16 with fp16 A/B and fp32 D:
//   bits  4..5   D format (1 = f32)
//   bits  7..9   A format (0 = f16)
//   bits 10..12  B format (0 = f16)
//   bit  15      A major (0 = K, 1 = MN)
//   bit  16      B major
//   bits 17..22  N >> 3
//   bits 24..28  M >> 4
B200_HD uint32_t make_idesc_f16_f32(uint32_t m, uint32_t n, Major a_major, Major b_major) {
  uint32_t d = 0;
  d |= 1u << 4;
  d |= (static_cast<uint32_t>(a_major) & 1u) << 15;
  d |= (static_cast<uint32_t>(b_major) & 1u) << 16;
  d |= ((n >> 3) & 0x3Fu) << 17;
  d |= ((m >> 4) & 0x1Fu) << 24;
  return d;
}

// Canonical 128-byte-swizzled layouts written by TMA with a 128-byte inner box
// (64 fp16) and consumed by the MMA:
//
// K-major tile (rows = M or N, 64 K-elements per row): row r lives at byte
//   r * 128, the 16-byte chunk c of that row at chunk c ^ (r & 7).  Groups of
//   8 rows (1024 B) follow one another, so SBO = 1024; LBO is unused.  Moving
//   16 K-elements to the right is +32 bytes on the start address.
constexpr uint32_t kSw128RowBytes = 128;
constexpr uint32_t kSw128AtomBytes = 1024;

B200_HD uint64_t make_desc_kmajor_sw128(uint32_t smem_addr) {
  return make_smem_desc(smem_addr, 16, kSw128AtomBytes, SmemSwizzle::kSw128);
}

// MN-major tile (B row-major, K rows of N): the tile is split into panels of
// 64 N-elements; a panel holds `k_rows` rows of 128 bytes (swizzled like
// above) and panels follow one another every `panel_bytes`.  Then
//   LBO = panel_bytes  (step between 64-element groups along N)
//   SBO = 1024         (step between groups of 8 K-rows)
// and moving 16 K-rows down is +2048 bytes on the start address.
B200_HD uint64_t make_desc_mnmajor_sw128(uint32_t smem_addr, uint32_t panel_bytes) {
  return make_smem_desc(smem_addr, panel_bytes, kSw128AtomBytes, SmemSwizzle::kSw128);
}

}  // namespace b200
