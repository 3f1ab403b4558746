// Constants, tile scheduler and abort-path helpers shared by the GEMM kernels.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "sm100_ptx.cuh"
#include "umma_desc.h"

namespace b200 {

constexpr int kBM = 128;         // rows of A / C per tile (one TMEM lane per row)
constexpr int kBK = 64;          // K per stage: one 128-byte swizzle row of fp16
constexpr int kUmmaK = 16;       // K per tcgen05.mma kind::f16
constexpr int kThreads = 192;    // 6 warps
constexpr int kEpiWarps = 4;
constexpr int kEpiCols = 64;     // columns per epilogue store box (128 bytes)
constexpr int kEpiRows = 32;     // rows per epilogue warp
constexpr int kEpiBufBytes = kEpiRows * kEpiCols * 2;   // 4 KB

template <int BN, int STAGES>
struct TileConfig {
  static constexpr int kABytes = kBM * kBK * 2;               // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;                // BN * 128
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBytes = kEpiWarps * 2 * kEpiBufBytes;
  static constexpr int kTmemCols = 2 * BN;                    // two accumulators
  static constexpr int kBarBytes = 256;
  // +1024 so the base can be rounded up to the 1024-byte swizzle atom.
  static constexpr int kSmemBytes = STAGES * kStageBytes + kEpiBytes + kBarBytes + 1024;
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 64 in [64, 256]");
  static_assert(kTmemCols <= 512, "two accumulators must fit the 512 TMEM columns");
  static_assert(kSmemBytes <= 232448, "shared memory per CTA exceeds 227 KB");
};

// Persistent tile order: bands of `group_m` row-blocks; inside a band the row
// block changes fastest, so CTAs that run together share B panels and a small
// set of A panels in L2.
struct TileScheduler {
  int num_m, num_n, group_m;
  __device__ __forceinline__ void tile_coords(int t, int& mb, int& nb) const {
    const int per_band = group_m * num_n;
    const int band = t / per_band;
    const int first_m = band * group_m;
    const int gsize = min(group_m, num_m - first_m);
    const int r = t - band * per_band;
    mb = first_m + r % gsize;
    nb = r / gsize;
  }
};

// Bounded wait used only on the abort path: ignores the error word (which is
// already set) and gives up after 100 ms.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > 100000000ull) {
      raise_device_error(kDevTimeoutDrain);
      return false;
    }
  }
  return true;
}

}  // namespace b200
