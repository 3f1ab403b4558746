// Constants, tile scheduler and abort-path helpers shared by the GEMM kernels.
#pragma once

#include <cuda.h>
#include <cstdint>
#include <cstring>

#include "sm100_ptx.cuh"
#include "umma_desc.h"

namespace b200 {

// Optional wait-time instrumentation (compile with -DB200_GEMM_PROFILE): per
// CTA, cycles each role spends blocked on each barrier.  Off in the product.
#ifdef B200_GEMM_PROFILE
__device__ unsigned long long g_prof[1024][8];
// Per-thread accumulators live in registers; flushed once at kernel end.
#define B200_PROF_DECL unsigned long long prof_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#define B200_TIMED(slot, expr)                   \
  ({                                             \
    const long long _t0 = clock64();             \
    const bool _r = (expr);                      \
    prof_acc[slot] += (unsigned long long)(clock64() - _t0); \
    _r;                                          \
  })
#define B200_PROF_ADD(slot, v) (prof_acc[slot] += (unsigned long long)(v))
// Split-tail step timestamps (ns since the unit's start), one row per CTA.
__device__ unsigned long long g_split_prof[1024][8];
#define B200_SPLIT_MARK(i, t0) \
  if (threadIdx.x == 64) g_split_prof[blockIdx.x & 1023][i] = global_timer_ns() - (t0)
#define B200_PROF_FLUSH                                                         \
  if (threadIdx.x == 0 || threadIdx.x == 32 || threadIdx.x == 64) {             \
    for (int _i = 0; _i < 8; ++_i)                                              \
      if (prof_acc[_i]) atomicAdd(&g_prof[blockIdx.x & 1023][_i], prof_acc[_i]); \
  }
#else
#define B200_PROF_DECL
#define B200_TIMED(slot, expr) (expr)
#define B200_PROF_ADD(slot, v) ((void)0)
#define B200_SPLIT_MARK(i, t0) ((void)0)
#define B200_PROF_FLUSH
#endif

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

// Persistent tile order.  group_m > 0: bands of group_m row blocks, row block
// fastest inside a band (a band of A stays hot while B streams).  group_m < 0:
// bands of -group_m column blocks, column block fastest (a band of B stays hot
// and each A panel is finished by consecutive tiles, then dropped) -- the
// better order when A is much larger than B.
struct TileScheduler {
  int num_m, num_n, group_m;
  __device__ __forceinline__ void tile_coords(int t, int& mb, int& nb) const {
    if (group_m > 0) {
      const int per_band = group_m * num_n;
      const int band = t / per_band;
      const int first_m = band * group_m;
      const int gsize = min(group_m, num_m - first_m);
      const int r = t - band * per_band;
      mb = first_m + r % gsize;
      nb = r / gsize;
    } else {
      const int gn = -group_m;
      const int per_band = gn * num_m;
      const int band = t / per_band;
      const int first_n = band * gn;
      const int gsize = min(gn, num_n - first_n);
      const int r = t - band * per_band;
      nb = first_n + r % gsize;
      mb = r / gsize;
    }
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

namespace b200 {

constexpr int kMaxPeers = 7;

// Epilogue parameters.
//  * alpha / beta, the reference kernels' scaling (tensorcore_gemm/gemm.cu
//    :1360-1364): C = fp16_rn(alpha * acc) when beta == 0, otherwise
//    C = fp16_rn(alpha * acc + beta * C_old), in fp32 with one rounding.
//  * m, n, ldc: C's extent and pitch (elements).
//  * n_tma: C's columns [0, n_tma) go through the TMA tensor map (encoded
//    n_tma wide).  A TMA store writes whole 16-byte pieces, so when n is not a
//    multiple of 8 the map stops at n rounded down to 8 and the last partial
//    piece of each row, columns [n_tma, n), is written by plain stores
//    through `c` (and, with beta != 0, its old values read by plain loads).
//  * peers (gathered-output mode): every finished C block is also written,
//    with plain 16-byte stores, to `n_peers` other buffers of the same pitch
//    -- the other GPUs' copies of the gathered C, mapped into this process
//    by CUDA IPC, each pointer at this shard's first row.  Never a TMA or
//    bulk access to peer memory.
struct EpiParams {
  float alpha = 1.0f;
  float beta = 0.0f;
  int m = 0;
  int n = 0;
  int n_tma = 0;
  int n_peers = 0;
  int64_t ldc = 0;
  uint16_t* c = nullptr;
  uint16_t* peer[kMaxPeers] = {};
  // 1 when C is larger than L2: its TMA stores are marked evict-first, so the
  // written lines make way for the operands that are still being re-read
  // (65536 x 8192 x 8192: 0.45 GB fewer DRAM reads per launch, 1-2 % faster).
  // A C that fits L2 keeps the default policy for the kernel that consumes it.
  int c_evict_first = 0;
};

// Copies the 16-byte pieces of the 32 x 64 fp16 block staged at `buf`
// (128B-swizzled, row r at r * 128) whose columns lie in [c_lo, c_hi) to
// element (x, y) of each of the `ndst` row-pitch-ldc buffers in `dst`.  Lane l
// moves piece l % 8 of rows l / 8, l / 8 + 4, ...: one store instruction
// writes four whole 128-byte row pieces.  A piece crossing c_hi is written
// element by element.
__device__ __forceinline__ void epi_plain_store(const uint8_t* buf, int lane, int x, int y, const EpiParams& ep,
                                                int c_lo, int c_hi, uint16_t* const* dst, int ndst) {
  const int seg = lane & 7;
  const int col = x + seg * 8;
  if (col >= c_hi || col + 8 <= c_lo) return;
  const bool whole = col + 8 <= c_hi;
#pragma unroll 1
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + (lane >> 3);
    if (y + r >= ep.m) break;
    const uint4 v = *reinterpret_cast<const uint4*>(buf + r * 128 + ((seg ^ (r & 7)) << 4));
    const int64_t off = static_cast<int64_t>(y + r) * ep.ldc + col;
#pragma unroll 1
    for (int p = 0; p < ndst; ++p) {
      uint16_t* d = dst[p] + off;
      if (whole) {
        *reinterpret_cast<uint4*>(d) = v;
      } else {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 7; ++e)
          if (e < c_hi - col) d[e] = static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16));
      }
    }
  }
}

// Second half of an epilogue block store: the staged 32 x 64 fp16 block at
// `buf` leaves through the TMA map (columns before n_tma, whole blocks of this
// tile), by plain stores (columns past the map or past x_end), and to the
// peers' copies in gathered-output mode; the staging ring then advances.
template <int NBUF>
__device__ __forceinline__ void epi_issue_store(const CUtensorMap* tmap_c, uint8_t* buf, int& sbuf, int lane, int x,
                                                int y, const EpiParams& sc, int x_end) {
  const bool in_tile = x + kEpiCols <= x_end;
  const bool tma_part = x < sc.n_tma && in_tile;
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && tma_part) {
    if (sc.c_evict_first)
      tma_store_2d_hint(tmap_c, buf, x, y, policy_evict_first());
    else
      tma_store_2d(tmap_c, buf, x, y);
    bulk_commit_group();
  }
  const int c_hi = x_end < sc.n ? x_end : sc.n;
  if (!in_tile)
    epi_plain_store(buf, lane, x, y, sc, x, c_hi, &sc.c, 1);
  else if (sc.n_tma < sc.n && x + kEpiCols > sc.n_tma)
    epi_plain_store(buf, lane, x, y, sc, sc.n_tma, sc.n, &sc.c, 1);
  if (sc.n_peers > 0) epi_plain_store(buf, lane, x, y, sc, 0, c_hi, sc.peer, sc.n_peers);
  // The ring advances with the bulk groups: a block past the map committed
  // none, so its buffer (only read synchronously) is reused by the next block;
  // otherwise the wait above would count one group short.
  if (tma_part) sbuf = (sbuf + 1) % NBUF;
}

// Writes one 32-row x 64-column block of C from the calling warp: lane l holds
// row l's 64 fp32 values in lo (columns 0..31) and hi (32..63).  The block goes
// through the warp's 128B-swizzled staging buffer (`NBUF` buffers, `sbuf`
// rotates) and leaves with a TMA store at element (x, y) of C (plus plain
// stores for a partial last piece and for the peers, see EpiParams).  With
// beta != 0 the old C block is first brought into the same buffer by a TMA
// load that completes on `cbar` (phase bit in `cphase`); the wait is bounded
// like every other wait of the kernels.  `x_end` bounds the columns this
// block may write: a tile whose width is not a multiple of 64 ends in a block
// of which only the columns before x_end are its own; that block leaves by
// plain stores (the next tile owns the rest of the 64).
template <int NBUF>
__device__ __forceinline__ void epi_store_block(const CUtensorMap* tmap_c, uint8_t* epi_buf, uint32_t epi_addr,
                                                int& sbuf, int lane, const uint32_t (&lo)[32],
                                                const uint32_t (&hi)[32], int x, int y, const EpiParams& sc,
                                                uint64_t* cbar, uint32_t& cphase, int x_end = 0x7fffffff) {
  if (lane == 0) bulk_wait_group_read<NBUF - 1>();
  __syncwarp();
  uint8_t* buf = epi_buf + sbuf * kEpiBufBytes;
  const uint32_t row_addr = epi_addr + sbuf * kEpiBufBytes + lane * 128;
  const bool load_part = x < sc.n_tma;          // old C can come in through the map (beta != 0)
  if (sc.alpha == 1.0f && sc.beta == 0.0f) {
    // Plain product (every call of the reference's launcher): pack the
    // accumulator bits directly; the skinny shapes are bound by this loop.
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t* v = (j < 4) ? (lo + 8 * j) : (hi + 8 * (j - 4));
      st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), pack_half2_rn(v[0], v[1]), pack_half2_rn(v[2], v[3]),
                   pack_half2_rn(v[4], v[5]), pack_half2_rn(v[6], v[7]));
    }
  } else {
    bool have_old = false;
    if (sc.beta != 0.0f) {
      bool ok = true;
      if (lane == 0 && load_part) {
        mbar_arrive_expect_tx(cbar, kEpiBufBytes);
        tma_load_2d(buf, tmap_c, cbar, x, y, policy_evict_first());
        ok = mbar_wait(cbar, cphase, kDevTimeoutEpilogue);
      }
      if (load_part) cphase ^= 1u;
      have_old = __shfl_sync(0xffffffffu, ok, 0);
    }
    const int row = y + lane;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t* v = (j < 4) ? (lo + 8 * j) : (hi + 8 * (j - 4));
      const uint32_t addr = row_addr + ((j ^ (lane & 7)) << 4);
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = sc.alpha * __uint_as_float(v[e]);
      if (have_old) {
        const int col = x + 8 * j;
        uint32_t o[4];
        if (col + 8 <= sc.n_tma) {
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
                       : "r"(addr));
        } else {
          // Past the map: the old values of the partial piece come from C itself.
#pragma unroll
          for (int e = 0; e < 4; ++e) o[e] = 0;
          if (row < sc.m) {
            const uint16_t* src = sc.c + static_cast<int64_t>(row) * sc.ldc + col;
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (col + e < sc.n) o[e >> 1] |= static_cast<uint32_t>(src[e]) << ((e & 1) * 16);
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 old = __half22float2(*reinterpret_cast<const __half2*>(&o[e]));
          f[2 * e] = fmaf(sc.beta, old.x, f[2 * e]);
          f[2 * e + 1] = fmaf(sc.beta, old.y, f[2 * e + 1]);
        }
      }
      st_shared_v4(addr, pack_half2_rn(__float_as_uint(f[0]), __float_as_uint(f[1])),
                   pack_half2_rn(__float_as_uint(f[2]), __float_as_uint(f[3])),
                   pack_half2_rn(__float_as_uint(f[4]), __float_as_uint(f[5])),
                   pack_half2_rn(__float_as_uint(f[6]), __float_as_uint(f[7])));
    }
  }
  epi_issue_store<NBUF>(tmap_c, buf, sbuf, lane, x, y, sc, x_end);
}

// epi_store_block for the plain product (alpha = 1, beta = 0) whose fp16
// pairs are packed already: pk[w] holds columns 2w and 2w + 1 of the lane's
// row, so the accumulator could be released before any store.
template <int NBUF>
__device__ __forceinline__ void epi_store_block_packed(const CUtensorMap* tmap_c, uint8_t* epi_buf, uint32_t epi_addr,
                                                       int& sbuf, int lane, const uint32_t (&pk)[32], int x, int y,
                                                       const EpiParams& sc, int x_end = 0x7fffffff) {
  if (lane == 0) bulk_wait_group_read<NBUF - 1>();
  __syncwarp();
  uint8_t* buf = epi_buf + sbuf * kEpiBufBytes;
  const uint32_t row_addr = epi_addr + sbuf * kEpiBufBytes + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
  epi_issue_store<NBUF>(tmap_c, buf, sbuf, lane, x, y, sc, x_end);
}

// End of an epilogue warp in gathered-output mode: its peer stores are
// performed system-wide before the kernel can complete.
__device__ __forceinline__ void epi_peer_fence(const EpiParams& ep) {
  if (ep.n_peers > 0) __threadfence_system();
}

}  // namespace b200

namespace b200 {

// K-means assignment fused into the epilogue: for every row i of A (a point)
// the kernel keeps min_j (cnorm[j] - 2 * acc[i][j]) over its N slice and
// merges slices with a 64-bit atomicMin on `keys[i]` (score in the high 32
// bits as an order-preserving integer, column index in the low 32 bits, so
// equal scores resolve to the smaller index whatever the order of arrival).
// keys must hold ~0ull on entry.
struct ArgminOut {
  const float* cnorm = nullptr;          // ||c_j||^2, N entries
  unsigned long long* keys = nullptr;    // M entries
};

// min of three floats in one instruction (sm_100); like fminf, a NaN operand
// yields the other operands' minimum.
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Two fmaf's in one packed instruction (fma.rn.f32x2, sm_100): d = a * b + c
// per lane, each rounded exactly as fmaf rounds it.
__device__ __forceinline__ void fma2f(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
      "fma.rn.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__host__ __device__ __forceinline__ uint32_t float_to_ordered(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__host__ __device__ __forceinline__ float ordered_to_float(uint32_t u) {
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// ---------------------------------------------------------------------------
// Split of the last, partial wave along K (2-CTA pair kernel, 256 x 256
// tiles).  A persistent kernel runs whole tiles in waves of `slots` pairs; when
// the last wave holds only R < slots tiles, those R tiles are cut into S
// K-ranges each (R * S <= slots units, one per pair), so the last wave takes
// about 1/S of a tile instead of a whole one.  Each unit writes its fp32 part
// (per CTA: 128 x 256) to a private workspace and bumps the tile's counter;
// the unit that arrives last sums the S parts in the fixed order 0..S-1 (its
// own from TMEM) and stores C through the normal epilogue.  No unit waits for
// another, and the result does not depend on the order of arrival.
// ---------------------------------------------------------------------------
struct SplitTail {
  int dp_tiles = 0x7fffffff;       // tiles [0, dp_tiles) run whole, in full waves
  int S = 1;                       // K ranges per tail tile (1: no split)
  float* ws = nullptr;             // parts: [tail tile][S][CTA of the pair], kPartFloats each
  uint32_t* counters = nullptr;    // [tail tile][CTA of the pair]: arrivals so far (0 between launches)
  // Self-test of the fixup's bounded wait: when non-zero, the last unit of a
  // tail tile issues none of its part loads and waits at most this long.
  uint64_t withhold_fixup_ns = 0;
};

constexpr int kPartFloats = 128 * 256;  // one CTA's share of a 256 x 256 tile

struct WorkUnit {
  int t;         // tile index (raster order)
  int kb0, kb1;  // K blocks [kb0, kb1)
  int s;         // K range of a tail tile, or -1 for a whole tile
};

// Unit number `it` of pair `slot` (of `num_slots`); false when it has none.
__device__ __forceinline__ bool work_unit(int it, int slot, int num_slots, int num_tiles, int num_kb,
                                          const SplitTail& st, WorkUnit& u) {
  const int full = (st.S <= 1) ? 0x7fffffff : st.dp_tiles / num_slots;
  if (it < full) {
    u.t = slot + it * num_slots;
    u.kb0 = 0;
    u.kb1 = num_kb;
    u.s = -1;
    return u.t < num_tiles;
  }
  if (it > full || slot >= (num_tiles - st.dp_tiles) * st.S) return false;
  u.t = st.dp_tiles + slot / st.S;
  u.s = slot % st.S;
  u.kb0 = static_cast<int>(static_cast<long long>(u.s) * num_kb / st.S);
  u.kb1 = static_cast<int>(static_cast<long long>(u.s + 1) * num_kb / st.S);
  return true;
}

// Float offset of lane `lane`'s float4 number q of 64-column chunk c of TMEM
// quadrant `quad` inside one part: consecutive lanes are consecutive 16-byte
// words, so every warp-wide access moves 512 contiguous bytes.
__device__ __forceinline__ int part_offset(int quad, int c, int q, int lane) {
  return (((quad * 4 + c) * 16 + q) * 32 + lane) * 4;
}

// Counts this unit's arrival at its tail tile; true for the last of S.  The
// last arrival resets the counter to 0 once the tile is stored, so every
// launch finds its counters at 0 (the library clears them after a launch that
// raised the device error word).
__device__ __forceinline__ bool split_arrive_last(uint32_t* ctr, int S) {
  return atomicAdd(ctr, 1u) == static_cast<uint32_t>(S - 1);
}


}  // namespace b200
