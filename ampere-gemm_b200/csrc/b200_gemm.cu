// B200 (sm_100a) FP16 GEMM: C[M,N] = A[M,K] * B, fp16 in, fp32 accumulate in
// tensor memory, fp16 out (round-to-nearest-even), behind a C ABI.
//
// Replaces the reference's L4/Ampere kernels (tensorcore_gemm/gemm.cu:1073
// `..._reg_pingpong_256`, :1373 `_colb`, :1811 `_MMA`, :1972 `_colb_MMA`) and
// their launcher `root_gemm_cuda` (tensorcore_gemm/gemm.py:31-154).  The math
// is the same as the reference epilogue `__float2half(alpha * acc)` with
// alpha = 1, beta = 0 (gemm.cu:1360-1361): an fp32 sum of fp16 products,
// rounded once to fp16.
//
// Kernel structure (one persistent CTA per SM, 192 threads, 6 warps):
//   warp 0      TMA producer: loads A (K-major) and B (K-major "colb" or
//               MN-major row-major) k-blocks into a STAGES-deep shared ring.
//   warp 1      allocates TMEM, and one lane issues tcgen05.mma (128 x BN x 16
//               per instruction) into one of two TMEM accumulators.
//   warps 2..5  epilogue: tcgen05.ld -> fp16 -> 128B-swizzled shared tile ->
//               TMA store; releases the accumulator as soon as it is read, so
//               the next tile's mainloop overlaps this tile's stores.
// Out-of-range rows/columns (any M, N, K) are handled by TMA zero fill on
// loads and clipping on stores.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "sm100_ptx.cuh"
#include "umma_desc.h"
#include "../../include/b200_gemm.h"

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

template <int BN, int STAGES, bool kBRowMajor>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_f16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                            const __grid_constant__ CUtensorMap tmap_c, int M, int N, int K, int group_m) {
  using Cfg = TileConfig<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * Cfg::kABytes;
  uint8_t* smem_epi = smem + STAGES * Cfg::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + Cfg::kEpiBytes);
  uint64_t* full_bar = bars;                    // [STAGES]  TMA -> MMA
  uint64_t* empty_bar = bars + STAGES;          // [STAGES]  MMA -> TMA
  uint64_t* tmem_full = bars + 2 * STAGES;      // [2]       MMA -> epilogue
  uint64_t* tmem_empty = bars + 2 * STAGES + 2; // [2]       epilogue -> MMA
  uint64_t* mma_drain = bars + 2 * STAGES + 4;  // [1]       abort path only
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  TileScheduler sched;
  sched.num_m = (M + kBM - 1) / kBM;
  sched.num_n = (N + BN - 1) / BN;
  sched.group_m = group_m;
  const int num_tiles = sched.num_m * sched.num_n;
  const int num_kb = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_c);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], kEpiWarps);
    }
    mbar_init(mma_drain, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(tmem_base_slot, Cfg::kTmemCols);
    tmem_relinquish_alloc_permit<1>();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ---------------- TMA producer (one lane) ----------------
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_normal();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        sched.tile_coords(t, mb, nb);
        const int m0 = mb * kBM, n0 = nb * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, kDevTimeoutProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
          const int k0 = kb * kBK;
          tma_load_2d(smem_a + stage * Cfg::kABytes, &tmap_a, &full_bar[stage], k0, m0, pol_a);
          uint8_t* b_dst = smem_b + stage * Cfg::kBBytes;
          if constexpr (kBRowMajor) {
            // B is K x N with N contiguous: BN/64 panels of 64 columns x 64 K-rows.
#pragma unroll
            for (int p = 0; p < BN / 64; ++p)
              tma_load_2d(b_dst + p * (kBK * 128), &tmap_b, &full_bar[stage], n0 + 64 * p, k0, pol_b);
          } else {
            // B is N x K with K contiguous: one box of BN rows x 64 K.
            tma_load_2d(b_dst, &tmap_b, &full_bar[stage], k0, n0, pol_b);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // Let every load still in flight land before the CTA leaves.
        const uint32_t pending = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (uint32_t i = 0; i < pending; ++i) {
          if (--s < 0) { s = STAGES - 1; ph ^= 1u; }
          mbar_wait_drain(&full_bar[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one lane) ----------------
    if (lane == 0) {
      constexpr uint32_t idesc =
          make_idesc_f16_f32(kBM, BN, Major::kK, kBRowMajor ? Major::kMN : Major::kK);
      const uint32_t a_base = smem_u32(smem_a);
      const uint32_t b_base = smem_u32(smem_b);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool any_mma = false;
      int local = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after_sync();
          const uint32_t a_addr = a_base + stage * Cfg::kABytes;
          const uint32_t b_addr = b_base + stage * Cfg::kBBytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t adesc = make_desc_kmajor_sw128(a_addr + k * (kUmmaK * 2));
            uint64_t bdesc;
            if constexpr (kBRowMajor)
              bdesc = make_desc_mnmajor_sw128(b_addr + k * (kUmmaK * 128), kBK * 128);
            else
              bdesc = make_desc_kmajor_sw128(b_addr + k * (kUmmaK * 2));
            umma_f16_cta1(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          any_mma = true;
          umma_commit_cta1(&empty_bar[stage]);  // frees the stage once these MMAs have read it
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_cta1(&tmem_full[acc]);       // accumulator ready for the epilogue
      }
      if (!ok && any_mma) {
        umma_commit_cta1(mma_drain);
        mbar_wait_drain(mma_drain, 0);
      }
    }
  } else {
    // ---------------- epilogue warps 2..5 ----------------
    const int quad = warp & 3;                    // TMEM lanes [32*quad, 32*quad+32)
    const int ew = warp - 2;                      // 0..3: private staging buffers
    uint8_t* epi_buf = smem_epi + ew * 2 * kEpiBufBytes;
    const uint32_t epi_addr = smem_u32(epi_buf);
    int buf = 0;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int mb, nb;
      sched.tile_coords(t, mb, nb);
      const int m0 = mb * kBM, n0 = nb * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tmem_full[acc], acc_phase, kDevTimeoutEpilogue)) break;
      tc_fence_after_sync();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / kEpiCols; ++c) {
        uint32_t lo[32], hi[32];
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, lo);
        tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, hi);
        tmem_ld_wait_regs(lo);
        tmem_ld_wait_regs(hi);
        if (c == BN / kEpiCols - 1) {
          // Whole accumulator is in registers: hand it back to the MMA warp.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[acc]);
        }
        // The store that last used this buffer must have finished reading it.
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        const uint32_t row_addr = epi_addr + buf * kEpiBufBytes + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t* v = (j < 4) ? (lo + 8 * j) : (hi + 8 * (j - 4));
          const uint32_t p0 = pack_half2_rn(v[0], v[1]);
          const uint32_t p1 = pack_half2_rn(v[2], v[3]);
          const uint32_t p2 = pack_half2_rn(v[4], v[5]);
          const uint32_t p3 = pack_half2_rn(v[6], v[7]);
          st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), p0, p1, p2, p3);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_c, epi_buf + buf * kEpiBufBytes, n0 + c * kEpiCols, m0 + quad * 32);
          bulk_commit_group();
        }
        buf ^= 1;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc<1>(tmem_base, Cfg::kTmemCols);
  }
}

// ===========================================================================
// Host side
// ===========================================================================
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool ready = false;
  bool sm100 = false;
  int sm_count = 0;
};

std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];

int current_device_info(DeviceInfo& out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B200_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return B200_ERR_CUDA;
    d.sm100 = (major == 10);
    d.sm_count = sms;
    d.ready = true;
  }
  out = d;
  return B200_OK;
}

// 2-D fp16 tensor map over a row-major matrix of `rows` x `cols` (cols
// contiguous, `ld` elements between rows), box `box_cols` x `box_rows`,
// 128-byte swizzle, zero fill out of bounds.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapL2promotion promo) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return B200_ERR_TENSOR_MAP;
  // A zero-extent dimension is not encodable; callers never pass one.
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TENSOR_MAP;
}

template <int BN, int STAGES, bool kBRowMajor>
int launch_tcgen05(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda, int64_t ldb,
                   int64_t ldc, int sm_count, int group_m, cudaStream_t stream) {
  using Cfg = TileConfig<BN, STAGES>;
  CUtensorMap ta, tb, tc;
  int rc = make_tmap_2d(&ta, A, M, K, lda, kBK, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  if (kBRowMajor)
    rc = make_tmap_2d(&tb, B, K, N, ldb, 64, kBK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  else
    rc = make_tmap_2d(&tb, B, N, K, ldb, kBK, BN, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = make_tmap_2d(&tc, C, M, N, ldc, kEpiCols, kEpiRows, CU_TENSOR_MAP_L2_PROMOTION_NONE);
  if (rc) return rc;

  auto kern = gemm_f16_tcgen05_kernel<BN, STAGES, kBRowMajor>;
  // Per-function attribute; cheap, and set every call so a new device or
  // context never sees the 48 KB default.
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) != cudaSuccess)
    return B200_ERR_CUDA;
  const long long tiles = (long long)((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int grid = (int)std::min<long long>(tiles, sm_count);
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tc, M, N, K, group_m);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b200

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" int b200_gemm_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                             int64_t ldb, int64_t ldc, int b_layout, void* stream_ptr) {
  using namespace b200;
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARGUMENT;
  if (b_layout != B200_B_ROW_MAJOR && b_layout != B200_B_COL_MAJOR) return B200_ERR_INVALID_ARGUMENT;
  const int64_t kMax = 0x7fffffff;
  if (M > kMax || N > kMax || K > kMax) return B200_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return B200_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (!C) return B200_ERR_INVALID_ARGUMENT;
  if (ldc < N) return B200_ERR_INVALID_ARGUMENT;
  if (!aligned16(C) || (ldc % 8) != 0) return B200_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (!dev.sm100) return B200_ERR_UNSUPPORTED_DEVICE;
  if (K == 0) {
    // Empty reduction: C is all zeros.
    return cudaMemset2DAsync(C, ldc * 2, 0, N * 2, M, stream) == cudaSuccess ? B200_OK : B200_ERR_CUDA;
  }
  if (!A || !B) return B200_ERR_INVALID_ARGUMENT;
  const bool row_b = (b_layout == B200_B_ROW_MAJOR);
  if (lda < K || ldb < (row_b ? N : K)) return B200_ERR_INVALID_ARGUMENT;
  if (!aligned16(A) || !aligned16(B) || (lda % 8) != 0 || (ldb % 8) != 0) return B200_ERR_MISALIGNED;

  const int m = (int)M, n = (int)N, k = (int)K;
  const int group_m = 8;
  if (row_b)
    return launch_tcgen05<256, 4, true>(A, B, C, m, n, k, lda, ldb, ldc, dev.sm_count, group_m, stream);
  return launch_tcgen05<256, 4, false>(A, B, C, m, n, k, lda, ldb, ldc, dev.sm_count, group_m, stream);
}

extern "C" const char* b200_gemm_strerror(int code) {
  switch (code) {
    case B200_OK: return "success";
    case B200_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, negative size, bad layout or leading dimension too small)";
    case B200_ERR_MISALIGNED: return "misaligned operand: base pointers must be 16-byte aligned and leading dimensions multiples of 8 elements";
    case B200_ERR_TOO_LARGE: return "dimension exceeds 2^31 - 1";
    case B200_ERR_CUDA: return "CUDA runtime error or kernel launch failure";
    case B200_ERR_TENSOR_MAP: return "cuTensorMapEncodeTiled unavailable or rejected the tensor map";
    case B200_ERR_DEVICE: return "device error word set: a bounded wait inside the kernel timed out";
    case B200_ERR_UNSUPPORTED_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    default: return "unknown error code";
  }
}

extern "C" int b200_gemm_last_device_error(void) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, b200::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  if (v != 0 && cudaMemcpyToSymbol(b200::g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
  return v;
}

extern "C" int b200_gemm_sm_count(void) {
  b200::DeviceInfo d;
  if (b200::current_device_info(d)) return 0;
  return d.sm_count;
}

extern "C" int b200_gemm_version(void) { return 100; }
