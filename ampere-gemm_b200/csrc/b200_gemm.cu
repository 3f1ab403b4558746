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
#include <atomic>
#include <cstdint>
#include <cstring>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <type_traits>
#include <utility>

#include "gemm_common.cuh"
#include "kernel_cta1.cuh"
#include "kernel_cta2.cuh"
#include "kernel_skinny.cuh"
#include "../../include/b200_gemm.h"

namespace b200 {

// Self-test of the bounded-wait path: one thread waits on an mbarrier that
// nothing ever arrives at, gives up after `limit_ns`, records
// kDevTimeoutSelftest in the device error word and returns.
__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
    mbar_wait(&bar, 0, kDevTimeoutSelftest, limit_ns);
  }
}

}  // namespace b200

// ===========================================================================
// Host side
// ===========================================================================
namespace b200 {
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
  int64_t l2_bytes = 0;
};

std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];

int current_device_info(DeviceInfo& out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B200_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int major = 0, sms = 0, l2 = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev) != cudaSuccess)
      return B200_ERR_CUDA;
    d.sm100 = (major == 10);
    d.sm_count = sms;
    d.l2_bytes = l2;
    d.ready = true;
  }
  out = d;
  return B200_OK;
}

// 2-D fp16 tensor map over a row-major matrix of `rows` x `cols` (cols
// contiguous, `ld` elements between rows), box `box_cols` x `box_rows`,
// 128-byte swizzle, zero fill out of bounds.
int encode_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols,
                   uint32_t box_rows, CUtensorMapL2promotion promo) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return B200_ERR_TENSOR_MAP;
  // A zero-extent dimension is not encodable; callers never pass one.
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  auto encode = [&] {
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    // A thread that has made no runtime call yet (e.g. autograd's device
    // thread) has no current context for this driver call: cudaSetDevice on
    // the current device makes the primary context current, then retry.
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = encode();
  }
  if (r != CUDA_SUCCESS && std::getenv("B200_GEMM_DEBUG"))
    std::fprintf(stderr, "b200_gemm: tensor map rejected (%d): base %p rows %llu cols %llu ld %llu box %u x %u\n",
                 (int)r, base, (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)ld, box_cols,
                 box_rows);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TENSOR_MAP;
}

// Encoding a tensor map is a driver call of about a microsecond; repeated
// GEMMs on the same buffers reuse the encoded map from a small per-thread
// cache keyed by every field that goes into it.
struct TmapKey {
  const void* base;
  uint64_t rows, cols, ld;
  uint32_t box_cols, box_rows, promo;
  bool operator==(const TmapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && ld == o.ld && box_cols == o.box_cols &&
           box_rows == o.box_rows && promo == o.promo;
  }
};

struct TmapCache {
  static constexpr int kEntries = 24;
  TmapKey key[kEntries];
  CUtensorMap map[kEntries];
  bool used[kEntries] = {};
  int next = 0;
};

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapL2promotion promo) {
  static thread_local TmapCache cache;
  const TmapKey k{base, rows, cols, ld, box_cols, box_rows, static_cast<uint32_t>(promo)};
  for (int i = 0; i < TmapCache::kEntries; ++i) {
    if (cache.used[i] && cache.key[i] == k) {
      *map = cache.map[i];
      return B200_OK;
    }
  }
  const int rc = encode_tmap_2d(map, base, rows, cols, ld, box_cols, box_rows, promo);
  if (rc != B200_OK) return rc;
  const int slot = cache.next;
  cache.next = (cache.next + 1) % TmapCache::kEntries;
  cache.key[slot] = k;
  cache.map[slot] = *map;
  cache.used[slot] = true;
  return B200_OK;
}

// cudaFuncSetAttribute once per (kernel instantiation, device); `done` is
// the calling launch template's own flag array (all kernels share one
// function-pointer type, so the flags cannot live here).
template <typename Kern>
int ensure_smem_attr(Kern kern, int smem_bytes, std::atomic<uint8_t>* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire)) return B200_OK;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
    return B200_ERR_CUDA;
  if (dev >= 0 && dev < kMaxDevices) done[dev].store(1, std::memory_order_release);
  return B200_OK;
}

// GEMM kernels go out with programmatic stream serialisation (PDL): a kernel
// may be scheduled while the previous one on the stream drains, runs its
// setup (barriers, TMEM, tensor-map prefetch), and waits in griddep_wait()
// before its first global access.  B200_GEMM_PDL=0 turns it off.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B200_GEMM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_gemm(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                        Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) (void)cudaGetLastError();
  return e;
}

// One GEMM call as the launchers see it (operands already TMA-compatible).
struct GemmArgs {
  const void* A;
  const void* B;
  void* C;
  int M, N, K;
  int64_t lda, ldb, ldc;
  EpiParams scale;
  int sm_count;
  cudaStream_t stream;
  ArgminOut argmin = ArgminOut{};
};

// Width of C's tensor map: the columns the TMA store covers (at least one
// column so the map encodes; when N < 8 it is never used).
inline int c_map_cols(const GemmArgs& g) { return g.scale.n_tma > 0 ? g.scale.n_tma : g.N; }

// Calls fn(row-major B, column-major A) with the two layouts as compile-time
// constants, so every launcher is instantiated for the four combinations.
template <typename Fn>
int with_layouts(bool row_b, bool col_a, Fn&& fn) {
  if (row_b) return col_a ? fn(std::true_type{}, std::true_type{}) : fn(std::true_type{}, std::false_type{});
  return col_a ? fn(std::false_type{}, std::true_type{}) : fn(std::false_type{}, std::false_type{});
}

template <int BN, int STAGES, bool kBRowMajor, bool kAColMajor>
int launch_tcgen05(const GemmArgs& g, int group_m) {
  using Cfg = TileConfig<BN, STAGES>;
  const void *A = g.A, *B = g.B;
  void* C = g.C;
  const int M = g.M, N = g.N, K = g.K;
  const int64_t lda = g.lda, ldb = g.ldb, ldc = g.ldc;
  const int sm_count = g.sm_count;
  cudaStream_t stream = g.stream;
  CUtensorMap ta, tb, tc;
  int rc = kAColMajor ? make_tmap_2d(&ta, A, K, M, lda, 64, kBK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)
                      : make_tmap_2d(&ta, A, M, K, lda, kBK, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  if (kBRowMajor)
    rc = make_tmap_2d(&tb, B, K, N, ldb, 64, kBK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  else
    rc = make_tmap_2d(&tb, B, N, K, ldb, kBK, BN, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = make_tmap_2d(&tc, C, M, c_map_cols(g), ldc, kEpiCols, kEpiRows, CU_TENSOR_MAP_L2_PROMOTION_NONE);
  if (rc) return rc;

  auto kern = gemm_f16_tcgen05_kernel<BN, STAGES, kBRowMajor, kAColMajor>;
  static std::atomic<uint8_t> attr_done[kMaxDevices];
  if (int e = ensure_smem_attr(kern, Cfg::kSmemBytes, attr_done)) return e;
  const long long tiles = (long long)((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int grid = (int)std::min<long long>(tiles, sm_count);
  const cudaError_t le = launch_gemm(kern, dim3(grid), dim3(kThreads), Cfg::kSmemBytes, stream, ta, tb, tc, M, N, K,
                                     group_m, g.scale);
  return le == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

// Largest number of 2-CTA clusters of `kern` that can be resident at once
// (clusters need both SMs in one GPC, so this can be below sm_count / 2).
template <typename Kern>
int max_active_pairs(Kern kern, int smem_bytes, int sm_count) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (sm_count / 2), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = sm_count / 2;
  }
  return n;
}

// ---- split of the last wave along K (pair kernel, MSUB = 1) ----
// Cost model in SM cycles: a 256 x 256 pair tile spends 1024 cycles per
// 128-deep K stage.  A split tail costs about 8.1k cycles plus 3.4k per K
// range (writing the parts, the arrival, the last unit's read-back and sum),
// fitted to 2560 x 2048 x 8192 at S = 2, 3, 4, 7 (saved time against the
// ideal T (1 - 1/S)).  So only deep K pays: at K = 2048 the split is slower,
// at K = 4096 even, at K = 8192 S = 4 saves 16 %.
constexpr double kPairStageCycles = 1024.0;
constexpr double kSplitFixedCycles = 8100.0;
constexpr double kSplitPartCycles = 3400.0;

// K ranges per tail tile that minimise the last wave's time (1 = no split).
int choose_split(int num_kb, long long smax) {
  // B200_GEMM_SPLIT_S forces the number of K ranges (tuning only).
  static const int forced = [] {
    const char* e = std::getenv("B200_GEMM_SPLIT_S");
    return e ? std::atoi(e) : 0;
  }();
  if (forced >= 1) return (int)std::max<long long>(1, std::min<long long>({(long long)forced, smax, kFixBufs + 1,
                                                                         num_kb / 2}));
  int best = 1;
  double best_cost = num_kb * kPairStageCycles;
  for (int S = 2; S <= smax && S <= kFixBufs + 1 && 2 * S <= num_kb; ++S) {  // fixup holds S - 1 parts
    const double c = num_kb * kPairStageCycles / S + kSplitFixedCycles + kSplitPartCycles * S;
    if (c < best_cost * 0.97) {
      best_cost = c;
      best = S;
    }
  }
  return best;
}

// Last wave's time as a fraction of a whole tile's, with the split the
// launcher would choose.
double pair_tail_fraction(int num_kb, long long tiles, int slots) {
  const long long r = tiles % slots;
  if (r == 0) return 1.0;
  if (tiles < slots) return 1.0;  // a single partial wave is never split
  const int S = choose_split(num_kb, slots / r);
  if (S == 1) return 1.0;
  return (num_kb * kPairStageCycles / S + kSplitFixedCycles + kSplitPartCycles * S) / (num_kb * kPairStageCycles);
}

bool split_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B200_GEMM_SPLIT");
    return !(e && e[0] == '0');
  }();
  return on;
}

// K ranges the 256 x 256 pair kernel cuts its last wave into (1 = none) for
// `tiles` tiles on `grid_pairs` resident pairs and `num_kb` 128-deep K stages.
int split_ranges_for(long long tiles, int grid_pairs, int num_kb) {
  if (!split_enabled() || grid_pairs <= 0 || tiles <= grid_pairs || tiles % grid_pairs == 0) return 1;
  return choose_split(num_kb, grid_pairs / (tiles % grid_pairs));
}

// One workspace per (device, stream): launches on one stream are ordered, so
// they can share it; other streams get their own.  Allocated on first use
// (never during a stream capture: that launch then runs unsplit).
struct SplitWorkspace {
  int dev;
  cudaStream_t stream;
  float* parts;
  uint32_t* counters;
  int max_parts;
};

std::mutex g_split_mu;
SplitWorkspace g_split_ws[64];
int g_split_n = 0;

bool split_workspace(cudaStream_t stream, int sm_count, SplitTail& st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(g_split_mu);
  SplitWorkspace* w = nullptr;
  for (int i = 0; i < g_split_n; ++i)
    if (g_split_ws[i].dev == dev && g_split_ws[i].stream == stream) w = &g_split_ws[i];
  if (!w) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
    if (g_split_n == 64) return false;
    const int max_parts = sm_count;  // R * S <= pairs, two CTAs each
    const size_t part_bytes = (size_t)max_parts * kPartFloats * sizeof(float);
    void* mem = nullptr;
    if (cudaMalloc(&mem, part_bytes + (size_t)max_parts * sizeof(uint32_t)) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    uint32_t* ctr = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(mem) + part_bytes);
    if (cudaMemsetAsync(ctr, 0, (size_t)max_parts * sizeof(uint32_t), stream) != cudaSuccess) {
      cudaFree(mem);
      return false;
    }
    w = &g_split_ws[g_split_n++];
    *w = SplitWorkspace{dev, stream, static_cast<float*>(mem), ctr, max_parts};
  }
  st.ws = w->parts;
  st.counters = w->counters;
  return true;  // R * S <= pairs <= sm_count / 2, so the parts always fit
}

// Zeroes the tail counters of every workspace on the current device (after a
// launch that gave up on a bounded wait; the device is idle then).
void reset_split_counters() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  std::lock_guard<std::mutex> lock(g_split_mu);
  for (int i = 0; i < g_split_n; ++i)
    if (g_split_ws[i].dev == dev)
      (void)cudaMemset(g_split_ws[i].counters, 0, (size_t)g_split_ws[i].max_parts * sizeof(uint32_t));
}

// Per-call launch options, set by an entry point for the duration of one
// (host-synchronous) call on this thread.
struct CallOptions {
  bool no_split = false;           // run every tile whole: no split workspace (allocation-free entry)
  uint64_t withhold_fixup_ns = 0;  // fixup-wait self-test (see SplitTail)
  int force_variant = -1;          // >= 0: this variant instead of b200_gemm_set_variant's / auto
};
thread_local CallOptions t_call;

struct ScopedCallOptions {
  CallOptions saved;
  explicit ScopedCallOptions(const CallOptions& o) : saved(t_call) { t_call = o; }
  ~ScopedCallOptions() { t_call = saved; }
};

template <int STAGES, int KSUB, int MSUB, bool kBRowMajor, bool kAColMajor, int BN = 256, bool kDyn = false>
int launch_tcgen05_pair(const GemmArgs& g, int group_m) {
  using Cfg = PairConfig<STAGES, KSUB, MSUB, BN>;
  const void *A = g.A, *B = g.B;
  void* C = g.C;
  const int M = g.M, N = g.N, K = g.K;
  const int64_t lda = g.lda, ldb = g.ldb, ldc = g.ldc;
  const int sm_count = g.sm_count;
  cudaStream_t stream = g.stream;
  CUtensorMap ta, tb, tc;
  int rc = kAColMajor ? make_tmap_2d(&ta, A, K, M, lda, 64, Cfg::kStageK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)
                      : make_tmap_2d(&ta, A, M, K, lda, kBK, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  if (kBRowMajor)
    rc = make_tmap_2d(&tb, B, K, N, ldb, 64, Cfg::kStageK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  else
    rc = make_tmap_2d(&tb, B, N, K, ldb, kBK, Cfg::kHalfN, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = make_tmap_2d(&tc, C, M, c_map_cols(g), ldc, kEpiCols, kEpiRows, CU_TENSOR_MAP_L2_PROMOTION_NONE);
  if (rc) return rc;
  auto kern = gemm_f16_tcgen05_pair_kernel<STAGES, KSUB, MSUB, kBRowMajor, kAColMajor, BN, kDyn>;
  static std::atomic<uint8_t> attr_done[kMaxDevices];
  if (int e = ensure_smem_attr(kern, Cfg::kSmemBytes, attr_done)) return e;
  static int pairs_cache[kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int pairs = (dev >= 0 && dev < kMaxDevices) ? pairs_cache[dev] : 0;
  if (pairs <= 0) {
    pairs = max_active_pairs(kern, Cfg::kSmemBytes, sm_count);
    if (dev >= 0 && dev < kMaxDevices) pairs_cache[dev] = pairs;
    if (std::getenv("B200_GEMM_DEBUG")) std::fprintf(stderr, "b200_gemm: %d resident 2-CTA clusters\n", pairs);
  }
  const long long tiles = (long long)((M + Cfg::kTileM - 1) / Cfg::kTileM) * ((N + Cfg::kTileN - 1) / Cfg::kTileN);
  // Dynamic tiles launch one cluster per tile (those that have not started
  // when a running pair needs work are cancelled and their tiles taken).
  const int grid_pairs = kDyn ? (int)tiles : (int)std::min<long long>(tiles, pairs);
  if (kDyn && tiles > 0x3fffffffLL) return B200_ERR_TOO_LARGE;
  SplitTail st;
  const int S = (MSUB == 1 && !kDyn && !t_call.no_split)
                    ? split_ranges_for(tiles, grid_pairs, (K + Cfg::kStageK - 1) / Cfg::kStageK)
                    : 1;
  if (S >= 2) {
    const long long r = tiles % grid_pairs;
    SplitTail s2;
    s2.dp_tiles = (int)(tiles - r);
    s2.S = S;
    s2.withhold_fixup_ns = t_call.withhold_fixup_ns;
    if (split_workspace(stream, sm_count, s2)) st = s2;
    if (std::getenv("B200_GEMM_DEBUG"))
      std::fprintf(stderr, "b200_gemm: %lld tiles on %d pairs, last %lld tiles split %d ways%s\n", tiles, grid_pairs, r,
                   S, st.S > 1 ? "" : " (no workspace: unsplit)");
  }
  const cudaError_t le = launch_gemm(kern, dim3(2 * grid_pairs), dim3(kThreads), Cfg::kSmemBytes, stream, ta, tb, tc,
                                     M, N, K, group_m, g.scale, st);
  return le == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

// Skinny (K <= 256) B-stationary kernel.  The grid is the largest multiple of
// the number of 256-column N slices that fits the SMs, so every CTA keeps one
// slice of B resident.  Returns B200_ERR_INVALID_ARGUMENT when the shape does
// not qualify (caller falls back to another variant).
template <int A_STAGES, int EPI_BUFS, bool kBRowMajor, bool kAColMajor, bool kArgmin = false, int EPI_W = kEpiWarps>
int launch_skinny(const GemmArgs& g) {
  using Cfg = SkinnyConfig<A_STAGES, EPI_BUFS, EPI_W>;
  const void *A = g.A, *B = g.B;
  void* C = g.C;
  const int M = g.M, N = g.N, K = g.K;
  const int64_t lda = g.lda, ldb = g.ldb, ldc = g.ldc;
  const int sm_count = g.sm_count;
  cudaStream_t stream = g.stream;
  const int num_nb = (N + Cfg::kBN - 1) / Cfg::kBN;
  if (K > Cfg::kMaxKBlocks * kBK || num_nb > sm_count) return B200_ERR_INVALID_ARGUMENT;
  CUtensorMap ta, tb, tc;
  int rc = kAColMajor ? make_tmap_2d(&ta, A, K, M, lda, 64, kBK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)
                      : make_tmap_2d(&ta, A, M, K, lda, kBK, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  if (kBRowMajor)
    rc = make_tmap_2d(&tb, B, K, N, ldb, 64, kBK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  else
    rc = make_tmap_2d(&tb, B, N, K, ldb, kBK, Cfg::kBN, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  if constexpr (kArgmin)
    tc = ta;  // no C: the argmin epilogue writes keys, the map is never used
  else
    rc = make_tmap_2d(&tc, C, M, c_map_cols(g), ldc, kEpiCols, kEpiRows, CU_TENSOR_MAP_L2_PROMOTION_NONE);
  if (rc) return rc;
  auto kern = gemm_f16_skinny_kernel<A_STAGES, EPI_BUFS, kBRowMajor, kAColMajor, kArgmin, EPI_W>;
  static std::atomic<uint8_t> attr_done[kMaxDevices];
  if (int e = ensure_smem_attr(kern, Cfg::kSmemBytes, attr_done)) return e;
  const long long tiles = (long long)((M + kBM - 1) / kBM) * num_nb;
  const int slots = (sm_count / num_nb) * num_nb;
  const int grid = (int)std::min<long long>(tiles, slots);
  const cudaError_t le = launch_gemm(kern, dim3(grid), dim3(skinny_threads(kArgmin, EPI_W)), Cfg::kSmemBytes, stream, ta, tb,
                                     tc, M, N, K, g.scale, g.argmin);
  return le == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

// Kernel choice for K > 256.  Each persistent variant runs its tiles in waves
// of `slots` concurrent tiles; the last wave is usually partial, so the
// estimate is  waves * (per-SM tile work) / (relative per-SM rate).  Rates are
// measured steady-state throughputs relative to the wide pair (8192^3:
// 1.00 wide pair, 0.96 pair, 0.93 one-CTA); the model reproduces the best
// measured variant on 2048^3 .. 8192^3, 4096 x 8192 x 4096, 8192 x 4096 x 4096,
// 4000 x 6000 x 3000 and 65536 x 8192 x 8192.
// Tile width of the wide pair kernel (256, 224 or 192 columns) for an
// m x n product on `slots` resident pairs.  The MMAs of a narrower tile take
// proportionally less time, but the kernel's stages hold the same bytes
// whatever the width, and measured tile times barely fall with it (4000 x
// 6000 x 3000: 120.4 us at 256 against 122.6 at 224 over the same 3 waves;
// 4096 x 8192 x 4096: 201.6 against 198.6 over 4 waves).  So a narrower tile
// pays only where it needs fewer waves, or within a single wave, where it
// spreads the same work over more SMs (2560 x 2048 x 2048: 23.9-27.0 us with
// 192-wide tiles against 31.5 with 256-wide); other ties keep the widest.
// Returns the width and, in *waves, its wave count.  B200_GEMM_WIDE_BN forces
// one (tuning only).
int wide_pair_bn(int m, int n, int slots, double* waves_out = nullptr) {
  static const int forced = [] {
    const char* e = std::getenv("B200_GEMM_WIDE_BN");
    const int v = e ? std::atoi(e) : 0;
    return (v == 256 || v == 224 || v == 192) ? v : 0;
  }();
  const int cand[3] = {256, 224, 192};
  int best = 256;
  long long best_w = -1;
  for (int bn : cand) {
    if (forced && bn != forced) continue;
    const long long tiles = (long long)((m + 511) / 512) * ((n + bn - 1) / bn);
    const long long w = (tiles + slots - 1) / slots;
    // Fewest waves; among equals the widest tile, except within a single
    // wave, where the narrowest gives each SM the least work.
    if (best_w < 0 || w < best_w || (w == best_w && w == 1 && bn < best)) {
      best_w = w;
      best = bn;
    }
  }
  if (waves_out) *waves_out = (double)best_w;
  return best;
}

int pick_tensor_variant(int m, int n, int k, int sm_count) {
  if (k < 512) return B200_VARIANT_CTA1;  // a pair's prologue is not amortised
  // One wave of 1-CTA tiles of moderate depth: every variant takes about one
  // tile's time and the 1-CTA kernel has the cheapest start (2048^3: 16.4-16.7
  // us against 17.3-17.6 for the pair kernel).  Deeper single-wave shapes go
  // through the model below (1536 x 1280 x 8192: pair 44.7 us against 47.5
  // for the 1-CTA kernel).
  if (k <= 4096 && (long long)((m + 127) / 128) * ((n + 255) / 256) <= sm_count) return B200_VARIANT_CTA1;
  // Cost in SM cycles: waves x one tile's MMA time / relative rate, plus the
  // last tile's accumulator drain (one 256-column block, two for the wide pair).
  struct Opt {
    int variant, tile_m, tile_n, slots, rows_per_sm;
    double rate, drain_cycles;
  };
  const int pairs = sm_count / 2;
  const Opt opts[3] = {
      // Wide pair drain: 3200 cycles since its epilogue releases each
      // accumulator block before storing it (3072^3: one wave of wide tiles
      // 43.0 us against 45.0 for two waves of the pair kernel).
      {B200_VARIANT_PAIR_WIDE, 512, 256, pairs, 256, 1.00, 3200.0},
      {B200_VARIANT_PAIR, 256, 256, pairs, 128, 0.96, 3200.0},
      {B200_VARIANT_CTA1, 128, 256, sm_count, 128, 0.93, 3200.0},
  };
  const double tile128_cycles = 8.0 * k;  // 128 x 256 rows x columns: k / 16 MMAs of 128 cycles
  int best = B200_VARIANT_CTA1;
  double best_cost = 1e300;
  for (const Opt& o : opts) {
    const long long tiles = (long long)((m + o.tile_m - 1) / o.tile_m) * ((n + o.tile_n - 1) / o.tile_n);
    double waves = (double)((tiles + o.slots - 1) / o.slots);
    double width = 1.0;  // tile time relative to a 256-wide tile
    if (o.variant == B200_VARIANT_PAIR_WIDE) {
      const int bn = wide_pair_bn(m, n, o.slots, &waves);  // best tile width's waves
      // In a single wave of moderate depth a narrower tile does finish sooner
      // (2560 x 2048 x 2048: 23.9 us for one wave of 192-wide tiles against
      // 26.0 for the pair kernel's two waves); over several waves it does not.
      if (waves <= 1.0 && k <= 4096) width = bn / 256.0;
    }
    if (o.variant == B200_VARIANT_PAIR && split_enabled() && tiles % o.slots != 0)
      waves = (double)(tiles / o.slots) + pair_tail_fraction((k + 127) / 128, tiles, o.slots);  // split last wave
    const double cost = waves * width * tile128_cycles * (o.rows_per_sm / 128.0) / o.rate + o.drain_cycles;
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = o.variant;
    }
  }
  if (best == B200_VARIANT_PAIR_WIDE) {
    const int bn = wide_pair_bn(m, n, pairs);
    if (bn == 224) return B200_VARIANT_PAIR_WIDE_224;
    if (bn == 192) return B200_VARIANT_PAIR_WIDE_192;
  }
  return best;
}

// The kernel the library runs for an m x n x k product when no variant is forced.
int auto_variant(int m, int n, int k, int sm_count) {
  if (k <= 256 && (n + 255) / 256 <= sm_count) {
    // B-stationary pays for its one-off B load once a CTA has several tiles
    // (measured: ahead from ~3 tiles per SM, behind at 1-2).
    const long long tiles = (long long)((m + 127) / 128) * ((n + 255) / 256);
    if (tiles >= 3LL * sm_count) return B200_VARIANT_SKINNY;
  }
  return pick_tensor_variant(m, n, k, sm_count);
}

// Process-wide kernel-variant override (b200_gemm_set_variant).
int g_variant = B200_VARIANT_AUTO;

// Raster band height in tiles; B200_GEMM_GROUP_M overrides it (tuning only).
int group_m_override() {
  static int v = [] {
    const char* e = std::getenv("B200_GEMM_GROUP_M");
    return e ? std::atoi(e) : 0;  // negative: bands of column blocks
  }();
  return v;
}

// Dynamic tile scheduling of the wide pair kernel (cluster launch control),
// used when its tiles take more than one wave: three interleaved rounds at
// 65536 x 8192 x 8192 ran 6341-6459 us against 6461-6506 static, 4000 x 6000
// x 3000 119.2 against 120.3; one-wave shapes have nothing to balance.
// B200_GEMM_DYN=0 turns it off (tuning).
bool dyn_tiles() {
  static const bool on = [] {
    const char* e = std::getenv("B200_GEMM_DYN");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b200

// ===========================================================================
// C ABI
// ===========================================================================
namespace b200 {
namespace {

// Arguments common to every entry point.  Returns B200_OK, or an error code;
// sets *nothing_to_do when the output is empty.
int validate_args(const void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                  int b_layout, const void* A, const void* B, bool* nothing_to_do, int a_layout = B200_A_ROW_MAJOR) {
  *nothing_to_do = false;
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARGUMENT;
  if (b_layout != B200_B_ROW_MAJOR && b_layout != B200_B_COL_MAJOR) return B200_ERR_INVALID_ARGUMENT;
  if (a_layout != B200_A_ROW_MAJOR && a_layout != B200_A_COL_MAJOR) return B200_ERR_INVALID_ARGUMENT;
  const int64_t kMax = 0x7fffffff;
  if (M > kMax || N > kMax || K > kMax) return B200_ERR_TOO_LARGE;
  if (M == 0 || N == 0) {
    *nothing_to_do = true;
    return B200_OK;
  }
  if (!C || ldc < N) return B200_ERR_INVALID_ARGUMENT;
  if (K > 0) {
    const bool row_b = (b_layout == B200_B_ROW_MAJOR);
    const bool col_a = (a_layout == B200_A_COL_MAJOR);
    if (!A || !B || lda < (col_a ? M : K) || ldb < (row_b ? N : K)) return B200_ERR_INVALID_ARGUMENT;
  }
  return B200_OK;
}

bool pitch_ok(const void* p, int64_t ld) { return aligned16(p) && (ld % 8) == 0; }

// C <- fp16_rn(beta * C) for an empty reduction (K == 0) with beta != 0.
__global__ void scale_c_kernel(uint16_t* C, int64_t ldc, int64_t rows, int64_t cols, float beta) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x) {
      __half h = *reinterpret_cast<__half*>(&C[r * ldc + c]);
      h = __float2half_rn(beta * __half2float(h));
      C[r * ldc + c] = *reinterpret_cast<uint16_t*>(&h);
    }
}

// C = alpha * op(A) * op(B) + beta * C on operands that already satisfy TMA's
// alignment rules.
int gemm_aligned(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                 int64_t ldc, int a_layout, int b_layout, const EpiParams& scale, const DeviceInfo& dev,
                 cudaStream_t stream) {
  if (K == 0) {
    // Empty reduction: C = beta * C (all zeros when beta == 0).
    if (scale.beta == 0.0f)
      return cudaMemset2DAsync(C, ldc * 2, 0, N * 2, M, stream) == cudaSuccess ? B200_OK : B200_ERR_CUDA;
    const unsigned gx = (unsigned)std::min<int64_t>((N + 255) / 256, 64);
    const unsigned gy = (unsigned)std::min<int64_t>(M, 65535);
    scale_c_kernel<<<dim3(gx, gy), 256, 0, stream>>>(static_cast<uint16_t*>(C), ldc, M, N, scale.beta);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
  }
  const bool row_b = (b_layout == B200_B_ROW_MAJOR);
  const bool col_a = (a_layout == B200_A_COL_MAJOR);
  const int m = (int)M, n = (int)N, k = (int)K;
  EpiParams ep = scale;
  ep.m = m;
  ep.n = n;
  ep.ldc = ldc;
  ep.c = static_cast<uint16_t*>(C);
  ep.n_tma = n & ~7;  // a TMA store writes whole 16-byte pieces: the partial last one goes by plain stores
  ep.c_evict_first = (dev.l2_bytes > 0 && 2 * M * N > dev.l2_bytes) ? 1 : 0;
  const GemmArgs g{A, B, C, m, n, k, lda, ldb, ldc, ep, dev.sm_count, stream};
  int variant = t_call.force_variant >= 0 ? t_call.force_variant : g_variant;
  if (variant == B200_VARIANT_AUTO) variant = auto_variant(m, n, k, dev.sm_count);
  if (variant == B200_VARIANT_SKINNY) {
    const int rc = with_layouts(row_b, col_a, [&](auto rb, auto ca) {
      // Measured: 5 A stages with 4 epilogue warps beat 4 stages with 8 warps
      // (the A stream, not the epilogue, then sets the pace) and 4 stages
      // with two staging buffers per warp.
      return launch_skinny<5, 1, decltype(rb)::value, decltype(ca)::value>(g);
    });
    if (rc != B200_ERR_INVALID_ARGUMENT) return rc;
    variant = B200_VARIANT_CTA1;  // shape outside the skinny kernel's range
  }
  const int gm = group_m_override();
  if (variant == B200_VARIANT_PAIR_WIDE || variant == B200_VARIANT_PAIR_WIDE_224 ||
      variant == B200_VARIANT_PAIR_WIDE_192) {
    // Raster: when A is much taller than B is wide, bands of 12 column blocks
    // (65536 x 8192 x 8192 with C stored evict-first, two interleaved rounds:
    // 6435-6465 us against 6452-6482 for bands of 8, 6495-6579 for 16,
    // 6689-6748 for 32 and 6561-6566 for 8-row bands; DRAM reads per launch
    // 8.9 GB against 9.7-11.2 for bands of 8); otherwise bands of 8 row blocks.
    const int group_m = gm ? gm : (m >= 4LL * n ? -12 : 8);
    const int bn = variant == B200_VARIANT_PAIR_WIDE_224 ? 224 : variant == B200_VARIANT_PAIR_WIDE_192 ? 192 : 256;
    return with_layouts(row_b, col_a, [&](auto rb, auto ca) {
      constexpr bool kRb = decltype(rb)::value, kCa = decltype(ca)::value;
      if (bn == 224) return launch_tcgen05_pair<4, 1, 2, kRb, kCa, 224>(g, group_m);
      if (bn == 192) return launch_tcgen05_pair<4, 1, 2, kRb, kCa, 192>(g, group_m);
      if (dyn_tiles() && (long long)((m + 511) / 512) * ((n + 255) / 256) > dev.sm_count / 2)
        return launch_tcgen05_pair<4, 1, 2, kRb, kCa, 256, true>(g, group_m);
      return launch_tcgen05_pair<4, 1, 2, kRb, kCa, 256>(g, group_m);
    });
  }
  if (variant == B200_VARIANT_PAIR) {
    const int group_m = gm ? gm : 8;  // 8 x 256-row bands: fewest DRAM bytes measured at 8192^3
    // Several waves and no split last wave: dynamic tiles, as for the wide pair.
    const long long tiles = (long long)((m + 255) / 256) * ((n + 255) / 256);
    const int pairs = dev.sm_count / 2;
    const bool dyn = dyn_tiles() && tiles > pairs &&
                     (t_call.no_split || split_ranges_for(tiles, pairs, (k + 127) / 128) == 1);
    return with_layouts(row_b, col_a, [&](auto rb, auto ca) {
      constexpr bool kRb = decltype(rb)::value, kCa = decltype(ca)::value;
      if (dyn) return launch_tcgen05_pair<3, 2, 1, kRb, kCa, 256, true>(g, group_m);
      return launch_tcgen05_pair<3, 2, 1, kRb, kCa, 256>(g, group_m);
    });
  }
  const int group_m = gm ? gm : 16;  // 16 x 128-row bands: fewest DRAM bytes measured at 8192^3
  return with_layouts(row_b, col_a, [&](auto rb, auto ca) {
    return launch_tcgen05<256, 4, decltype(rb)::value, decltype(ca)::value>(g, group_m);
  });
}

// Copies a rows x cols fp16 matrix between row pitches (elements).
__global__ void pitched_copy_f16_kernel(const uint16_t* __restrict__ src, int64_t src_ld, uint16_t* __restrict__ dst,
                                        int64_t dst_ld, int64_t rows, int64_t cols) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x)
      dst[r * dst_ld + c] = src[r * src_ld + c];
}

int pitched_copy(const void* src, int64_t src_ld, void* dst, int64_t dst_ld, int64_t rows, int64_t cols,
                 cudaStream_t stream) {
  if (rows == 0 || cols == 0) return B200_OK;
  const unsigned gx = (unsigned)std::min<int64_t>((cols + 255) / 256, 64);
  const unsigned gy = (unsigned)std::min<int64_t>(rows, 65535);
  pitched_copy_f16_kernel<<<dim3(gx, gy), 256, 0, stream>>>(static_cast<const uint16_t*>(src), src_ld,
                                                             static_cast<uint16_t*>(dst), dst_ld, rows, cols);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

// Workspace plan for operands whose base or row pitch TMA cannot describe:
// each such operand gets a copy with a 16-byte row pitch (pitch rounded up
// to 8 elements) at a 256-byte aligned offset.  Unaligned C is computed into
// its copy and copied back.
struct RepackPlan {
  bool a = false, b = false, c = false;
  int64_t lda2 = 0, ldb2 = 0, ldc2 = 0;
  int64_t off_a = 0, off_b = 0, off_c = 0, bytes = 0;
};

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

RepackPlan plan_repack(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                       int64_t ldb, int64_t ldc, int b_layout, int a_layout = B200_A_ROW_MAJOR) {
  RepackPlan p;
  const bool row_b = (b_layout == B200_B_ROW_MAJOR);
  const bool col_a = (a_layout == B200_A_COL_MAJOR);
  if (K > 0) {
    p.a = !pitch_ok(A, lda);
    p.b = !pitch_ok(B, ldb);
  }
  p.c = !pitch_ok(C, ldc);
  int64_t off = 0;
  if (p.a) {
    const int64_t rows = col_a ? K : M, cols = col_a ? M : K;
    p.lda2 = round_up(cols, 8);
    p.off_a = off;
    off = round_up(off + rows * p.lda2 * 2, 256);
  }
  if (p.b) {
    const int64_t rows = row_b ? K : N, cols = row_b ? N : K;
    p.ldb2 = round_up(cols, 8);
    p.off_b = off;
    off = round_up(off + rows * p.ldb2 * 2, 256);
  }
  if (p.c) {
    p.ldc2 = round_up(N, 8);
    p.off_c = off;
    off = round_up(off + M * p.ldc2 * 2, 256);
  }
  p.bytes = off;
  return p;
}

// Repack (as planned), multiply, copy C back; `ws` is device memory of at
// least plan.bytes, 256-byte aligned.
int gemm_repacked(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                  int64_t ldc, int a_layout, int b_layout, const EpiParams& scale, const RepackPlan& p, uint8_t* ws,
                  const DeviceInfo& dev, cudaStream_t stream) {
  const bool row_b = (b_layout == B200_B_ROW_MAJOR);
  const bool col_a = (a_layout == B200_A_COL_MAJOR);
  const void* a = A;
  const void* b = B;
  void* c = C;
  int64_t la = lda, lb = ldb, lc = ldc;
  int rc = B200_OK;
  if (p.a) {
    a = ws + p.off_a;
    la = p.lda2;
    if ((rc = pitched_copy(A, lda, ws + p.off_a, la, col_a ? K : M, col_a ? M : K, stream))) return rc;
  }
  if (p.b) {
    b = ws + p.off_b;
    lb = p.ldb2;
    if ((rc = pitched_copy(B, ldb, ws + p.off_b, lb, row_b ? K : N, row_b ? N : K, stream))) return rc;
  }
  if (p.c) {
    c = ws + p.off_c;
    lc = p.ldc2;
    if (scale.beta != 0.0f && (rc = pitched_copy(C, ldc, c, lc, M, N, stream))) return rc;  // old C is an input
  }
  if ((rc = gemm_aligned(a, b, c, M, N, K, la, lb, lc, a_layout, b_layout, scale, dev, stream))) return rc;
  if (p.c) rc = pitched_copy(c, lc, C, ldc, M, N, stream);
  return rc;
}

}  // namespace
}  // namespace b200

extern "C" int b200_gemm_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                             int64_t ldb, int64_t ldc, int b_layout, void* stream_ptr) {
  using namespace b200;
  bool done = false;
  if (int rc = validate_args(C, M, N, K, lda, ldb, ldc, b_layout, A, B, &done)) return rc;
  if (done) return B200_OK;
  if (!pitch_ok(C, ldc)) return B200_ERR_MISALIGNED;
  if (K > 0 && (!pitch_ok(A, lda) || !pitch_ok(B, ldb))) return B200_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (!dev.sm100) return B200_ERR_UNSUPPORTED_DEVICE;
  return gemm_aligned(A, B, C, M, N, K, lda, ldb, ldc, B200_A_ROW_MAJOR, b_layout, EpiParams{}, dev,
                      static_cast<cudaStream_t>(stream_ptr));
}

extern "C" int64_t b200_gemm_workspace_size_ex(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                                               int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int a_layout,
                                               int b_layout) {
  using namespace b200;
  bool done = false;
  if (int rc = validate_args(C, M, N, K, lda, ldb, ldc, b_layout, A, B, &done, a_layout)) return -rc;
  if (done) return 0;
  return plan_repack(A, B, C, M, N, K, lda, ldb, ldc, b_layout, a_layout).bytes;
}

extern "C" int64_t b200_gemm_workspace_size(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                                            int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int b_layout) {
  return b200_gemm_workspace_size_ex(A, B, C, M, N, K, lda, ldb, ldc, B200_A_ROW_MAJOR, b_layout);
}

extern "C" int b200_gemm_f16_ex(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                                int64_t ldb, int64_t ldc, int a_layout, int b_layout, float alpha, float beta,
                                void* workspace, int64_t workspace_bytes, void* stream_ptr) {
  using namespace b200;
  bool done = false;
  if (int rc = validate_args(C, M, N, K, lda, ldb, ldc, b_layout, A, B, &done, a_layout)) return rc;
  if (done) return B200_OK;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (!dev.sm100) return B200_ERR_UNSUPPORTED_DEVICE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const EpiParams scale{alpha, beta};
  const RepackPlan p = plan_repack(A, B, C, M, N, K, lda, ldb, ldc, b_layout, a_layout);
  if (p.bytes == 0) return gemm_aligned(A, B, C, M, N, K, lda, ldb, ldc, a_layout, b_layout, scale, dev, stream);
  if (!workspace || workspace_bytes < p.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return B200_ERR_WORKSPACE;
  return gemm_repacked(A, B, C, M, N, K, lda, ldb, ldc, a_layout, b_layout, scale, p,
                       static_cast<uint8_t*>(workspace), dev, stream);
}

extern "C" int b200_gemm_f16_ws(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                                int64_t ldb, int64_t ldc, int b_layout, void* workspace, int64_t workspace_bytes,
                                void* stream_ptr) {
  return b200_gemm_f16_ex(A, B, C, M, N, K, lda, ldb, ldc, B200_A_ROW_MAJOR, b_layout, 1.0f, 0.0f, workspace,
                          workspace_bytes, stream_ptr);
}

extern "C" int b200_gemm_set_variant(int variant) {
  if (variant < B200_VARIANT_AUTO || variant > B200_VARIANT_PAIR_WIDE_192) return B200_ERR_INVALID_ARGUMENT;
  b200::g_variant = variant;
  return B200_OK;
}

extern "C" int b200_gemm_plan(int64_t M, int64_t N, int64_t K, int sm_count, int* variant, int* k_ranges) {
  using namespace b200;
  if (M <= 0 || N <= 0 || K <= 0 || sm_count < 2 || !variant || !k_ranges) return B200_ERR_INVALID_ARGUMENT;
  if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return B200_ERR_TOO_LARGE;
  const int m = (int)M, n = (int)N, k = (int)K;
  int v = g_variant != B200_VARIANT_AUTO ? g_variant : auto_variant(m, n, k, sm_count);
  if (v == B200_VARIANT_SKINNY && (k > 256 || (n + 255) / 256 > sm_count)) v = B200_VARIANT_CTA1;
  int ranges = 1;
  if (v == B200_VARIANT_PAIR) {
    const long long tiles = (long long)((m + 255) / 256) * ((n + 255) / 256);
    ranges = split_ranges_for(tiles, (int)std::min<long long>(tiles, sm_count / 2), (k + 127) / 128);
  }
  *variant = v;
  *k_ranges = ranges;
  return B200_OK;
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
    case B200_ERR_WORKSPACE: return "workspace missing, too small, or not 256-byte aligned (see b200_gemm_workspace_size)";
    case B200_ERR_SCRATCH_LIMIT: return "operands need more re-pitch scratch than the 32 MiB built into b200_gemm_f16_noalloc";
    default: return "unknown error code";
  }
}

extern "C" int b200_gemm_last_device_error(void) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, b200::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  if (v != 0 && cudaMemcpyToSymbol(b200::g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) b200::reset_split_counters();  // an aborted launch may have left tail counters counting
  return v;
}

extern "C" int b200_gemm_sm_count(void) {
  b200::DeviceInfo d;
  if (b200::current_device_info(d)) return 0;
  return d.sm_count;
}

extern "C" int b200_gemm_version(void) { return 101; }

#ifdef B200_GEMM_PROFILE
// Copies and clears the per-CTA split-tail step timestamps (profiling builds only).
extern "C" __attribute__((visibility("default"))) int b200_gemm_debug_read_split_profile(unsigned long long* host,
                                                                                       int rows) {
  if (rows > 1024) rows = 1024;
  if (cudaMemcpyFromSymbol(host, b200::g_split_prof, sizeof(unsigned long long) * 8 * rows) != cudaSuccess) return -1;
  static unsigned long long zero[1024][8];
  return cudaMemcpyToSymbol(b200::g_split_prof, zero, sizeof(zero)) == cudaSuccess ? 0 : -1;
}

// Copies and clears the per-CTA wait counters (profiling builds only).
extern "C" __attribute__((visibility("default"))) int b200_gemm_debug_read_profile(unsigned long long* host, int rows) {
  if (rows > 1024) rows = 1024;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(host, b200::g_prof, sizeof(unsigned long long) * 8 * rows) != cudaSuccess) return -1;
  static unsigned long long zeros[1024][8];
  return cudaMemcpyToSymbol(b200::g_prof, zeros, sizeof(zeros)) == cudaSuccess ? 0 : -1;
}
#endif

extern "C" int b200_gemm_selftest_bounded_wait(int64_t limit_ns) {
  if (limit_ns <= 0 || limit_ns > 1000000000LL) return -B200_ERR_INVALID_ARGUMENT;
  const int before = b200_gemm_last_device_error();  // clears any earlier word
  if (before < 0) return -B200_ERR_CUDA;
  b200::bounded_wait_selftest_kernel<<<1, 32>>>(static_cast<uint64_t>(limit_ns));
  if (cudaGetLastError() != cudaSuccess) return -B200_ERR_CUDA;
  const int word = b200_gemm_last_device_error();
  return word < 0 ? -B200_ERR_CUDA : word;
}

extern "C" int b200_gemm_selftest_split_fixup(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                              int64_t limit_ns, void* stream_ptr) {
  using namespace b200;
  if (limit_ns <= 0 || limit_ns > 1000000000LL) return -B200_ERR_INVALID_ARGUMENT;
  bool done = false;
  if (int rc = validate_args(C, M, N, K, K, N, N, B200_B_ROW_MAJOR, A, B, &done)) return -rc;
  if (done || K == 0) return -B200_ERR_INVALID_ARGUMENT;
  if (!pitch_ok(A, K) || !pitch_ok(B, N) || !pitch_ok(C, N)) return -B200_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return -rc;
  if (!dev.sm100) return -B200_ERR_UNSUPPORTED_DEVICE;
  const long long tiles = ((M + 255) / 256) * ((N + 255) / 256);
  if (split_ranges_for(tiles, (int)std::min<long long>(tiles, dev.sm_count / 2), (int)((K + 127) / 128)) < 2)
    return -B200_ERR_INVALID_ARGUMENT;  // this shape's pair launch has no split last wave
  const int before = b200_gemm_last_device_error();  // clears any earlier word
  if (before < 0) return -B200_ERR_CUDA;
  CallOptions opts;
  opts.withhold_fixup_ns = static_cast<uint64_t>(limit_ns);
  opts.force_variant = B200_VARIANT_PAIR;
  int rc;
  {
    const ScopedCallOptions scoped(opts);
    rc = gemm_aligned(A, B, C, M, N, K, K, N, N, B200_A_ROW_MAJOR, B200_B_ROW_MAJOR, EpiParams{}, dev,
                      static_cast<cudaStream_t>(stream_ptr));
  }
  if (rc) return -rc;
  const int word = b200_gemm_last_device_error();  // synchronises, clears the word, resets the tail counters
  return word < 0 ? -B200_ERR_CUDA : word;
}

// ===========================================================================
// Allocation-free entry point (b200_gemm_f16_noalloc)
//
// Same product as b200_gemm_f16_ws, for callers that may not allocate device
// memory at all: the re-pitch copies live in one fixed scratch array compiled
// into this library.  Every GPU that loads the library holds the array
// (kNoAllocScratchBytes) until the process exits.
// ===========================================================================
namespace b200 {

constexpr int64_t kNoAllocScratchBytes = 32ll << 20;  // 32 MiB

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[kMaxDevices] = {};

// The array's name is only a host-side handle; the device address comes from
// cudaGetSymbolAddress, asked once per device with that device current.
int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B200_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return B200_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return B200_OK;
}

}  // namespace
}  // namespace b200

extern "C" int b200_gemm_f16_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                     int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* stream_ptr) {
  using namespace b200;
  bool done = false;
  if (int rc = validate_args(C, M, N, K, lda, ldb, ldc, b_layout, A, B, &done)) return rc;
  if (done) return B200_OK;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (!dev.sm100) return B200_ERR_UNSUPPORTED_DEVICE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  // The split last wave of the pair kernel keeps its parts in a per-stream
  // workspace that is allocated on first use; this entry runs every tile whole.
  CallOptions opts;
  opts.no_split = true;
  const ScopedCallOptions scoped(opts);
  const RepackPlan p = plan_repack(A, B, C, M, N, K, lda, ldb, ldc, b_layout);
  if (p.bytes == 0)
    return gemm_aligned(A, B, C, M, N, K, lda, ldb, ldc, B200_A_ROW_MAJOR, b_layout, EpiParams{}, dev, stream);
  if (p.bytes > kNoAllocScratchBytes) return B200_ERR_SCRATCH_LIMIT;
  uint8_t* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // Nothing in the scratch has to start at zero: the call writes every byte it
  // later reads (the re-pitched operand rows, and all of C's copy) first.
  return gemm_repacked(A, B, C, M, N, K, lda, ldb, ldc, B200_A_ROW_MAJOR, b_layout, EpiParams{}, p, scratch, dev,
                       stream);
}

// ===========================================================================
// K-means assignment (b200_kmeans_assign_f16)
// ===========================================================================
namespace b200 {
namespace {

// ||c_j||^2 in fp32 for each centroid j (column j of a row-major K x N matrix,
// or row j of an N x K one).
__global__ void centroid_norms_kernel(const __half* Cent, int64_t ld, int N, int K, int row_major_kn, float* out) {
  if (row_major_kn) {
    // Column j of K x N: consecutive threads read consecutive columns.
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= N) return;
    float s = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float v = __half2float(Cent[(int64_t)k * ld + j]);
      s = fmaf(v, v, s);
    }
    out[j] = s;
  } else {
    // Row j of N x K: one warp per centroid, lanes stride along the row.
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (j >= N) return;
    float s = 0.0f;
    for (int k = lane; k < K; k += 32) {
      const float v = __half2float(Cent[(int64_t)j * ld + k]);
      s = fmaf(v, v, s);
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[j] = s;
  }
}

__global__ void unpack_keys_kernel(const unsigned long long* keys, int M, int* idx, float* score) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M) return;
  const unsigned long long k = keys[i];
  idx[i] = (int)(k & 0xffffffffu);
  if (score) score[i] = ordered_to_float((uint32_t)(k >> 32));
}

int64_t kmeans_ws_parts(int64_t M, int64_t N, int64_t* keys_off) {
  *keys_off = round_up(N * 4, 256);
  return *keys_off + round_up(M * 8, 256);
}

}  // namespace
}  // namespace b200

extern "C" int64_t b200_kmeans_workspace_size(int64_t M, int64_t N) {
  if (M < 0 || N < 0) return -B200_ERR_INVALID_ARGUMENT;
  int64_t off = 0;
  return b200::kmeans_ws_parts(M, N, &off);
}

extern "C" int b200_kmeans_assign_f16(const void* X, const void* Cent, int64_t M, int64_t N, int64_t K, int64_t ldx,
                                      int64_t ldcent, int cent_layout, void* workspace, int64_t workspace_bytes,
                                      int32_t* out_idx, float* out_score, void* stream_ptr) {
  using namespace b200;
  if (M < 0 || N <= 0 || K <= 0 || K > 256) return K > 256 ? B200_ERR_TOO_LARGE : B200_ERR_INVALID_ARGUMENT;
  if (cent_layout != B200_B_ROW_MAJOR && cent_layout != B200_B_COL_MAJOR) return B200_ERR_INVALID_ARGUMENT;
  if (M > 0x7fffffff || N > 0x7fffffff) return B200_ERR_TOO_LARGE;
  if (M == 0) return B200_OK;
  const bool row_b = (cent_layout == B200_B_ROW_MAJOR);
  if (!X || !Cent || !out_idx || ldx < K || ldcent < (row_b ? N : K)) return B200_ERR_INVALID_ARGUMENT;
  if (!pitch_ok(X, ldx) || !pitch_ok(Cent, ldcent)) return B200_ERR_MISALIGNED;
  int64_t keys_off = 0;
  const int64_t need = kmeans_ws_parts(M, N, &keys_off);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return B200_ERR_WORKSPACE;
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (!dev.sm100) return B200_ERR_UNSUPPORTED_DEVICE;
  if ((N + 255) / 256 > dev.sm_count) return B200_ERR_TOO_LARGE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  float* cnorm = static_cast<float*>(workspace);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + keys_off);
  const unsigned norm_blocks = row_b ? (unsigned)((N + 127) / 128) : (unsigned)((N * 32 + 127) / 128);
  centroid_norms_kernel<<<norm_blocks, 128, 0, stream>>>(static_cast<const __half*>(Cent), ldcent, (int)N, (int)K,
                                                          row_b ? 1 : 0, cnorm);
  if (cudaGetLastError() != cudaSuccess) return B200_ERR_CUDA;
  if (cudaMemsetAsync(keys, 0xff, M * 8, stream) != cudaSuccess) return B200_ERR_CUDA;
  GemmArgs g{X, Cent, nullptr, (int)M, (int)N, (int)K, ldx, ldcent, 0, EpiParams{}, dev.sm_count, stream};
  g.argmin.cnorm = cnorm;
  g.argmin.keys = keys;
  // The argmin epilogue stages no C, so its staging space is a sixth A stage
  // (measured ~1 % faster than five at 262144 x 1024 x 256).
  // 16 epilogue warps for K <= 128, 8 above (B200_GEMM_KM16=0/1 forces one; tuning only).
  static const int km16_env = [] { const char* e = std::getenv("B200_GEMM_KM16"); return e ? std::atoi(e) : -1; }();
  const bool km16 = km16_env >= 0 ? km16_env == 1 : K <= 128;
  const int rc = km16 ? (row_b ? launch_skinny<6, 0, true, false, true, 16>(g) : launch_skinny<6, 0, false, false, true, 16>(g))
                      : (row_b ? launch_skinny<6, 0, true, false, true>(g) : launch_skinny<6, 0, false, false, true>(g));
  if (rc) return rc;
  unpack_keys_kernel<<<(unsigned)((M + 255) / 256), 256, 0, stream>>>(keys, (int)M, out_idx, out_score);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Gathered output (multi-GPU): every rank computes its row shard of C and its
// epilogue writes each finished block both to its own copy of the gathered C
// and, with plain 16-byte stores over NVLink, to every peer's copy, so the
// all-gather of C runs tile by tile under the GEMM instead of after it.  The
// peers' buffers come from this library's IPC helpers (legacy CUDA IPC: one
// cudaMalloc per buffer, no multicast object).  The kernels never wait on a
// peer: completion is the caller's device-side barrier after the launch.
// ---------------------------------------------------------------------------
namespace b200 {

// K == 0 in gathered mode: zero this shard's rows in the local and every peer
// buffer (plain stores, like the epilogue's).
__global__ void zero_rows_kernel(uint16_t* c, const __grid_constant__ EpiParams ep, int64_t rows, int64_t cols) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
    for (int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; col < cols;
         col += (int64_t)gridDim.x * blockDim.x) {
      c[r * ep.ldc + col] = 0;
      for (int p = 0; p < ep.n_peers; ++p) ep.peer[p][r * ep.ldc + col] = 0;
    }
  if (ep.n_peers > 0) __threadfence_system();
}

}  // namespace b200

extern "C" int b200_ipc_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int b200_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  if (bytes <= 0 || !ptr || !handle) return B200_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return B200_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return B200_ERR_CUDA;
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return B200_OK;
}

extern "C" int b200_ipc_free(void* ptr) {
  if (!ptr) return B200_OK;
  return cudaFree(ptr) == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" int b200_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return B200_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return B200_ERR_CUDA;
  *ptr = p;
  return B200_OK;
}

extern "C" int b200_ipc_close(void* ptr) {
  if (!ptr) return B200_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" int b200_gemm_f16_gather(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                    int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* const* peer_c,
                                    int n_peers, void* stream_ptr) {
  using namespace b200;
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && !peer_c)) return B200_ERR_INVALID_ARGUMENT;
  bool done = false;
  if (int rc = validate_args(C, M, N, K, lda, ldb, ldc, b_layout, A, B, &done)) return rc;
  if (done) return B200_OK;
  EpiParams ep;
  ep.n_peers = n_peers;
  ep.m = (int)M;
  ep.n = (int)N;
  ep.ldc = ldc;
  for (int p = 0; p < n_peers; ++p) {
    if (!peer_c[p]) return B200_ERR_INVALID_ARGUMENT;
    if (!aligned16(peer_c[p])) return B200_ERR_MISALIGNED;
    ep.peer[p] = static_cast<uint16_t*>(peer_c[p]);
  }
  DeviceInfo dev;
  if (int rc = current_device_info(dev)) return rc;
  if (!dev.sm100) return B200_ERR_UNSUPPORTED_DEVICE;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (K == 0) {
    const unsigned gx = (unsigned)std::min<int64_t>((N + 255) / 256, 64);
    const unsigned gy = (unsigned)std::min<int64_t>(M, 65535);
    zero_rows_kernel<<<dim3(gx, gy), 256, 0, stream>>>(static_cast<uint16_t*>(C), ep, M, N);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
  }
  // Operands must be TMA-addressable as they are: a re-pitched C would leave
  // the peers' copies unwritten.
  if (plan_repack(A, B, C, M, N, K, lda, ldb, ldc, b_layout, B200_A_ROW_MAJOR).bytes != 0) return B200_ERR_MISALIGNED;
  return gemm_aligned(A, B, C, M, N, K, lda, ldb, ldc, B200_A_ROW_MAJOR, b_layout, ep, dev, stream);
}
