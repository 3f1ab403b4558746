// B-stationary split-N kernel for short reductions (K <= 256), the HBM-bound
// "K-means-like" shapes (M x N x 256 with N <= a few thousand).
//
// With K <= 256 a 256-column slice of B is at most 128 KB, so each persistent
// CTA loads its slice of B ONCE into shared memory and keeps it there, then
// streams 128-row blocks of A through a small ring.  The grid is a multiple
// of the number of N slices and tiles are dealt N-slice-fastest, so a CTA
// keeps the same slice for its whole life.  Per output tile the CTA then
// moves only the A block (16 KB per 64-deep K step, read from HBM once for
// the whole grid thanks to L2) and the C tile (64 KB store), instead of the
// 128 KB of B that the general kernel re-stages per tile.
//
//   warp 0      TMA producer: B slice once, then A blocks into the ring
//   warp 1      TMEM alloc + MMA issue (128 x 256 x 16 per instruction)
//   warps 2..5  epilogue (same TMEM -> fp16 -> swizzled smem -> TMA store
//               path as the 1-CTA kernel), accumulator double-buffered;
//               EPI_BUFS staging buffers per warp (one frees room for a
//               deeper A ring, which matters more: A streams from HBM)
#pragma once

#include "gemm_common.cuh"

namespace b200 {

template <int A_STAGES, int EPI_BUFS, int EPI_W = kEpiWarps>
struct SkinnyConfig {
  static constexpr int kBN = 256;
  static constexpr int kMaxKBlocks = 4;                     // K <= 256
  static constexpr int kABytes = kBM * kBK * 2;             // 16 KB per A stage
  static constexpr int kBBlockBytes = kBN * kBK * 2;        // 32 KB per 64-deep K block of B
  static constexpr int kBBytes = kMaxKBlocks * kBBlockBytes;
  static constexpr int kEpiBytes = EPI_W * EPI_BUFS * kEpiBufBytes;
  static constexpr int kTmemCols = 2 * kBN;
  static constexpr int kNormBytes = kBN * 4;                // argmin mode: the CTA's slice of ||c||^2
  static constexpr int kSmemBytes = kBBytes + A_STAGES * kABytes + kEpiBytes + kNormBytes + 256 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA exceeds 227 KB");
};

// Threads of a skinny launch: two role warps plus the epilogue warps (argmin
// mode: 8, or 16 when EPI_W is 16).
constexpr int skinny_threads(bool argmin, int epi_w) {
  return argmin ? (epi_w == 16 ? 64 + 16 * 32 : 320) : (epi_w == 8 ? 320 : kThreads);
}

template <int A_STAGES, int EPI_BUFS, bool kBRowMajor, bool kAColMajor, bool kArgmin = false, int EPI_W = kEpiWarps>
__global__ void __launch_bounds__(skinny_threads(kArgmin, EPI_W), 1)
    gemm_f16_skinny_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_c, int M, int N, int K,
                           const __grid_constant__ EpiParams sc, const ArgminOut am = ArgminOut{}) {
  using Cfg = SkinnyConfig<A_STAGES, EPI_BUFS, EPI_W>;
  // The epilogue sets the pace of this kernel (per tile it drains 128 x 256
  // fp32 while the MMAs take ~2k cycles), so it may run on 8 warps: two per
  // TMEM lane quadrant, each on half of the columns.  The argmin epilogue
  // runs on 8 warps, or on 16 (four per quadrant, one 64-column chunk each,
  // scored per 32-column half to stay within 112 registers) when its caller
  // asks: measured faster for K <= 128 (65536 x 4096 x 128: 93.5 against
  // 115.0 us), slower for K = 256 (262144 x 1024 x 256: 132.6 against 124.9).
  constexpr int kEpiW = kArgmin ? (EPI_W == 16 ? 16 : 8) : EPI_W;
  static_assert(EPI_W == 4 || EPI_W == 8 || (kArgmin && EPI_W == 16), "4 or 8 epilogue warps (16: argmin only)");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_b = smem;                                   // resident B slice
  uint8_t* smem_a = smem + Cfg::kBBytes;                    // A ring
  uint8_t* smem_epi = smem_a + A_STAGES * Cfg::kABytes;
  float* s_norm = reinterpret_cast<float*>(smem_epi + Cfg::kEpiBytes);   // [kBN], argmin mode
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + Cfg::kEpiBytes + Cfg::kNormBytes);
  uint64_t* full_bar = bars;                                // [A_STAGES]
  uint64_t* empty_bar = bars + A_STAGES;                    // [A_STAGES]
  uint64_t* tmem_full = bars + 2 * A_STAGES;                // [2]
  uint64_t* tmem_empty = bars + 2 * A_STAGES + 2;           // [2]
  uint64_t* b_full = bars + 2 * A_STAGES + 4;               // [4] B slice, one per 64-deep K block
  uint64_t* mma_drain = bars + 2 * A_STAGES + 8;            // [1] abort path only
  uint64_t* c_bar = bars + 2 * A_STAGES + 9;                // [8] old-C loads of the epilogue warps (beta != 0)
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * A_STAGES + 17);

  B200_PROF_DECL
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_nb = (N + Cfg::kBN - 1) / Cfg::kBN;
  const int num_mb = (M + kBM - 1) / kBM;
  const int num_tiles = num_mb * num_nb;
  const int num_kb = (K + kBK - 1) / kBK;                   // 1..4
  // gridDim.x is a multiple of num_nb: this CTA's N slice never changes.
  const int my_nb = blockIdx.x % num_nb;
  const int n0 = my_nb * Cfg::kBN;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_c);
    for (int s = 0; s < A_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], kEpiW);
    }
    for (int kb = 0; kb < Cfg::kMaxKBlocks; ++kb) mbar_init(&b_full[kb], 1);
    mbar_init(mma_drain, 1);
    for (int e = 0; e < (kEpiW < 8 ? kEpiW : 8); ++e) mbar_init(&c_bar[e], 1);  // [8] slots; argmin uses none
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
  // Setup above overlaps the previous kernel on the stream; nothing below
  // touches global memory before that kernel's results are visible.
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_first();   // A is read once per N slice, then dead
      const uint64_t pol_b = policy_evict_last();
      // B slice: num_kb blocks of 64 K x 256 N, loaded once; one barrier per
      // block so the first MMAs start as soon as the first block lands.
      for (int kb = 0; kb < num_kb; ++kb) {
        uint8_t* dst = smem_b + kb * Cfg::kBBlockBytes;
        mbar_arrive_expect_tx(&b_full[kb], Cfg::kBBlockBytes);
        if constexpr (kBRowMajor) {
#pragma unroll
          for (int p = 0; p < Cfg::kBN / 64; ++p)
            tma_load_2d(dst + p * (kBK * 128), &tmap_b, &b_full[kb], n0 + 64 * p, kb * kBK, pol_b);
        } else {
          tma_load_2d(dst, &tmap_b, &b_full[kb], kb * kBK, n0, pol_b);
        }
      }
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = (t / num_nb) * kBM;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!B200_TIMED(0, mbar_wait(&empty_bar[stage], phase ^ 1u, kDevTimeoutProducer))) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kABytes);
          if constexpr (kAColMajor) {
#pragma unroll
            for (int p = 0; p < kBM / 64; ++p)
              tma_load_2d(smem_a + stage * Cfg::kABytes + p * (kBK * 128), &tmap_a, &full_bar[stage], m0 + 64 * p,
                          kb * kBK, pol_a);
          } else {
            tma_load_2d(smem_a + stage * Cfg::kABytes, &tmap_a, &full_bar[stage], kb * kBK, m0, pol_a);
          }
          ++issued;
          if (++stage == A_STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        const uint32_t pending = issued < (uint32_t)A_STAGES ? issued : (uint32_t)A_STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (uint32_t i = 0; i < pending; ++i) {
          if (--s < 0) { s = A_STAGES - 1; ph ^= 1u; }
          mbar_wait_drain(&full_bar[s], ph);
        }
        for (int kb = 0; kb < num_kb; ++kb) mbar_wait_drain(&b_full[kb], 0);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc =
          make_idesc_f16_f32(kBM, Cfg::kBN, kAColMajor ? Major::kMN : Major::kK, kBRowMajor ? Major::kMN : Major::kK);
      const uint32_t a_base = smem_u32(smem_a);
      const uint32_t b_base = smem_u32(smem_b);
      int stage = 0;
      uint32_t phase = 0;
#ifdef B200_GEMM_PROFILE
      const long long prof_t0 = clock64();
#endif
      bool ok = true;
      bool b_ready = false;  // B blocks are waited for during the first tile only
      bool any_mma = false;
      int local = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!B200_TIMED(1, mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, kDevTimeoutMma))) { ok = false; break; }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kBN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!b_ready && !B200_TIMED(2, mbar_wait(&b_full[kb], 0, kDevTimeoutMma))) { ok = false; break; }
          if (!B200_TIMED(2, mbar_wait(&full_bar[stage], phase, kDevTimeoutMma))) { ok = false; break; }
          tc_fence_after_sync();
          const uint32_t a_addr = a_base + stage * Cfg::kABytes;
          const uint32_t b_addr = b_base + kb * Cfg::kBBlockBytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t adesc = kAColMajor ? make_desc_mnmajor_sw128(a_addr + k * (kUmmaK * 128), kBK * 128)
                                              : make_desc_kmajor_sw128(a_addr + k * (kUmmaK * 2));
            uint64_t bdesc;
            if constexpr (kBRowMajor)
              bdesc = make_desc_mnmajor_sw128(b_addr + k * (kUmmaK * 128), kBK * 128);
            else
              bdesc = make_desc_kmajor_sw128(b_addr + k * (kUmmaK * 2));
            umma_f16_cta1(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          any_mma = true;
          umma_commit_cta1(&empty_bar[stage]);
          if (++stage == A_STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        b_ready = true;
        umma_commit_cta1(&tmem_full[acc]);
      }
      B200_PROF_ADD(4, clock64() - prof_t0);
      if (!ok && any_mma) {
        umma_commit_cta1(mma_drain);
        mbar_wait_drain(mma_drain, 0);
      }
    }
  } else {
    // ---------------- epilogue warps 2 .. 1 + kEpiW ----------------
    const int quad = warp & 3;
    const int ew = warp - 2;
    constexpr int kChunksPerWarp = (Cfg::kBN / kEpiCols) * kEpiWarps / kEpiW;
    const int c_begin = (ew / kEpiWarps) * kChunksPerWarp;
    const int c_end = c_begin + kChunksPerWarp;
    uint8_t* epi_buf = smem_epi + ew * EPI_BUFS * kEpiBufBytes;
    const uint32_t epi_addr = smem_u32(epi_buf);
    int buf = 0;
    uint32_t c_phase = 0;
    int local = 0;
    if constexpr (kArgmin) {
      // This CTA's N slice never changes: stage its norms once (+inf past N,
      // so those columns never win), then sync the four epilogue warps.
      for (int j = threadIdx.x - 64; j < Cfg::kBN; j += kEpiW * 32)
        s_norm[j] = (n0 + j < N) ? am.cnorm[n0 + j] : __int_as_float(0x7f800000);
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiW * 32) : "memory");
    }
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int m0 = (t / num_nb) * kBM;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      bool got = true;
      if (lane == 0) got = B200_TIMED(3, mbar_wait(&tmem_full[acc], acc_phase, kDevTimeoutEpilogue));
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after_sync();
#ifdef B200_GEMM_PROFILE
      const long long prof_e0 = clock64();
#endif
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * Cfg::kBN;
      float best_d = __int_as_float(0x7f800000);  // +inf
      int best_i = 0x7fffffff;
#pragma unroll 1
      for (int c = c_begin; c < c_end; ++c) {
        if constexpr (kArgmin && kEpiW == 16) {
          // Per 32-column half: its scores, their minimum (a tree of
          // three-input mins), then the first column reaching it; a later
          // half or chunk replaces the best only when strictly smaller, so
          // ties go to the smallest index.
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32 * h, r);
            tmem_ld_wait_regs(r);
            if (h == 1 && c == c_end - 1) {
              tc_fence_before_sync();
              __syncwarp();
              if (lane == 0) mbar_arrive(&tmem_empty[acc]);
            }
            float d[32];
            const float4* nrm = reinterpret_cast<const float4*>(s_norm + c * kEpiCols + 32 * h);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 v = nrm[q];
              fma2f(d[4 * q], d[4 * q + 1], -2.0f, -2.0f, __uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                    v.x, v.y);
              fma2f(d[4 * q + 2], d[4 * q + 3], -2.0f, -2.0f, __uint_as_float(r[4 * q + 2]),
                    __uint_as_float(r[4 * q + 3]), v.z, v.w);
            }
            float t1[11], t2[4];
#pragma unroll
            for (int i = 0; i < 10; ++i) t1[i] = min3f(d[3 * i], d[3 * i + 1], d[3 * i + 2]);
            t1[10] = fminf(d[30], d[31]);
#pragma unroll
            for (int i = 0; i < 3; ++i) t2[i] = min3f(t1[3 * i], t1[3 * i + 1], t1[3 * i + 2]);
            t2[3] = fminf(t1[9], t1[10]);
            const float m = fminf(min3f(t2[0], t2[1], t2[2]), t2[3]);
            if (m < best_d) {
              int first = 31;
#pragma unroll
              for (int e = 31; e >= 0; --e)
                if (d[e] == m) first = e;
              best_d = m;
              best_i = n0 + c * kEpiCols + 32 * h + first;
            }
          }
          continue;
        }
        uint32_t lo[32], hi[32];
#ifdef B200_GEMM_PROFILE
        const long long prof_l0 = clock64();
#endif
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, lo);
        tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, hi);
        tmem_ld_wait_regs(lo);
        tmem_ld_wait_regs(hi);
        B200_PROF_ADD(6, clock64() - prof_l0);
        if (c == c_end - 1) {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[acc]);
        }
        if constexpr (kArgmin) {
          // Scores of this 64-column chunk, their minimum, then the first
          // column reaching it (smallest index on ties).
          float d[kEpiCols];
          const float4* nrm = reinterpret_cast<const float4*>(s_norm + c * kEpiCols);
#pragma unroll
          for (int q = 0; q < kEpiCols / 4; ++q) {
            const float4 v = nrm[q];
            const float nv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int t = 0; t < 4; t += 2) {
              const int e = 4 * q + t;
              fma2f(d[e], d[e + 1], -2.0f, -2.0f, __uint_as_float(e < 32 ? lo[e] : hi[e - 32]),
                    __uint_as_float(e + 1 < 32 ? lo[e + 1] : hi[e + 1 - 32]), nv[t], nv[t + 1]);
            }
          }
          // Minimum by a tree of three-input mins (31 instructions, depth 4).
          static_assert(kEpiCols == 64, "the min tree is laid out for 64 columns");
          float t1[22], t2[8];
#pragma unroll
          for (int i = 0; i < 21; ++i) t1[i] = min3f(d[3 * i], d[3 * i + 1], d[3 * i + 2]);
          t1[21] = d[63];
#pragma unroll
          for (int i = 0; i < 7; ++i) t2[i] = min3f(t1[3 * i], t1[3 * i + 1], t1[3 * i + 2]);
          t2[7] = t1[21];
          const float m = min3f(min3f(t2[0], t2[1], t2[2]), min3f(t2[3], t2[4], t2[5]), fminf(t2[6], t2[7]));
          if (m < best_d) {
            int first = kEpiCols - 1;
#pragma unroll
            for (int e = kEpiCols - 1; e >= 0; --e)
              if (d[e] == m) first = e;
            best_d = m;
            best_i = n0 + c * kEpiCols + first;
          }
          continue;
        }
        if constexpr (!kArgmin)
          epi_store_block<EPI_BUFS>(&tmap_c, epi_buf, epi_addr, buf, lane, lo, hi, n0 + c * kEpiCols, m0 + quad * 32,
                                  sc, &c_bar[ew], c_phase);
      }
      if constexpr (kArgmin) {
        const int row = m0 + quad * 32 + lane;
        if (row < M && best_i != 0x7fffffff)
          atomicMin(am.keys + row, ((unsigned long long)float_to_ordered(best_d) << 32) | (unsigned)best_i);
      }
      B200_PROF_ADD(5, clock64() - prof_e0);
      B200_PROF_ADD(7, 1);
    }
    epi_peer_fence(sc);
    if (lane == 0) bulk_wait_group<0>();
  }

  B200_PROF_FLUSH
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc<1>(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace b200
