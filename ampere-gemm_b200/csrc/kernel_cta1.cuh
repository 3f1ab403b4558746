// 1-CTA tcgen05 GEMM kernel: 128 x BN output tiles, one persistent CTA per SM.
#pragma once

#include "gemm_common.cuh"

namespace b200 {

template <int BN, int STAGES, bool kBRowMajor, bool kAColMajor>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_f16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                            const __grid_constant__ CUtensorMap tmap_c, int M, int N, int K, int group_m,
                            const __grid_constant__ EpiParams sc) {
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
  uint64_t* c_bar = bars + 2 * STAGES + 5;      // [4]       old-C loads of the epilogue warps (beta != 0)
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 9);

  B200_PROF_DECL
#ifdef B200_GEMM_PROFILE
  // Timeline of one launch (profile build): entry time, then per role the
  // nanoseconds from entry to the first data / the end of the epilogue.
  const uint64_t prof_entry = global_timer_ns();
  bool prof_first = true;
#endif
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
    for (int e = 0; e < kEpiWarps; ++e) mbar_init(&c_bar[e], 1);
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
    // ---------------- TMA producer (one lane) ----------------
    if (lane == 0) {
      // Measured (ncu DRAM bytes, 8192^3): A evict_normal + B evict_last reads
      // the least; the reverse hints read 30-60 % more.
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
          if (!B200_TIMED(0, mbar_wait(&empty_bar[stage], phase ^ 1u, kDevTimeoutProducer))) { ok = false; break; }
#ifdef B200_GEMM_NOLOAD
          mbar_arrive(&full_bar[stage]);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          continue;
#endif
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
          const int k0 = kb * kBK;
          if constexpr (kAColMajor) {
            // A stored K x M (M contiguous): two panels of 64 rows x 64 K.
#pragma unroll
            for (int p = 0; p < kBM / 64; ++p)
              tma_load_2d(smem_a + stage * Cfg::kABytes + p * (kBK * 128), &tmap_a, &full_bar[stage], m0 + 64 * p, k0,
                          pol_a);
          } else {
            tma_load_2d(smem_a + stage * Cfg::kABytes, &tmap_a, &full_bar[stage], k0, m0, pol_a);
          }
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
          make_idesc_f16_f32(kBM, BN, kAColMajor ? Major::kMN : Major::kK, kBRowMajor ? Major::kMN : Major::kK);
      const uint32_t a_base = smem_u32(smem_a);
      const uint32_t b_base = smem_u32(smem_b);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool any_mma = false;
      int local = 0;
#ifdef B200_GEMM_PROFILE
      const long long prof_t0 = clock64();
#endif
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!B200_TIMED(1, mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, kDevTimeoutMma))) { ok = false; break; }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!B200_TIMED(2, mbar_wait(&full_bar[stage], phase, kDevTimeoutMma))) { ok = false; break; }
#ifdef B200_GEMM_PROFILE
          if (prof_first) { B200_PROF_ADD(6, global_timer_ns() - prof_entry); prof_first = false; }
#endif
          tc_fence_after_sync();
          const uint32_t a_addr = a_base + stage * Cfg::kABytes;
          const uint32_t b_addr = b_base + stage * Cfg::kBBytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t adesc = kAColMajor ? make_desc_mnmajor_sw128(a_addr + k * (kUmmaK * 128), kBK * 128)
                                              : make_desc_kmajor_sw128(a_addr + k * (kUmmaK * 2));
            uint64_t bdesc;
            if constexpr (kBRowMajor)
              bdesc = make_desc_mnmajor_sw128(b_addr + k * (kUmmaK * 128), kBK * 128);
            else
              bdesc = make_desc_kmajor_sw128(b_addr + k * (kUmmaK * 2));
#ifndef B200_GEMM_NOMMA
            umma_f16_cta1(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
#endif
          }
          any_mma = true;
          umma_commit_cta1(&empty_bar[stage]);  // frees the stage once these MMAs have read it
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_cta1(&tmem_full[acc]);       // accumulator ready for the epilogue
      }
      B200_PROF_ADD(4, clock64() - prof_t0);
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
    uint32_t c_phase = 0;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int mb, nb;
      sched.tile_coords(t, mb, nb);
      const int m0 = mb * kBM, n0 = nb * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // One lane per warp polls; the other 31 park at __syncwarp instead of
      // hammering the barrier word in shared memory beside the tensor core.
      bool got = true;
      if (lane == 0) got = B200_TIMED(3, mbar_wait(&tmem_full[acc], acc_phase, kDevTimeoutEpilogue));
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after_sync();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
#ifdef B200_GEMM_NOEPI
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (false) mbar_arrive_cluster(mapa_shared(smem_u32(&tmem_empty[acc]), 0));
        else mbar_arrive(&tmem_empty[acc]);
      }
      continue;
#endif
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
        epi_store_block<2>(&tmap_c, epi_buf, epi_addr, buf, lane, lo, hi, n0 + c * kEpiCols, m0 + quad * 32, sc,
                           &c_bar[ew], c_phase);
      }
    }
    epi_peer_fence(sc);
    if (lane == 0) bulk_wait_group<0>();
#ifdef B200_GEMM_PROFILE
    B200_PROF_ADD(5, prof_entry);
    B200_PROF_ADD(7, global_timer_ns() - prof_entry);
#endif
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
