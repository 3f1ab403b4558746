// 2-CTA (cta_group::2) tcgen05 GEMM kernel: a cluster of two CTAs on two SMs
// computes one (256 * MSUB) x 256 output tile with M=256, N=256 MMAs.
//
//   * CTA r of the pair owns MSUB blocks of 128 A rows,
//     [m0 + 128 * (MSUB * r + s), +128) for s < MSUB, and B columns
//     [n0 + 128 r, +128); it loads them into its own shared memory with plain
//     TMA (no multicast).  The loads of both CTAs complete on the leader's
//     (r = 0) full barrier.
//   * Per 16-deep K step the leader issues MSUB MMAs of tcgen05.mma.cta_group::2:
//     MMA s reads A block s of both CTAs and all 256 staged B columns and
//     writes rows [128 r, +128) of its 256 x 256 fp32 result into CTA r's TMEM
//     columns [256 s, +256).  With MSUB = 2 every staged B column feeds two
//     MMAs, so a pair stages 25 % fewer bytes per FLOP than with MSUB = 1.
//   * The leader frees a stage / publishes an accumulator with one
//     tcgen05.commit per CTA (own barrier, then the peer's through mapa).
//   * Each CTA's epilogue stores its own rows; the peer's epilogue warps
//     release accumulator space with remote arrives on the leader's barriers.
//
// TMEM (512 columns) holds two tiles' accumulators when MSUB = 1 (double
// buffer: the epilogue of tile i overlaps the mainloop of tile i+1) and one
// tile when MSUB = 2; then each 256-column half is released separately, so the
// next tile's MMAs into the first half start while the second half drains.
//
// A stage holds KSUB 64-wide K slices.  Commits of a pair reach their barriers
// late (about 1.6k cycles after issue), so a stage must carry at least 8 MMAs
// (MSUB * KSUB * 4 >= 8) to keep the tensor pipe fed.
#pragma once

#include "gemm_common.cuh"

namespace b200 {

// Split-tail fixup: per epilogue warp, kFixBufs 8 KB buffers (one 32 x 64
// fp32 chunk each) carved from the pipeline stages, which are idle by then.
constexpr int kFixBufs = 6;
constexpr uint32_t kEpiChunkF32Bytes = kEpiRows * kEpiCols * 4;  // 8 KB

// BN: columns per pair tile (256, 224 or 192).  tcgen05.mma's time is
// proportional to N (N / 2 cycles per 128 x N x 16 MMA for N >= 128, measured),
// so a narrower tile costs nothing per FLOP and is picked where it fills the
// waves better (4000 x 6000: 27 column tiles of 224 against 24 of 256).  Each
// CTA stages 128 B columns whatever BN is and its MMAs read the first BN / 2;
// a tile ends in a partial 64-column epilogue block when BN % 64 != 0.
template <int STAGES, int KSUB, int MSUB, int BN = 256>
struct PairConfig {
  static_assert(BN == 256 || BN == 224 || BN == 192, "pair tiles are 256, 224 or 192 columns wide");
  static_assert(BN == 256 || MSUB == 2, "narrow tiles only for the wide pair (no split tail)");
  static constexpr int kStageK = kBK * KSUB;         // K per stage (KSUB swizzle atoms)
  static constexpr int kTileM = 256 * MSUB;          // rows per pair tile
  static constexpr int kTileN = BN;                  // columns per pair tile
  static constexpr int kChunksN = (BN + 63) / 64;    // 64-column epilogue blocks per 256-row block
  static constexpr int kHalfN = 128;                 // B columns staged per CTA (>= BN / 2)
  static constexpr int kAccCols = 256;               // TMEM columns per accumulator block (>= BN)
  static constexpr int kASub = kBM * kBK * 2;        // 16 KB: 128 rows x 64 K of A
  static constexpr int kBSub = kHalfN * kBK * 2;     // 16 KB per 64-wide K slice of B (col-major B)
  static constexpr int kABytes = kASub * KSUB * MSUB;  // A stage: [msub][ksub] blocks
  static constexpr int kBBytes = kBSub * KSUB;
  static constexpr int kBPanel = kStageK * 128;      // row-major B: one 64-column panel of kStageK rows
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBytes = kEpiWarps * 2 * kEpiBufBytes;
  static constexpr int kAccBufs = (MSUB == 1) ? 2 : 1;  // tiles resident in TMEM
  static constexpr int kTmemCols = 512;
  static constexpr int kSmemBytes = STAGES * kStageBytes + kEpiBytes + 512 + 1024;
  static_assert(kAccBufs * MSUB * kAccCols <= kTmemCols, "accumulators exceed TMEM");
  static_assert(MSUB * KSUB * (kBK / kUmmaK) >= 8, "a pair stage needs at least 8 MMAs");
  static_assert(kSmemBytes <= 232448, "shared memory per CTA exceeds 227 KB");
  static_assert(MSUB != 1 || STAGES * kStageBytes >= kEpiWarps * kFixBufs * (int)kEpiChunkF32Bytes,
                "split-tail fixup buffers must fit in the pipeline stages");
};

// kDyn (no split tail): the grid has one cluster per tile; a running pair
// processes its own tile, then takes the tiles of clusters that have not
// started yet by cancelling their launch (cluster launch control), so pairs
// that run ahead take more tiles and the set of tiles in flight stays compact
// in raster order.  The leader's producer fetches each next tile while the
// current one loads and hands it to every role of both CTAs through a
// two-slot queue in shared memory (tile -1 ends the loop).
template <int STAGES, int KSUB, int MSUB, bool kBRowMajor, bool kAColMajor, int BN = 256, bool kDyn = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_f16_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                 const __grid_constant__ CUtensorMap tmap_b,
                                 const __grid_constant__ CUtensorMap tmap_c, int M, int N, int K, int group_m,
                                 const __grid_constant__ EpiParams sc, const __grid_constant__ SplitTail st) {
  using Cfg = PairConfig<STAGES, KSUB, MSUB, BN>;
  constexpr int kAcc = Cfg::kAccBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * Cfg::kABytes;
  uint8_t* smem_epi = smem + STAGES * Cfg::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + Cfg::kEpiBytes);
  uint64_t* full_bar = bars;                          // [STAGES] leader: both CTAs' loads landed
  uint64_t* empty_bar = bars + STAGES;                // [STAGES] each CTA: its stage may be refilled
  uint64_t* tmem_full = bars + 2 * STAGES;            // [kAcc * MSUB] each CTA: one 256-column block final
  uint64_t* tmem_empty = tmem_full + kAcc * MSUB;     // [kAcc * MSUB] leader: one 256-column block drained
  uint64_t* mma_drain = tmem_empty + kAcc * MSUB;     // [1]      abort path only
  uint64_t* c_bar = mma_drain + 1;                    // [4]      old-C loads of the epilogue warps (beta != 0)
  uint64_t* fix_bar = c_bar + kEpiWarps;              // [4 x kFixBufs] split-tail fixup loads, per epilogue warp
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(fix_bar + kEpiWarps * kFixBufs);
  uint32_t* split_last = tmem_base_slot + 1;          // split tail: this CTA's unit arrived last
  uint8_t* bar_bytes = reinterpret_cast<uint8_t*>(bars);
  uint8_t* clc_resp = bar_bytes + 352;                            // 16 B, dynamic tiles only
  uint32_t* tq_tile = reinterpret_cast<uint32_t*>(bar_bytes + 368);  // [2] tile queue slots
  uint64_t* tq_full = reinterpret_cast<uint64_t*>(bar_bytes + 384);  // [2] slot written (each CTA)
  uint64_t* tq_empty = reinterpret_cast<uint64_t*>(bar_bytes + 400); // [2] slot read by all ten readers (leader)
  uint64_t* clc_bar = reinterpret_cast<uint64_t*>(bar_bytes + 416);  // [1] answer of the launch-control request
  static_assert(sizeof(uint64_t) * (2 * STAGES + 2 * kAcc * MSUB + 1 + kEpiWarps + kEpiWarps * kFixBufs) + 8 <= 352,
                "barrier area overlaps the tile queue");

  B200_PROF_DECL
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  TileScheduler sched;
  sched.num_m = (M + Cfg::kTileM - 1) / Cfg::kTileM;
  sched.num_n = (N + Cfg::kTileN - 1) / Cfg::kTileN;
  sched.group_m = group_m;
  const int num_tiles = sched.num_m * sched.num_n;
  const int num_kb = (K + Cfg::kStageK - 1) / Cfg::kStageK;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_c);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < kAcc * MSUB; ++a) mbar_init(&tmem_full[a], 1);
    for (int a = 0; a < kAcc * MSUB; ++a) mbar_init(&tmem_empty[a], 2 * kEpiWarps);
    mbar_init(mma_drain, 1);
    for (int e = 0; e < kEpiWarps; ++e) mbar_init(&c_bar[e], 1);
    for (int e = 0; e < kEpiWarps * kFixBufs; ++e) mbar_init(&fix_bar[e], 1);
    if constexpr (kDyn) {
      for (int q = 0; q < 2; ++q) {
        mbar_init(&tq_full[q], 1);
        mbar_init(&tq_empty[q], 2 + 2 * kEpiWarps);  // leader MMA, peer producer, both CTAs' epilogue warps
      }
      mbar_init(clc_bar, 1);
    }
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc<2>(tmem_base_slot, Cfg::kTmemCols);
    tmem_relinquish_alloc_permit<2>();
  }
  tc_fence_before_sync();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_base_slot;
  // Setup above overlaps the previous kernel on the stream; nothing below
  // touches global memory before that kernel's results are visible.
  griddep_wait();
  griddep_launch_dependents();

  // ---- dynamic tiles: the queue's reader side (any role of either CTA) ----
  // Returns false on a timed-out wait; *tile = -1 means no more tiles.
  auto dyn_pop = [&](int idx, int* tile, int err) -> bool {
    const int q = idx & 1;
    const uint32_t ph = static_cast<uint32_t>(idx >> 1) & 1u;
    if (!mbar_wait_cluster(&tq_full[q], ph, err)) return false;
    *tile = static_cast<int>(*reinterpret_cast<volatile uint32_t*>(&tq_tile[q]));
    if (leader)
      mbar_arrive(&tq_empty[q]);
    else
      mbar_arrive_cluster(mapa_shared(smem_u32(&tq_empty[q]), 0));
    return true;
  };

  if (warp == 0) {
    // ---------------- TMA producer (one lane per CTA) ----------------
    if (lane == 0) {
      // Measured (ncu DRAM bytes, 8192^3): A evict_normal + B evict_last reads
      // the least; the reverse hints read 30-60 % more.
      const uint64_t pol_a = policy_evict_normal();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      WorkUnit u;
      bool clc_more = true, clc_pending = false, dyn_fail = false;
      uint32_t clc_phase = 0;
      // Next unit of this CTA's producer.  Dynamic tiles: the leader takes its
      // own tile first, then the answer to the launch-control request it made
      // when the previous tile started, publishes it to both CTAs' queues, and
      // asks for the following one; the peer's producer reads its queue.
      auto next_unit = [&](int it, WorkUnit& w) -> bool {
        if constexpr (!kDyn) {
          return work_unit(it, pair, num_pairs, num_tiles, num_kb, st, w);
        } else {
          int tile;
          if (leader) {
            if (it == 0) {
              tile = pair;
            } else if (clc_pending) {
              if (!mbar_wait(clc_bar, clc_phase, kDevTimeoutProducer)) { dyn_fail = true; return false; }
              clc_phase ^= 1u;
              clc_pending = false;
              uint32_t x = 0;
              if (clc_decode(clc_resp, &x)) {
                tile = static_cast<int>(x >> 1);
              } else {
                tile = -1;
                clc_more = false;  // no request may follow a refused one
              }
            } else {
              tile = -1;
            }
            const int q = it & 1;
            const uint32_t ph = static_cast<uint32_t>(it >> 1) & 1u;
            if (!mbar_wait(&tq_empty[q], ph ^ 1u, kDevTimeoutProducer)) { dyn_fail = true; return false; }
            tq_tile[q] = static_cast<uint32_t>(tile);
            st_shared_cluster_u32(mapa_shared(smem_u32(&tq_tile[q]), 1), static_cast<uint32_t>(tile));
            mbar_arrive(&tq_full[q]);
            mbar_arrive_cluster(mapa_shared(smem_u32(&tq_full[q]), 1));
            if (tile < 0) return false;
            if (clc_more) {
              fence_proxy_async_smem();  // the previous answer was read before the next one is written
              mbar_arrive_expect_tx(clc_bar, 16);
              clc_try_cancel(clc_resp, clc_bar);
              clc_pending = true;
            }
          } else {
            if (!dyn_pop(it, &tile, kDevTimeoutProducer)) { dyn_fail = true; return false; }
            if (tile < 0) return false;
          }
          w.t = tile;
          w.kb0 = 0;
          w.kb1 = num_kb;
          w.s = -1;
          return true;
        }
      };
      for (int it = 0; ok && next_unit(it, u); ++it) {
        int mb, nb;
        sched.tile_coords(u.t, mb, nb);
        const int m0 = mb * Cfg::kTileM + static_cast<int>(rank) * (kBM * MSUB);
        const int nh0 = nb * Cfg::kTileN + static_cast<int>(rank) * (Cfg::kTileN / 2);
        for (int kb = u.kb0; kb < u.kb1; ++kb) {
          if (!B200_TIMED(0, mbar_wait(&empty_bar[stage], phase ^ 1u, kDevTimeoutProducer))) { ok = false; break; }
#ifdef B200_GEMM_NOLOAD
          if (leader) mbar_arrive(&full_bar[stage]);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          continue;
#endif
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::kStageBytes);
          const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[stage]), 0);
          const int k0 = kb * Cfg::kStageK;
          uint8_t* a_dst = smem_a + stage * Cfg::kABytes;
          uint8_t* b_dst = smem_b + stage * Cfg::kBBytes;
          if constexpr (kAColMajor) {
            // A stored K x M: each 128-row block is two panels of 64 rows x kStageK.
#pragma unroll
            for (int s = 0; s < MSUB; ++s)
#pragma unroll
              for (int p = 0; p < kBM / 64; ++p)
                tma_load_2d_pair(a_dst + s * (Cfg::kASub * KSUB) + p * Cfg::kBPanel, &tmap_a, full_leader,
                                 m0 + kBM * s + 64 * p, k0, pol_a);
          } else {
#pragma unroll
            for (int s = 0; s < MSUB; ++s)
#pragma unroll
              for (int sub = 0; sub < KSUB; ++sub)
                tma_load_2d_pair(a_dst + (s * KSUB + sub) * Cfg::kASub, &tmap_a, full_leader, k0 + kBK * sub,
                                 m0 + kBM * s, pol_a);
          }
          if constexpr (kBRowMajor) {
            // Panels of 64 columns x kStageK rows (one box each).
#pragma unroll
            for (int p = 0; p < Cfg::kHalfN / 64; ++p)
              tma_load_2d_pair(b_dst + p * Cfg::kBPanel, &tmap_b, full_leader, nh0 + 64 * p, k0, pol_b);
          } else {
#pragma unroll
            for (int sub = 0; sub < KSUB; ++sub)
              tma_load_2d_pair(b_dst + sub * Cfg::kBSub, &tmap_b, full_leader, k0 + kBK * sub, nh0, pol_b);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (dyn_fail) ok = false;
      if (clc_pending) mbar_wait_drain(clc_bar, clc_phase);  // no request may be in flight at exit
      if (!ok && leader) {
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
    // ---------------- MMA issuer (leader CTA, one lane) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16_f32(256, Cfg::kTileN, kAColMajor ? Major::kMN : Major::kK,
                                                    kBRowMajor ? Major::kMN : Major::kK);
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
      WorkUnit u;
      auto next_unit = [&](int it, WorkUnit& w) -> bool {
        if constexpr (!kDyn) {
          return work_unit(it, pair, num_pairs, num_tiles, num_kb, st, w);
        } else {
          int tile = -1;
          if (!dyn_pop(it, &tile, kDevTimeoutMma)) { ok = false; return false; }
          if (tile < 0) return false;
          w.t = tile;
          w.kb0 = 0;
          w.kb1 = num_kb;
          w.s = -1;
          return true;
        }
      };
      for (int it = 0; ok && next_unit(it, u); ++it, ++local) {
        const int buf = local % kAcc;
        const uint32_t acc_phase = (local / kAcc) & 1;
        // The MMAs of one K step: 256-column block s of this tile's accumulator.
        auto issue_block = [&](int stg, int kb, int s) {
          const uint32_t a_addr = a_base + stg * Cfg::kABytes;
          const uint32_t b_addr = b_base + stg * Cfg::kBBytes;
#pragma unroll
          for (int k = 0; k < Cfg::kStageK / kUmmaK; ++k) {
            const int sub = k / (kBK / kUmmaK), j = k % (kBK / kUmmaK);
            uint64_t bdesc;
            if constexpr (kBRowMajor)
              bdesc = make_desc_mnmajor_sw128(b_addr + k * (kUmmaK * 128), Cfg::kBPanel);
            else
              bdesc = make_desc_kmajor_sw128(b_addr + sub * Cfg::kBSub + j * (kUmmaK * 2));
            const uint64_t adesc =
                kAColMajor ? make_desc_mnmajor_sw128(a_addr + s * (Cfg::kASub * KSUB) + k * (kUmmaK * 128), Cfg::kBPanel)
                           : make_desc_kmajor_sw128(a_addr + (s * KSUB + sub) * Cfg::kASub + j * (kUmmaK * 2));
            const uint32_t d_tmem = tmem_base + (buf * MSUB + s) * Cfg::kAccCols;
#ifndef B200_GEMM_NOMMA
            umma_f16_cta2(d_tmem, adesc, bdesc, idesc, (kb != u.kb0 || k != 0) ? 1u : 0u);
#endif
          }
          any_mma = true;
        };
        int kb_first = u.kb0;
        if constexpr (MSUB == 2) {
          // Tile start: the previous tile's two 256-column blocks are drained
          // one after the other.  Run the first P stages into block 0 alone
          // (they stay resident), then, once block 1 is free, the same stages
          // into block 1, and release them: the tensor pipe works while
          // block 1 drains instead of waiting for both.
          const int P = (u.kb1 - u.kb0) < STAGES ? (u.kb1 - u.kb0) : STAGES;
          if (!B200_TIMED(1, mbar_wait_cluster(&tmem_empty[buf * MSUB + 0], acc_phase ^ 1u, kDevTimeoutMma))) {
            ok = false;
          }
          tc_fence_after_sync();
          int stg = stage;
          uint32_t ph = phase;
          for (int j = 0; j < P && ok; ++j) {
            if (!B200_TIMED(2, mbar_wait(&full_bar[stg], ph, kDevTimeoutMma))) { ok = false; break; }
            tc_fence_after_sync();
            issue_block(stg, u.kb0 + j, 0);
            if (++stg == STAGES) { stg = 0; ph ^= 1u; }
          }
          if (ok && P == u.kb1 - u.kb0) {
            // The whole tile fit these stages: block 0 is final already.
            const uint32_t f0 = smem_u32(&tmem_full[buf * MSUB + 0]);
            umma_commit_cta2(f0);
            umma_commit_cta2(mapa_shared(f0, 1));
          }
          if (ok && !B200_TIMED(1, mbar_wait_cluster(&tmem_empty[buf * MSUB + 1], acc_phase ^ 1u, kDevTimeoutMma)))
            ok = false;
          if (!ok) break;
          tc_fence_after_sync();
          for (int j = 0; j < P; ++j) {
            issue_block(stage, u.kb0 + j, 1);
            const uint32_t e = smem_u32(&empty_bar[stage]);
            umma_commit_cta2(e);
            umma_commit_cta2(mapa_shared(e, 1));
            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          }
          kb_first = u.kb0 + P;
        }
        // Tile end (MSUB = 2): the last P_end stages run into block 0 first,
        // which is then published, and only then into block 1, so block 0
        // drains while block 1's last MMAs run.
        const int rest = u.kb1 - kb_first;
        const int P_end = (MSUB == 2) ? (rest < STAGES ? rest : STAGES) : 0;
        const int kb_end = u.kb1 - P_end;
        for (int kb = kb_first; kb < kb_end && ok; ++kb) {
          if (!B200_TIMED(2, mbar_wait(&full_bar[stage], phase, kDevTimeoutMma))) { ok = false; break; }
          tc_fence_after_sync();
          const uint32_t a_addr = a_base + stage * Cfg::kABytes;
          const uint32_t b_addr = b_base + stage * Cfg::kBBytes;
#pragma unroll
          for (int k = 0; k < Cfg::kStageK / kUmmaK; ++k) {
            const int sub = k / (kBK / kUmmaK), j = k % (kBK / kUmmaK);
            uint64_t bdesc;
            if constexpr (kBRowMajor)
              bdesc = make_desc_mnmajor_sw128(b_addr + k * (kUmmaK * 128), Cfg::kBPanel);
            else
              bdesc = make_desc_kmajor_sw128(b_addr + sub * Cfg::kBSub + j * (kUmmaK * 2));
#pragma unroll
            for (int s = 0; s < MSUB; ++s) {
              if (MSUB == 1 && kb == u.kb0 && k == 0) {
                // First write of this 256-column block in the tile: the
                // epilogue must have drained it (both CTAs).
                if (!B200_TIMED(1, mbar_wait_cluster(&tmem_empty[buf * MSUB + s], acc_phase ^ 1u, kDevTimeoutMma))) {
                  ok = false;
                  break;
                }
                tc_fence_after_sync();
              }
              const uint64_t adesc =
                  kAColMajor
                      ? make_desc_mnmajor_sw128(a_addr + s * (Cfg::kASub * KSUB) + k * (kUmmaK * 128), Cfg::kBPanel)
                      : make_desc_kmajor_sw128(a_addr + (s * KSUB + sub) * Cfg::kASub + j * (kUmmaK * 2));
              const uint32_t d_tmem = tmem_base + (buf * MSUB + s) * Cfg::kAccCols;
#ifndef B200_GEMM_NOMMA
              umma_f16_cta2(d_tmem, adesc, bdesc, idesc, (kb != u.kb0 || k != 0) ? 1u : 0u);
#endif
              any_mma = true;
            }
            if (!ok) break;
          }
          if (!ok) break;
          const uint32_t e = smem_u32(&empty_bar[stage]);
          umma_commit_cta2(e);
          umma_commit_cta2(mapa_shared(e, 1));
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if constexpr (MSUB == 2) {
          if (P_end > 0) {
            int stg = stage;
            uint32_t ph = phase;
            for (int j = 0; j < P_end && ok; ++j) {
              if (!B200_TIMED(2, mbar_wait(&full_bar[stg], ph, kDevTimeoutMma))) { ok = false; break; }
              tc_fence_after_sync();
              issue_block(stg, kb_end + j, 0);
              if (++stg == STAGES) { stg = 0; ph ^= 1u; }
            }
            if (!ok) break;
            const uint32_t f0 = smem_u32(&tmem_full[buf * MSUB + 0]);
            umma_commit_cta2(f0);
            umma_commit_cta2(mapa_shared(f0, 1));
            for (int j = 0; j < P_end; ++j) {
              issue_block(stage, kb_end + j, 1);
              const uint32_t e = smem_u32(&empty_bar[stage]);
              umma_commit_cta2(e);
              umma_commit_cta2(mapa_shared(e, 1));
              if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
          }
        }
        const uint32_t f = smem_u32(&tmem_full[buf * MSUB + MSUB - 1]);
        umma_commit_cta2(f);
        umma_commit_cta2(mapa_shared(f, 1));
      }
      B200_PROF_ADD(4, clock64() - prof_t0);
      if (!ok && any_mma) {
        umma_commit_cta2(smem_u32(mma_drain));
        mbar_wait_drain(mma_drain, 0);
      }
    }
  } else {
    // ---------------- epilogue warps 2..5 (both CTAs) ----------------
    const int quad = warp & 3;
    const int ew = warp - 2;
    uint8_t* epi_buf = smem_epi + ew * 2 * kEpiBufBytes;
    const uint32_t epi_addr = smem_u32(epi_buf);
    int sbuf = 0;
    uint32_t c_phase = 0;
    int local = 0;
    WorkUnit u;
    auto next_unit = [&](int it, WorkUnit& w) -> bool {
      if constexpr (!kDyn) {
        return work_unit(it, pair, num_pairs, num_tiles, num_kb, st, w);
      } else {
        int tile = -1;
        bool popped = true;
        if (lane == 0) popped = dyn_pop(it, &tile, kDevTimeoutEpilogue);
        popped = __shfl_sync(0xffffffffu, popped, 0);
        tile = __shfl_sync(0xffffffffu, tile, 0);
        if (!popped || tile < 0) return false;
        w.t = tile;
        w.kb0 = 0;
        w.kb1 = num_kb;
        w.s = -1;
        return true;
      }
    };
    for (int it = 0; next_unit(it, u); ++it, ++local) {
      int mb, nb;
      sched.tile_coords(u.t, mb, nb);
      const int n0 = nb * Cfg::kTileN;
      const int buf = local % kAcc;
      const uint32_t acc_phase = (local / kAcc) & 1;
      bool got = true;
#pragma unroll 1
      for (int s = 0; s < MSUB; ++s) {
        // Each 256-column block is published on its own barrier.
        if (lane == 0) got = B200_TIMED(3, mbar_wait(&tmem_full[buf * MSUB + s], acc_phase, kDevTimeoutEpilogue));
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) break;
        tc_fence_after_sync();
        const int m0 = mb * Cfg::kTileM + (static_cast<int>(rank) * MSUB + s) * kBM;
        const uint32_t t_row =
            tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + (buf * MSUB + s) * Cfg::kAccCols;
#ifdef B200_GEMM_NOEPI
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tmem_empty[buf * MSUB + s]), 0));
        continue;
#endif
        if (MSUB == 1 && u.s >= 0) {
          // Tail unit of a split tile: publish this K range's part, and if it
          // is the last to arrive, sum all parts and store the tile.  Parts
          // move as 8 KB bulk copies ([quad][chunk] blocks of [q][lane]
          // float4) staged in this warp's share of the pipeline stages, which
          // are idle once the tail unit's MMAs have completed.
#ifdef B200_GEMM_PROFILE
          const uint64_t prof_s0 = global_timer_ns();
#endif
          const int tail = u.t - st.dp_tiles;
          float* part0 = st.ws + static_cast<size_t>(tail * st.S * 2 + static_cast<int>(rank)) * kPartFloats;
          const size_t part_stride = 2 * static_cast<size_t>(kPartFloats);   // next K range, same CTA
          uint8_t* fix_buf = smem + ew * (kFixBufs * kEpiChunkF32Bytes);   // kFixBufs x 8 KB
          uint64_t* fbar = fix_bar + ew * kFixBufs;
          constexpr int kChunks = Cfg::kTileN / kEpiCols;                   // 4
          static_assert(kChunks <= kFixBufs, "a part's chunks must fit the warp's buffers");
#pragma unroll 1
          for (int c = 0; c < kChunks; ++c) {
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(t_row + c * kEpiCols, lo);
            tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, hi);
            tmem_ld_wait_regs(lo);
            tmem_ld_wait_regs(hi);
            float* stage_f = reinterpret_cast<float*>(fix_buf + c * kEpiChunkF32Bytes);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const uint32_t* v = (q < 8) ? (lo + 4 * q) : (hi + 4 * (q - 8));
              st_shared_v4(smem_u32(stage_f + (q * 32 + lane) * 4), v[0], v[1], v[2], v[3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int c = 0; c < kChunks; ++c)
              bulk_store_s2g(part0 + u.s * part_stride + part_offset(quad, c, 0, 0), fix_buf + c * kEpiChunkF32Bytes,
                             kEpiChunkF32Bytes);
            bulk_commit_group();
            bulk_wait_group<0>();        // the part is in global memory
            fence_proxy_async_global();
          }
          B200_SPLIT_MARK(0, prof_s0);
          __syncwarp();
          __threadfence();
          asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
          B200_SPLIT_MARK(3, prof_s0);
          if (threadIdx.x == 64) *split_last = split_arrive_last(st.counters + tail * 2 + rank, st.S) ? 1u : 0u;
          B200_SPLIT_MARK(4, prof_s0);
          asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
          B200_SPLIT_MARK(5, prof_s0);
#ifdef B200_GEMM_PROFILE
          const uint64_t prof_s1 = global_timer_ns();
          B200_PROF_ADD(5, prof_s1 - prof_s0);
          B200_PROF_ADD(7, 1);
#endif
          if (*reinterpret_cast<volatile uint32_t*>(split_last)) {
            // The S - 1 other parts stream through the kFixBufs-buffer ring,
            // up to kFixBufs 8 KB loads in flight: load L (chunk L / (S-1))
            // uses buffer L % kFixBufs, phase (L / kFixBufs) & 1.
            __threadfence();
            fence_proxy_async_global();
            const int others = st.S - 1;
            const int total = kChunks * others;
            int issued = 0;
            auto issue_upto = [&](int limit) {
              if (lane == 0 && st.withhold_fixup_ns == 0) {
                for (int L = issued; L < limit && L < total; ++L) {
                  const int c = L / others, i = L % others;
                  const int r = i < u.s ? i : i + 1;  // the other K ranges in order
                  mbar_arrive_expect_tx(&fbar[L % kFixBufs], kEpiChunkF32Bytes);
                  bulk_load_g2s(fix_buf + (L % kFixBufs) * kEpiChunkF32Bytes,
                                part0 + r * part_stride + part_offset(quad, c, 0, 0), kEpiChunkF32Bytes,
                                &fbar[L % kFixBufs]);
                }
              }
              if (st.withhold_fixup_ns == 0) issued = limit < total ? limit : total;
            };
            issue_upto(kFixBufs);
            // A fixup wait that runs out abandons the tile: C is not stored
            // (the device error word says why), the loads still in flight
            // into this warp's buffers are drained, and the warp still joins
            // the epilogue barrier below.
            bool fix_ok = true;
#pragma unroll 1
            for (int c = 0; c < kChunks; ++c) {
              uint32_t lo[32], hi[32];
              tmem_ld_32x32b_x32(t_row + c * kEpiCols, lo);
              tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, hi);
              tmem_ld_wait_regs(lo);
              tmem_ld_wait_regs(hi);
              float acc[64];
#pragma unroll 1
              for (int r = 0; r < st.S; ++r) {
                const float* src = nullptr;
                if (r != u.s) {
                  const int L = c * others + (r < u.s ? r : r - 1);
                  const bool arrived = __all_sync(
                      0xffffffffu,
                      mbar_wait(&fbar[L % kFixBufs], static_cast<uint32_t>((L / kFixBufs) & 1), kDevTimeoutSplitFixup,
                                st.withhold_fixup_ns ? st.withhold_fixup_ns : kWaitLimitNs));
                  if (!arrived) {
                    if (lane == 0)
                      for (int L2 = L; L2 < issued; ++L2)
                        mbar_wait_drain(&fbar[L2 % kFixBufs], static_cast<uint32_t>((L2 / kFixBufs) & 1));
                    fix_ok = false;
                    break;
                  }
                  src = reinterpret_cast<const float*>(fix_buf + (L % kFixBufs) * kEpiChunkF32Bytes);
                }
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                  const uint32_t* own = (q < 8) ? (lo + 4 * q) : (hi + 4 * (q - 8));
                  float4 v;
                  if (src) {
                    v = *reinterpret_cast<const float4*>(src + (q * 32 + lane) * 4);
                  } else {
                    v = make_float4(__uint_as_float(own[0]), __uint_as_float(own[1]), __uint_as_float(own[2]),
                                    __uint_as_float(own[3]));
                  }
                  if (r == 0) {
                    acc[4 * q] = v.x; acc[4 * q + 1] = v.y; acc[4 * q + 2] = v.z; acc[4 * q + 3] = v.w;
                  } else {
                    acc[4 * q] += v.x; acc[4 * q + 1] += v.y; acc[4 * q + 2] += v.z; acc[4 * q + 3] += v.w;
                  }
                }
              }
              __syncwarp();                            // this chunk's buffers are free again
              if (!fix_ok) break;
              issue_upto((c + 1) * others + kFixBufs);
              if (c == 0) B200_SPLIT_MARK(6, prof_s0);
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                lo[e] = __float_as_uint(acc[e]);
                hi[e] = __float_as_uint(acc[32 + e]);
              }
              epi_store_block<2>(&tmap_c, epi_buf, epi_addr, sbuf, lane, lo, hi, n0 + c * kEpiCols, m0 + quad * 32,
                                 sc, &c_bar[ew], c_phase);
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
            if (threadIdx.x == 64) atomicExch(st.counters + tail * 2 + rank, 0u);  // ready for the next launch
            B200_SPLIT_MARK(7, prof_s0);
#ifdef B200_GEMM_PROFILE
            B200_PROF_ADD(6, global_timer_ns() - prof_s1);
#endif
          }
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tmem_empty[buf * MSUB + s]), 0));
          continue;
        }
        if (MSUB == 2 && sc.alpha == 1.0f && sc.beta == 0.0f) {
          // Plain product, wide pair (one tile fills TMEM, so the next tile's
          // MMAs wait for this block): the whole 256-column block goes to
          // registers as packed fp16 and the accumulator is handed back
          // before any store (measured 0.4-2 % faster than storing chunk by
          // chunk first, 8192^3 to 4000 x 6000 x 3000).
          uint32_t pk[Cfg::kChunksN][32];
#pragma unroll
          for (int c = 0; c < Cfg::kChunksN; ++c) {
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(t_row + c * kEpiCols, lo);
            tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, hi);
            tmem_ld_wait_regs(lo);
            tmem_ld_wait_regs(hi);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              pk[c][e] = pack_half2_rn(lo[2 * e], lo[2 * e + 1]);
              pk[c][16 + e] = pack_half2_rn(hi[2 * e], hi[2 * e + 1]);
            }
          }
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tmem_empty[buf * MSUB + s]), 0));
#pragma unroll
          for (int c = 0; c < Cfg::kChunksN; ++c)
            epi_store_block_packed<2>(&tmap_c, epi_buf, epi_addr, sbuf, lane, pk[c], n0 + c * kEpiCols,
                                      m0 + quad * 32, sc, n0 + Cfg::kTileN);
          continue;
        }
#pragma unroll 1
        for (int c = 0; c < Cfg::kChunksN; ++c) {
          uint32_t lo[32], hi[32];
          // (With BN % 64 != 0 the last block's upper columns read the unused
          // end of this accumulator block; they are never stored.)
          tmem_ld_32x32b_x32(t_row + c * kEpiCols, lo);
          tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, hi);
          tmem_ld_wait_regs(lo);
          tmem_ld_wait_regs(hi);
          if (c == Cfg::kChunksN - 1) {
            // This 256-column block is in registers: hand it back to the MMA warp.
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tmem_empty[buf * MSUB + s]), 0));
          }
          epi_store_block<2>(&tmap_c, epi_buf, epi_addr, sbuf, lane, lo, hi, n0 + c * kEpiCols, m0 + quad * 32, sc,
                             &c_bar[ew], c_phase, n0 + Cfg::kTileN);
        }
      }
      if (!got) break;
    }
    epi_peer_fence(sc);
    if (lane == 0) bulk_wait_group<0>();
  }

  B200_PROF_FLUSH
  tc_fence_before_sync();
  cluster_sync();  // no CTA leaves while its peer may still signal it or read its smem
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc<2>(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace b200
