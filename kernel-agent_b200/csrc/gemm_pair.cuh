// The CTA-pair GEMM: two CTAs of a cluster (two SMs) compute one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256). Each CTA loads 128 rows of A and 128 rows of B
// (half of the tile's columns) per stage; the MMA, issued by the even CTA of the pair (the
// leader), reads both CTAs' shared memory and writes each CTA's 128 x 256 accumulator into its
// own TMEM. Per SM, every byte staged in shared memory feeds twice the tensor work of the
// one-CTA kernel's 128 x 192 tile, and A and B are each read from L2 N / 256 and M / 256
// times instead of N / 192 and M / 128.
//
// Block scales: each CTA loads, per stage, the scale chunks of its 128 rows of A and of the
// tile's 256 rows of B (the MMA of either CTA needs all 256 columns' scales) by TMA, counted on
// the leader's stage barrier like A and B. The leader's MMA thread copies them into a TMEM slot
// of both CTAs (tcgen05.cp.cta_group::2, 32x128b.warpx4: chunk row l into lane l of every
// lane quarter) right before the stage's MMAs; tcgen05 operations of one thread execute in
// issue order, so the copies land before the MMAs read them and a slot is rewritten only after
// the MMAs that read it.
//
// Roles per CTA (warps): 0 TMA producer, 1 MMA issuer (leader only), 2-9 epilogue. Barriers:
//   full[s]      leader: stage s landed in both CTAs (the peer's TMA loads count their bytes
//                on the leader's barrier; the leader's producer expects both CTAs' bytes)
//   empty[s]     each CTA: the MMAs that read stage s completed (the leader commits to both)
//   acc_full[b]  each CTA: accumulator b is final
//   acc_empty[b] leader: both CTAs' epilogue warps read accumulator b (16 arrivals)
// Barriers the other CTA arrives on are waited on with cluster scope. No load uses cluster
// multicast: each CTA loads its own operands. Every wait is bounded (~1 s): a timeout sets
// kDevTimeout and the role winds down, and both CTAs still meet at the final cluster barriers.
//
// TMEM per CTA (512 columns): int8 / fp8, two 256-column accumulators; block-scaled kinds,
// one accumulator and a ring of scale-factor slots in the other 256 columns.
#pragma once

#include "gemm.cuh"

namespace kab {

template <int KIND, int OUT>
struct PairLayout {
  static constexpr int kBM = 128;      // rows of A per CTA (256 per pair)
  static constexpr int kBN = 256;      // columns of the pair's tile = accumulator columns per CTA
  static constexpr int kBNHalf = 128;  // rows of B per CTA
  static constexpr int BKB = 128;      // bytes of K per row per stage
  static constexpr int kKSteps = BKB / 32;
  static constexpr bool kScaled = KIND >= 2;
  static constexpr int kABytes = kBM * BKB;
  static constexpr int kBBytes = kBNHalf * BKB;
  static constexpr int kGroups = kBN / 32;  // 32-column groups of B's scale factors per tile
  // scale bytes per 128 rows per stage: one 512-byte chunk per 64 elements of K (NVFP4), per
  // 128 (MXFP4: two 32-element blocks per word pair), per 128 (MXFP8)
  static constexpr int kSfChunkBytes = KIND == 3 ? 512 * kKSteps : (KIND == 4 ? 256 * kKSteps : 512);
  static constexpr int kSfRows = kSfChunkBytes / 256;  // rows of the [*, 256]-byte scale tensor map
  static constexpr int kSfaBytes = kScaled ? kSfChunkBytes : 0;
  static constexpr int kSfbBytes = kScaled ? 2 * kSfChunkBytes : 0;  // the tile's 256 rows of B
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr int kSfSets = KIND == 3 ? kKSteps : (KIND == 4 ? kKSteps / 2 : 1);
  static constexpr int kSfaCols = kScaled ? 4 * kSfSets : 0;
  static constexpr int kSfbCols = kScaled ? kGroups * kSfSets : 0;
  static constexpr int kSfColsPerStage = kSfaCols + kSfbCols;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 32 * (2 + kEpiWarps);
  static constexpr int kAccBufs = kScaled ? 1 : 2;
  static constexpr int kSfCol = kAccBufs * kBN;
  static constexpr int kSfSlotsFit = kScaled ? (512 - kSfCol) / kSfColsPerStage : 0;
  static constexpr int kSfSlots = kSfSlotsFit > 5 ? 5 : kSfSlotsFit;
  static constexpr int kStageOutBytes = 32 * 128;  // one [32 rows, 128 bytes] store per warp
  static constexpr int kStagingBytes = kEpiWarps * kStageOutBytes;
  static_assert(kStagingBytes % 1024 == 0, "the operand tiles after the staging tiles need 1024-byte alignment");
  static constexpr int kSmemLimit = 232448;
  static constexpr int kFixed = 1024 + kStagingBytes + 256;
  static constexpr int kStagesFit = (kSmemLimit - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kBarriers = 2 * kStages + 2 * kAccBufs + 1 + kSfSlots;
  static constexpr int kSmem = 1024 + kStagingBytes + kStages * kStageBytes + kBarriers * 8 + 16;
  static_assert(kStages >= 2, "shared memory does not fit two stages");
  static_assert(!kScaled || kSfSlots >= 2, "TMEM does not fit two scale-factor slots");
  static_assert(kSfCol + kSfSlots * kSfColsPerStage <= 512, "TMEM overflow");
  static_assert(kSmem <= kSmemLimit, "shared memory overflow");
};

// g.m_tiles / g.n_tiles count 256 x 256 pair tiles; the grid is 2 x the number of pairs.
// tma_sfa / tma_sfb: the swizzled scale tensors as [rows, 256] bytes (block-scaled kinds).
template <int KIND, int OUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairLayout<KIND, OUT>::kThreads, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 const __grid_constant__ CUtensorMap tma_sfa, const __grid_constant__ CUtensorMap tma_sfb,
                 const __grid_constant__ CUtensorMap tma_out, GemmArgs g, const __grid_constant__ PeerMaps peers) {
  using L = PairLayout<KIND, OUT>;
  constexpr int STAGES = L::kStages;
  constexpr int KS = L::kKSteps;
  constexpr int BN = L::kBN;
  constexpr int BKB = L::BKB;
  constexpr int AB = L::kAccBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sOut = smem;
  uint8_t* sA = sOut + L::kStagingBytes;
  uint8_t* sB = sA + STAGES * L::kABytes;
  uint8_t* sSFA = sB + STAGES * L::kBBytes;
  uint8_t* sSFB = sSFA + STAGES * L::kSfaBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + STAGES * L::kSfbBytes);
  uint64_t* full = bars;
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + AB;
  uint64_t* drain = acc_empty + AB;
  uint64_t* sf_empty = drain + 1;  // leader: the MMAs that read scale-factor slot i completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_empty + L::kSfSlots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();  // 0: the leader
  const int pair0 = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < AB; ++b) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 2 * L::kEpiWarps);
    }
    tc::mbar_init(drain, 1);
    for (int i = 0; i < L::kSfSlots; ++i) tc::mbar_init(&sf_empty[i], 1);
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tma_a);
    tc::prefetch_tensormap(&tma_b);
    if constexpr (L::kScaled) {
      tc::prefetch_tensormap(&tma_sfa);
      tc::prefetch_tensormap(&tma_sfb);
    }
    tc::prefetch_tensormap(&tma_out);
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, 512);
    tc::tmem_relinquish_pair();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int total = g.m_tiles * g.n_tiles;

  if (warp == 0) {
    {  // ------------------------------------------------------------------- TMA producer
      // the whole warp walks the loop and waits (as the MMA warp does); one elected lane issues
      const bool issuer = tc::elect_one();
      const uint32_t full_leader = tc::mapa(full, 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = pair0; ok && t < total; t += npairs) {
        int mt, nt;
        tile_coords(t, g.m_tiles, g.n_tiles, g.group_n, mt, nt);
        const int arow = mt * 256 + static_cast<int>(rank) * 128;
        const int brow = nt * 256 + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < g.k_stages; ++kb) {
          if (!__all_sync(0xffffffffu, tc::mbar_wait_cluster(&empty[s], ph ^ 1u))) { ok = false; break; }
          if (issuer) {
            const uint32_t bar = full_leader + 8 * s;
            if (rank == 0) tc::mbar_arrive_expect_tx(&full[s], 2 * L::kStageBytes);
            tc::tma_load_2d_pair(&tma_a, bar, sA + s * L::kABytes, kb * BKB, arow);
            tc::tma_load_2d_pair(&tma_b, bar, sB + s * L::kBBytes, kb * BKB, brow);
            if constexpr (L::kScaled) {
              // the stage's chunk of 128-row block r starts at byte (r * ncb + kc) * 512; a block
              // past the end of the tensor reads as zeros (and counts its bytes)
              const int64_t kc = KIND == 3 ? static_cast<int64_t>(KS) * kb : (KIND == 4 ? static_cast<int64_t>(KS / 2) * kb : kb);
              const int64_t ra = static_cast<int64_t>(mt) * 2 + rank;
              tc::tma_load_2d_pair(&tma_sfa, bar, sSFA + s * L::kSfaBytes, 0, static_cast<int>(2 * (ra * g.sfa_ncb + kc)));
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                const int64_t rb = static_cast<int64_t>(nt) * 2 + c;
                tc::tma_load_2d_pair(&tma_sfb, bar, sSFB + s * L::kSfbBytes + c * L::kSfChunkBytes, 0,
                                     static_cast<int>(2 * (rb * g.sfb_ncb + kc)));
              }
            }
          }
          __syncwarp();
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok && lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
    }
  } else if (warp == 1) {
    if (rank == 0) {  // ---------------------------------------------------- MMA issuer (leader)
      // The whole warp walks the loop and waits; one elected lane issues the tcgen05
      // instructions, and the warp reconverges after each group. Issued from a lone lane
      // whose warp-mates wait elsewhere (at the final barrier), each tcgen05.cp took ~47
      // cycles to issue and the twelve copies of a stage did not overlap the MMAs (B200,
      // 256 x 256 x 64 NVFP4 pair MMAs: 819 vs 512 cycles per stage with the warp converged).
      const bool leader = tc::elect_one();
      const uint32_t empty_own = tc::smem_u32(empty), acc_full_own = tc::smem_u32(acc_full);
      // The block scales of a stage go into a TMEM slot one k-step ahead of the MMAs that read
      // them (the copies of step i + 1 are issued before the MMAs of step i); a slot is
      // rewritten only after the MMAs that read it have completed (sf_empty).
      const int my_tiles = pair0 < total ? (total - pair0 + npairs - 1) / npairs : 0;
      const int64_t steps = static_cast<int64_t>(my_tiles) * g.k_stages;
      int s = 0, ab = 0, slot = 0;        // the MMAs' stage, accumulator and scale slot
      int cs = 0, cslot = 0;              // the next copies' stage and slot
      uint32_t aph = 0, cph = 0, csph = 0;
      bool ok = true;
      // every lane waits (the verdict is the warp's), the elected lane issues
      auto wait_all = [&](uint64_t* bar, uint32_t parity, bool cluster) -> bool {
        const bool done = cluster ? tc::mbar_wait_cluster(bar, parity) : tc::mbar_wait(bar, parity);
        return __all_sync(0xffffffffu, done);
      };
      // waits for stage cs to land and slot cslot to be free, then copies the stage's scales
      auto copy_next = [&]() -> bool {
        if (!wait_all(&full[cs], cph, true)) return false;
        if constexpr (L::kScaled) {
          if (!wait_all(&sf_empty[cslot], csph ^ 1u, false)) return false;
        }
        if constexpr (L::kScaled) {  // set j: A's chunk j -> 4 columns, B's two chunks j -> 8
          if (leader) {
            const uint32_t sf = tmem + L::kSfCol + cslot * L::kSfColsPerStage;
            const uint32_t fa = tc::smem_u32(sSFA + cs * L::kSfaBytes);
            const uint32_t fb = tc::smem_u32(sSFB + cs * L::kSfbBytes);
#pragma unroll
            for (int j = 0; j < L::kSfSets; ++j) {
              tc::cp_sf_pair(sf + 4 * j, tc::desc_sf(fa + j * 512));
#pragma unroll
              for (int c = 0; c < 2; ++c)
                tc::cp_sf_pair(sf + L::kSfaCols + L::kGroups * j + 4 * c, tc::desc_sf(fb + c * L::kSfChunkBytes + j * 512));
            }
          }
          __syncwarp();
          if (++cslot == L::kSfSlots) { cslot = 0; csph ^= 1u; }
        }
        if (++cs == STAGES) { cs = 0; cph ^= 1u; }
        return true;
      };
      int64_t step = 0;
      if (steps > 0 && !copy_next()) ok = false;
      for (int t = pair0; ok && t < total; t += npairs) {
        if (!wait_all(&acc_empty[ab], aph ^ 1u, true)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + ab * BN;
        for (int kb = 0; kb < g.k_stages; ++kb, ++step) {
          // stage s has landed (copy_next waited for it one step ago)
          if (step + 1 < steps && !copy_next()) { ok = false; break; }
          if (leader) {
            const uint64_t adesc = tc::desc_sw128(tc::smem_u32(sA + s * L::kABytes));
            const uint64_t bdesc = tc::desc_sw128(tc::smem_u32(sB + s * L::kBBytes));
            const uint32_t sf = tmem + L::kSfCol + slot * L::kSfColsPerStage;
#pragma unroll
            for (int j = 0; j < KS; ++j) {
              const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
              const uint64_t a = adesc + static_cast<uint64_t>(2 * j);  // +32 bytes of K
              const uint64_t b = bdesc + static_cast<uint64_t>(2 * j);
              if constexpr (KIND == 0) {
                tc::mma_i8_pair(d, a, b, tc::idesc_i8(256, BN), acc);
              } else if constexpr (KIND == 1) {
                tc::mma_f8_pair(d, a, b, tc::idesc_f8(256, BN), acc);
              } else if constexpr (KIND == 2) {
                tc::mma_mxf8_pair(d, a, b, tc::idesc_mxf8(256, BN, j), sf, sf + L::kSfaCols, acc);
              } else if constexpr (KIND == 3) {
                tc::mma_nvf4_pair(d, a, b, tc::idesc_nvf4(256, BN), sf + 4 * j, sf + L::kSfaCols + L::kGroups * j, acc);
              } else {
                tc::mma_mxf4_pair(d, a, b, tc::idesc_mxf4(256, BN, 2 * (j & 1)), sf + 4 * (j >> 1),
                                  sf + L::kSfaCols + L::kGroups * (j >> 1), acc);
              }
            }
            tc::commit_pair_both(empty_own + 8 * s);  // stage s is free in both CTAs
            if constexpr (L::kScaled) tc::commit_pair(tc::smem_u32(&sf_empty[slot]));
          }
          __syncwarp();
          if (++s == STAGES) s = 0;
          if constexpr (L::kScaled) {
            if (++slot == L::kSfSlots) slot = 0;
          }
        }
        if (!ok) break;
        if (leader) {
          tc::commit_pair_both(acc_full_own + 8 * ab);
        }
        __syncwarp();
        if (++ab == AB) { ab = 0; aph ^= 1u; }
      }
      if (leader) tc::commit_pair(tc::smem_u32(drain));  // every MMA issued has completed once this arrives
      __syncwarp();
      if (!wait_all(drain, 0, false)) ok = false;
      if (!ok && leader) atomicOr(&g_gemm_status, kDevTimeout);
    }
  } else {  // ------------------------------------------------------------- epilogue warps
    constexpr int HC = BN / 64;  // 32-column chunks per warp per tile
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    const uint32_t acc_empty_leader = tc::mapa(acc_empty, 0);
    uint8_t* stage0 = sOut + (warp - 2) * L::kStageOutBytes;
    int ab = 0;
    uint32_t aph = 0;
    for (int t = pair0; t < total; t += npairs) {
      int mt, nt;
      tile_coords(t, g.m_tiles, g.n_tiles, g.group_n, mt, nt);
      const int row0 = mt * 256 + static_cast<int>(rank) * 128 + 32 * quarter;
      const int colh = nt * BN + half * (BN / 2);
      EpilogueOperands<KIND, OUT, HC> ops;
      ops.load(g, row0, colh, lane);  // before the accumulator is ready
      if (!tc::mbar_wait_cluster(&acc_full[ab], aph)) {
        if (lane == 0) atomicOr(&g_gemm_status, kDevTimeout);
        break;
      }
      tc::fence_after_sync();
      const uint32_t tbase = tmem + lane_base + ab * BN + half * (BN / 2);
      const uint32_t release_bar = acc_empty_leader + 8 * ab;
      epilogue_tile_wide<KIND, OUT, HC>(g, ops, &tma_out, g.npeers > 0 ? &peers : nullptr, tbase, row0, colh, stage0,
                                        lane, [release_bar] { tc::mbar_arrive_cluster(release_bar); });
      if (++ab == AB) { ab = 0; aph ^= 1u; }
    }
    if (lane == 0) tc::bulk_wait_all();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync();  // neither CTA's barriers or TMEM are used by the other after this
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc_pair(tmem, 512);
  }
  tc::cluster_sync();  // both deallocations are done before either CTA exits
}

}  // namespace kab
