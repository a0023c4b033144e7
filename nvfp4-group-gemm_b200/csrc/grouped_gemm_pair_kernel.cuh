// CTA-pair (cta_group::2) variant of the persistent NVFP4 grouped GEMM.
//
// A cluster of two CTAs on two SMs computes one 256 x 256 tile per step (gated:
// 256 rows x 128 output columns, the MMA's 256 B rows being 128 gate + 128 up rows):
//
//   CTA r (r = 0, 1) loads the 128 A rows [256 mt + 128 r, +128) and one half of the
//   256 B rows, plus the scale factors of its A rows and of all 256 B rows; the even
//   CTA issues tcgen05.mma.cta_group::2 (M = 256, N = 256), which reads A and B from
//   both CTAs' shared memory and writes each CTA's 128 accumulator rows into that
//   CTA's TMEM. Per SM this halves the B bytes per MMA compared with a 128 x 256 tile
//   on one SM, which is what lets the mainloop keep the tensor pipe fed.
//
// Synchronisation between the two CTAs (no TMA multicast anywhere):
//   full[s]   even CTA; one arrive.expect_tx (both CTAs' bytes) by its producer, and
//             every load of both CTAs completes its bytes there (cta_group::2 TMA)
//   empty[s]  each CTA; the even CTA's MMA commit arrives on both CTAs' barriers
//             (tcgen05.commit .multicast::cluster, mask 0x3). Forwarding the release
//             to the odd CTA from the even CTA's producer instead left the odd CTA's
//             refill behind that producer's wake-up: cfg2's MMA issuer waited for data
//             46 % of each k-tile.
//   accf[a]   each CTA; the same two-CTA commit
//   acce[a]   even CTA; the 8 epilogue warps of both CTAs release accumulators there
// All waits are bounded (same timeout/abort scheme as the single-CTA kernel); a
// final cluster barrier keeps both CTAs alive until every cross-CTA access is done.
#pragma once

#include <cuda_fp16.h>

#include "grouped_gemm_kernel.cuh"
#include "nvfp4_types.cuh"
#include "sm100_ptx.cuh"

namespace nvfp4 {

// K bytes of A/B rows per pipeline stage of the pair kernel: 128 (a whole 256-element
// k-tile, 128-byte swizzle) or 64 (half a k-tile, 64-byte swizzle: twice the stages of half
// the size, released after two MMAs instead of four). The host encodes the pair launches'
// operand and scale maps to match. 128 by default: with 64 (ten 19-KiB stages instead of
// five 38-KiB ones, the same bytes in flight) cfg2 took 107.1 vs 97.3 us per call, the gated
// G=8 configuration about 125 vs 89-108 us and cfg5 about 3500 vs 3200 us on one B200.
#ifndef NVFP4_PAIR_STAGE_KBYTES
#define NVFP4_PAIR_STAGE_KBYTES 128
#endif
constexpr int kPairStageKBytes = NVFP4_PAIR_STAGE_KBYTES;
static_assert(kPairStageKBytes == 128 || kPairStageKBytes == 64, "64 or 128 K bytes per stage");
constexpr int kPairStagesPerKTile = kRowBytesPerStage / kPairStageKBytes;
constexpr int kPairSfBlocksPerStage = kPairStageKBytes / 32;  // one 512-B block per 64 K
constexpr int kPairSfRowsPerStage = 4 * kPairSfBlocksPerStage;  // 128-byte rows of a scale map

template <bool GATED, int STAGES>
struct PairConfig {
  static constexpr int kMmaN = 256;
  static constexpr int kOutN = GATED ? 128 : 256;  // output columns per tile
  static constexpr int kABytes = 128 * kPairStageKBytes;
  static constexpr int kBBytes = 128 * kPairStageKBytes;  // this CTA's half of B
  static constexpr int kSfaBytes = kPairSfBlocksPerStage * kSfBlockBytes;      // its 128 A rows
  static constexpr int kSfbBytes = 2 * kPairSfBlocksPerStage * kSfBlockBytes;  // all 256 B rows
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr uint32_t kPairTxBytes = 2u * kStageBytes;  // both CTAs, every stage
  // Overlapped accumulator stages (stride 192 columns) and one scale-factor slot.
  static constexpr int kAccStride = kMmaN - 64;
  static constexpr int kSfColBase = kAccStride + kMmaN;
  static constexpr int kSfaCols = 16;
  static constexpr int kSfbColsPerMma = kMmaN / 32;
  static_assert(kSfColBase + kSfaCols + 4 * kSfbColsPerMma <= kTmemCols, "TMEM over-subscribed");
  static constexpr int kEpiBufBytes = 32 * 128;
  static constexpr int kEpiBufsPerWarp = 2;
  static constexpr int kEpiBytes = kEpilogueWarps * kEpiBufsPerWarp * kEpiBufBytes;
  static constexpr int kBarrierBytes = 8 * (2 * STAGES + 2 * 2 + 1) + 16;
  static constexpr int kSmemBytes =
      1024 + STAGES * kStageBytes + kEpiBytes + kBarrierBytes + kTileEndBytes;
  static_assert(kSmemBytes <= 232448, "exceeds 227 KB of shared memory per CTA");
  static constexpr uint32_t kIdesc = ptx::make_idesc_mxf4nvf4(256, kMmaN);
  static constexpr uint32_t kEpilogueArrivals = 2 * kEpilogueWarps;
};

template <bool GATED, int STAGES>
__global__ void __launch_bounds__(kNumThreads, 1)
    nvfp4_grouped_gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = PairConfig<GATED, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stage_base = smem;
  uint8_t* epi_base = smem + STAGES * Cfg::kStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_base + Cfg::kEpiBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* drain_bar = acce_bar + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile uint32_t* abort_flag = tmem_holder + 1;
  int32_t* tile_ends = reinterpret_cast<int32_t*>(tmem_holder + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const GroupDev* __restrict__ groups = p.groups;
  const uint32_t rank = ptx::cluster_ctarank();  // 0: issues the MMAs
  const bool leader = rank == 0;
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int num_clusters = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full_bar[s], 1);
      ptx::mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&accf_bar[a], 1);
      ptx::mbar_init(&acce_bar[a], Cfg::kEpilogueArrivals);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    ptx::fence_mbarrier_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_holder, kTmemCols);
    ptx::tmem_relinquish_alloc_permit_pair();
  }
  // Local set-up above; data written by earlier kernels in the stream is read only after
  // this wait. The next launch may then be scheduled as this grid's CTAs retire.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  stage_tile_ends(tile_ends, groups, p.num_groups);  // ordered by the cluster barrier below
  // Segment launches learn their tile count from the workspace (written by the segment
  // set-up kernel); clusters beyond it have no tile and end at once.
  const int total_tiles = p.seg_total_tiles != nullptr ? *p.seg_total_tiles : p.total_tiles;
  // Barriers of both CTAs initialised and TMEM allocated in both before any
  // cross-CTA arrive, load completion or MMA.
  ptx::tcgen05_fence_before_sync();
  ptx::cluster_sync_all();
  ptx::tcgen05_fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (ptx::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      int acquired_g = -1;
      bool ok = true;
      // The record of the next tile's group is loaded while this tile's loads are issued.
      int g = advance_group(tile_ends, groups, p.num_groups, 0, cluster);
      GroupDev next_gd = groups[g];
      for (int tile = cluster; ok && tile < total_tiles; tile += num_clusters) {
        const GroupDev gd = next_gd;
        const int g_next = advance_group(tile_ends, groups, p.num_groups, g, tile + num_clusters);
        next_gd = groups[g_next];
        const TmaDesc* maps = p.maps + static_cast<size_t>(g) * kMapsPerGroup;
        // Tensor maps of a group are acquired before its first loads: here for the CTA's
        // first tile, and otherwise behind the previous tile's first loads (below).
        auto acquire_maps = [&](const TmaDesc* m) {
          ptx::tensormap_fence_acquire(&m[kMapA]);
          ptx::tensormap_fence_acquire(&m[kMapB]);
          ptx::tensormap_fence_acquire(&m[kMapSfa]);
          ptx::tensormap_fence_acquire(&m[kMapSfb]);
          if (GATED) {
            ptx::tensormap_fence_acquire(&m[kMapB2]);
            ptx::tensormap_fence_acquire(&m[kMapSfb2]);
          }
        };
        if (g != acquired_g) {
          acquire_maps(maps);
          acquired_g = g;
        }
        const int local = tile - gd.tile_start;
        const int mt = local % gd.tiles_m;
        const int nt = local / gd.tiles_m;
        const int ktiles = gd.k / kBlockK;
        const int rest_k = gd.k / 64;
        const int rb = seg_row(p, g);  // first row of the group's segment (0 normally)
        const int row_a = rb + mt * 256 + 128 * static_cast<int>(rank);
        // This CTA's half of the MMA's B rows.
        const TmaDesc* map_b = (GATED && rank == 1) ? &maps[kMapB2] : &maps[kMapB];
        const int row_b = GATED ? nt * 128 : nt * 256 + 128 * static_cast<int>(rank);
        // Scale blocks, in 128-byte rows of the scale maps (16 rows = one k-tile of a
        // 128-row block; a block out of range reads as 0).
        const int sfa_y0 = (rb / 128 + 2 * mt + static_cast<int>(rank)) * rest_k * 4;
        const TmaDesc* map_sfb1 = GATED ? &maps[kMapSfb2] : &maps[kMapSfb];
        const int sfb0_y0 = (GATED ? nt : 2 * nt) * rest_k * 4;
        const int sfb1_y0 = (GATED ? nt : 2 * nt + 1) * rest_k * 4;
        const bool warm_a = kL2PrefetchModePair == 2 || (kL2PrefetchModePair == 1 && nt == 0);
        const bool warm_b = kL2PrefetchModePair == 2 || (kL2PrefetchModePair == 1 && mt == 0);
        // Stages of this tile (kPairStagesPerKTile per 256-element k-tile).
        const int kstages = ktiles * kPairStagesPerKTile;
        const int prefetch_ahead = kL2PrefetchKTiles * kPairStagesPerKTile;
        auto prefetch_stage = [&](int kp) {
          if (warm_a) {
            ptx::tma_prefetch_l2_2d(&maps[kMapA], kp * kPairStageKBytes, row_a);
            ptx::tma_prefetch_l2_2d(&maps[kMapSfa], 0, sfa_y0 + kp * kPairSfRowsPerStage);
          }
          if (warm_b) {
            ptx::tma_prefetch_l2_2d(map_b, kp * kPairStageKBytes, row_b);
            ptx::tma_prefetch_l2_2d(&maps[kMapSfb], 0, sfb0_y0 + kp * kPairSfRowsPerStage);
            ptx::tma_prefetch_l2_2d(map_sfb1, 0, sfb1_y0 + kp * kPairSfRowsPerStage);
          }
        };
        if (warm_a || warm_b)
          for (int kp = 0; kp < prefetch_ahead && kp < kstages; ++kp) prefetch_stage(kp);
        for (int kt = 0; kt < kstages; ++kt) {
          if ((warm_a || warm_b) && kt + prefetch_ahead < kstages)
            prefetch_stage(kt + prefetch_ahead);
          if (!wait_phase(&empty_bar[stage], phase ^ 1u, abort_flag, p.error_bits,
                                  kDevErrProducerTimeout)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = ptx::mapa_shared(ptx::smem_u32(&full_bar[stage]), 0);
          // Both CTAs' empty barriers are arrived by the MMAs' commit, so the odd CTA may
          // load its half before the leader has armed the full barrier with both halves'
          // byte count: its completed bytes then wait in the barrier's transaction count,
          // and the phase cannot complete before the leader's arrival.
          if (leader) ptx::mbar_arrive_expect_tx(&full_bar[stage], Cfg::kPairTxBytes);
          uint8_t* sA = stage_base + stage * Cfg::kStageBytes;
          uint8_t* sB = sA + Cfg::kABytes;
          uint8_t* sSFA = sB + Cfg::kBBytes;
          uint8_t* sSFB = sSFA + Cfg::kSfaBytes;
          const int kx = kt * kPairStageKBytes;
          const int sfy = kt * kPairSfRowsPerStage;
          ptx::tma_load_2d_pair(sA, &maps[kMapA], full_leader, kx, row_a);
          ptx::tma_load_2d_pair(sB, map_b, full_leader, kx, row_b);
          ptx::tma_load_2d_pair(sSFA, &maps[kMapSfa], full_leader, 0, sfa_y0 + sfy);
          ptx::tma_load_2d_pair(sSFB, &maps[kMapSfb], full_leader, 0, sfb0_y0 + sfy);
          ptx::tma_load_2d_pair(sSFB + kPairSfBlocksPerStage * kSfBlockBytes, map_sfb1,
                                full_leader, 0, sfb1_y0 + sfy);
          if (kt == 0 && g_next != acquired_g) {
            acquire_maps(p.maps + static_cast<size_t>(g_next) * kMapsPerGroup);
            acquired_g = g_next;
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        g = g_next;
      }
      if (leader) {
        // Every fill of both CTAs completes on these barriers: wait for the most recent
        // fill of each stage before the cluster may exit.
        const uint32_t recent = issued < static_cast<uint32_t>(STAGES) ? issued : STAGES;
        for (uint32_t i = 0; i < recent; ++i) {
          const uint32_t n = issued - 1 - i;
          const uint32_t s = n % STAGES;
          const uint32_t ph = (n / STAGES) & 1u;
          const uint64_t t0 = ptx::globaltimer_ns();
          while (!ptx::mbar_try_wait(&full_bar[s], ph)) {
            if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
              atomicOr(p.error_bits, kDevErrDrainTimeout);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && ptx::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_parity = 0x1u;  // overlapped stages: only the first tile passes freely
      uint32_t local = 0;
      bool ok = p.diag_skip_mma == 0;
      int g = advance_group(tile_ends, groups, p.num_groups, 0, cluster);
      int next_k = groups[g].k;
      for (int tile = cluster; ok && tile < total_tiles; tile += num_clusters, ++local) {
        const int ktiles = next_k / kBlockK;
        g = advance_group(tile_ends, groups, p.num_groups, g, tile + num_clusters);
        next_k = groups[g].k;
        const int acc = static_cast<int>(local & 1u);
        if (!wait_phase(&acce_bar[acc], (acc_parity >> acc) & 1u, abort_flag,
                                p.error_bits, kDevErrAccTimeout)) {
          break;
        }
        acc_parity ^= 1u << acc;
        ptx::tcgen05_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccStride;
        for (int kt = 0; kt < ktiles * kPairStagesPerKTile; ++kt) {
          if (!wait_phase(&full_bar[stage], phase, abort_flag, p.error_bits,
                                  kDevErrMmaTimeout)) {
            ok = false;
            break;
          }
          ptx::tcgen05_fence_after_sync();
          const uint32_t sA = ptx::smem_u32(stage_base + stage * Cfg::kStageBytes);
          const uint32_t sB = sA + Cfg::kABytes;
          const uint32_t sSFA = sB + Cfg::kBBytes;
          const uint32_t sSFB = sSFA + Cfg::kSfaBytes;
          const uint32_t sfa_t = tmem_base + Cfg::kSfColBase;
          const uint32_t sfb_t = sfa_t + Cfg::kSfaCols;
#pragma unroll
          for (int kb = 0; kb < kPairSfBlocksPerStage; ++kb)
            ptx::tmem_cp_32x128b_warpx4_pair(sfa_t + 4 * kb,
                                             ptx::make_sf_block_desc(sSFA + kb * kSfBlockBytes));
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int kb = 0; kb < kPairSfBlocksPerStage; ++kb)
              ptx::tmem_cp_32x128b_warpx4_pair(
                  sfb_t + Cfg::kSfbColsPerMma * kb + 4 * j,
                  ptx::make_sf_block_desc(sSFB + j * kPairSfBlocksPerStage * kSfBlockBytes +
                                          kb * kSfBlockBytes));
          }
          const uint64_t a_desc = kPairStageKBytes == 128 ? ptx::make_sw128_kmajor_desc(sA)
                                                          : ptx::make_sw64_kmajor_desc(sA);
          const uint64_t b_desc = kPairStageKBytes == 128 ? ptx::make_sw128_kmajor_desc(sB)
                                                          : ptx::make_sw64_kmajor_desc(sB);
#pragma unroll
          for (int kb = 0; kb < kPairSfBlocksPerStage; ++kb) {
            ptx::mma_mxf4nvf4_pair(d_tmem, a_desc + 2 * kb, b_desc + 2 * kb, Cfg::kIdesc,
                                   sfa_t + 4 * kb, sfb_t + Cfg::kSfbColsPerMma * kb,
                                   (kt | kb) != 0 ? 1u : 0u);
          }
          ptx::tcgen05_commit_pair_both(&empty_bar[stage]);  // frees the stage in both CTAs
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::tcgen05_commit_pair_both(&accf_bar[acc]);  // both CTAs' epilogues may start
      }
      ptx::tcgen05_commit_pair(drain_bar);
      const uint64_t t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(drain_bar, 0)) {
        if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
          atomicOr(p.error_bits, kDevErrDrainTimeout);
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - kEpilogueWarp0;
    const int quarter = warp & 3;
    uint8_t* my_bufs = epi_base + ew * Cfg::kEpiBufsPerWarp * Cfg::kEpiBufBytes;
    const uint32_t my_bufs_s = ptx::smem_u32(my_bufs);
    uint32_t full_parity = 0;
    uint32_t stores = 0;
    uint32_t local = 0;
    int acquired_g = -1;
    constexpr int kBoxes = Cfg::kOutN / 64;
    int g_next = advance_group(tile_ends, groups, p.num_groups, 0, cluster);
    GroupDev next_gd = groups[g_next];
    for (int tile = cluster; tile < total_tiles; tile += num_clusters, ++local) {
      const GroupDev gd = next_gd;
      const int g = g_next;
      const int rb = seg_row(p, g);  // C rows of the group start here
      g_next = advance_group(tile_ends, groups, p.num_groups, g, tile + num_clusters);
      next_gd = groups[g_next];
      const TmaDesc* map_c = p.maps + static_cast<size_t>(g) * kMapsPerGroup + kMapC;
      if (g != acquired_g) {
        if (lane == 0) ptx::tensormap_fence_acquire(map_c);
        acquired_g = g;
      }
      const int tl = tile - gd.tile_start;
      const int mt = tl % gd.tiles_m;
      const int nt = tl / gd.tiles_m;
      const int acc = static_cast<int>(local & 1u);
      if (!warp_wait_phase(&accf_bar[acc], (full_parity >> acc) & 1u, abort_flag,
                                   p.error_bits, kDevErrEpilogueTimeout, lane)) {
        break;
      }
      full_parity ^= 1u << acc;
      ptx::tcgen05_fence_after_sync();
      const uint32_t release_bar = ptx::mapa_shared(ptx::smem_u32(&acce_bar[acc ^ 1]), 0);
      const int first_box = (acc == 0) ? kBoxes - 1 : 0;
      const int row0 = mt * 256 + 128 * static_cast<int>(rank) + 32 * quarter;
      bool released = false;
      if (row0 < gd.m) {
        const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(32 * quarter) << 16) +
                               acc * Cfg::kAccStride;
        // Scattered output: where this thread's row goes (nullptr: not stored).
        const bool scatter = !GATED && p.row_dest != nullptr;
        uint8_t* out_row = nullptr;
        if (scatter && row0 + lane < gd.m)
          out_row = scatter_row(p, static_cast<int64_t>(rb) + row0 + lane);
        // This thread's C row (for replicated output; nullptr past the group's rows).
        uint8_t* c_row = row0 + lane < gd.m
                             ? gd.c + static_cast<size_t>(rb + row0 + lane) * gd.n * sizeof(__half)
                             : nullptr;
        // Drains one box (32 rows x 64 columns of this warp's quarter) whose accumulator
        // values (and, gated, the up projection's) are in registers.
        auto drain_box = [&](int box, const uint32_t (&v0)[32], const uint32_t (&v1)[32],
                             const uint32_t (&u0)[32], const uint32_t (&u1)[32]) {
          const uint32_t buf = my_bufs_s + (stores & 1u) * Cfg::kEpiBufBytes;
          if (GATED && p.out_sf != nullptr) {
            // NVFP4 output (codes and blocked scales; no fp16 staging).
            const int row = row0 + lane;
            if (row < gd.m) {
              const int col0 = nt * Cfg::kOutN + box * 64;
              const int64_t r = static_cast<int64_t>(rb) + row;
              store_gated_box_nvfp4(v0, v1, u0, u1, gd.alpha, gd.alpha2, p.out_scale,
                                    p.out_d6, gd.c + r * (gd.n / 2) + col0 / 2,
                                    p.out_sf + blocked_sf_offset(r, col0 / 16, (gd.n + 63) / 64));
            }
            return;
          }
          if (lane == 0) ptx::bulk_wait_group_read<1>();
          __syncwarp();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint32_t* v = half ? v1 : v0;
            uint32_t packed[16];
            if (GATED) {
              const uint32_t* u = half ? u1 : u0;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                __half2 hv = __floats2half2_rn(
                    gated_value(v[2 * i], u[2 * i], gd.alpha, gd.alpha2),
                    gated_value(v[2 * i + 1], u[2 * i + 1], gd.alpha, gd.alpha2));
                packed[i] = *reinterpret_cast<uint32_t*>(&hv);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                __half2 hv = __floats2half2_rn(__uint_as_float(v[2 * i]) * gd.alpha,
                                               __uint_as_float(v[2 * i + 1]) * gd.alpha);
                packed[i] = *reinterpret_cast<uint32_t*>(&hv);
              }
            }
            const uint32_t row_addr = buf + lane * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t chunk = static_cast<uint32_t>(half * 4 + c) ^ (lane & 7);
              ptx::st_shared_v4(row_addr + chunk * 16, packed[4 * c], packed[4 * c + 1],
                                packed[4 * c + 2], packed[4 * c + 3]);
            }
          }
          if (scatter) {
            __syncwarp();
            store_box_rows(my_bufs + (stores & 1u) * Cfg::kEpiBufBytes, out_row,
                           nt * Cfg::kOutN + box * 64, gd.n, lane);
            __syncwarp();  // the box is read before it is written again
            ++stores;
            return;
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d(map_c, my_bufs + (stores & 1u) * Cfg::kEpiBufBytes,
                              nt * Cfg::kOutN + box * 64, rb + row0);
            ptx::bulk_commit_group();
          }
          // Replicas: the same staged box into each peer copy of C, four 128-byte row
          // pieces per warp store, while the TMA store writes the local copy.
          for (int r = 0; r < p.num_replicas; ++r)
            store_box_rows(my_bufs + (stores & 1u) * Cfg::kEpiBufBytes,
                           c_row != nullptr ? c_row + p.replica_offset[r] : nullptr,
                           nt * Cfg::kOutN + box * 64, gd.n, lane);
          ++stores;
        };
        auto release_shared_box = [&]() {
          // The box shared by both accumulator stages is drained: the next tile's MMAs may
          // start.
          ptx::tcgen05_fence_before_sync();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive_cluster(release_bar);
          released = true;
        };
        if constexpr (GATED) {
#pragma unroll 1
          for (int bi = 0; bi < kBoxes; ++bi) {
            const int box = (first_box + bi) % kBoxes;
            uint32_t v0[32], v1[32], u0[32], u1[32];
            ptx::tmem_ld_32x32b_x32(t_acc + box * 64, v0);
            ptx::tmem_ld_32x32b_x32(t_acc + box * 64 + 32, v1);
            ptx::tmem_ld_32x32b_x32(t_acc + 128 + box * 64, u0);
            ptx::tmem_ld_32x32b_x32(t_acc + 128 + box * 64 + 32, u1);
            ptx::tmem_ld_wait();
            if (bi == 0) release_shared_box();
            drain_box(box, v0, v1, u0, u1);
          }
        } else {
          // Box bi + 1's TMEM loads are issued before box bi is converted and stored, so
          // they run under its shared-memory writes and TMA store.
          uint32_t a0[32], a1[32], b0[32], b1[32];
          ptx::tmem_ld_32x32b_x32(t_acc + first_box * 64, a0);
          ptx::tmem_ld_32x32b_x32(t_acc + first_box * 64 + 32, a1);
#pragma unroll
          for (int bi = 0; bi < kBoxes; ++bi) {
            const int box = (first_box + bi) % kBoxes;
            ptx::tmem_ld_wait();
            if (bi & 1) {
              ptx::reg_fence(b0);
              ptx::reg_fence(b1);
            } else {
              ptx::reg_fence(a0);
              ptx::reg_fence(a1);
            }
            if (bi == 0) release_shared_box();
            if (bi + 1 < kBoxes) {
              const int next = (first_box + bi + 1) % kBoxes;
              if (bi & 1) {
                ptx::tmem_ld_32x32b_x32(t_acc + next * 64, a0);
                ptx::tmem_ld_32x32b_x32(t_acc + next * 64 + 32, a1);
              } else {
                ptx::tmem_ld_32x32b_x32(t_acc + next * 64, b0);
                ptx::tmem_ld_32x32b_x32(t_acc + next * 64 + 32, b1);
              }
            }
            if (bi & 1)
              drain_box(box, b0, b1, b0, b1);
            else
              drain_box(box, a0, a1, a0, a1);
          }
        }
      }
      if (!released) {
        ptx::tcgen05_fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(release_bar);
      }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

  // Keep both CTAs resident until every remote arrive, load completion and MMA that
  // touches the other CTA is done, then free the pair's TMEM.
  ptx::tcgen05_fence_before_sync();
  ptx::cluster_sync_all();
  if (warp == 1) {
    ptx::tcgen05_fence_after_sync();
    ptx::tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace nvfp4
