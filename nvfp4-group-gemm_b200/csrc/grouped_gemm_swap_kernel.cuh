// Weight-stationary ("swap A/B") variant of the persistent NVFP4 grouped GEMM, for
// groups with few rows (decode-style MoE routing: many experts see a handful of tokens).
//
// The GEMM is computed transposed, C_g^T = B_g A_g^T: each tile is 128 weight rows
// (n) x 64 token rows (m), with the weights as the MMA's 128-row A operand and the
// tokens as its 64-column B operand (tcgen05.mma M = 128, N = 64). With the usual
// orientation a 128-token tile of a 10-token group is 92 % zero padding that still
// occupies the shared-memory ring; here a pipeline stage is 16 KiB of weights, 8 KiB
// of tokens and 4 KiB of scale factors, so seven stages keep 112 KiB of weights in
// flight per SM (the row tiles of the other kernels fit three stages, 96 KiB of
// B and 48 KiB of mostly-empty A). The epilogue writes C straight from registers:
// lane l of epilogue warp q holds output column n = 128 nt + 32 q + l for 64
// consecutive rows, so every store instruction writes 64 contiguous bytes.
//
// Scheduling, failure handling and the tile-schedule ring are those of the
// single-CTA kernel (grouped_gemm_kernel.cuh).
#pragma once

#include <cuda_fp16.h>

#include "grouped_gemm_kernel.cuh"
#include "nvfp4_types.cuh"
#include "sm100_ptx.cuh"

namespace nvfp4 {

template <int STAGES>
struct SwapConfig {
  static constexpr int kTokens = 64;  // MMA N: token rows per tile
  static constexpr int kWBytes = 128 * kRowBytesPerStage;
  static constexpr int kXBytes = kTokens * kRowBytesPerStage;
  static constexpr int kSfwBytes = 4 * kSfBlockBytes;  // weight rows' 128-row scale block
  static constexpr int kSfxBytes = 4 * kSfBlockBytes;  // token rows' 128-row scale block
  static constexpr int kStageBytes = kWBytes + kXBytes + kSfwBytes + kSfxBytes;
  static constexpr uint32_t kTxBytes = kStageBytes;
  static constexpr int kAccStages = 2;
  static constexpr int kSfColBase = kAccStages * kTokens;  // accumulators in columns [0, 128)
  static constexpr int kSfwCols = 16;                      // 4 MMAs x 4 columns
  static constexpr uint32_t kTmemAllocCols = 256;
  static_assert(kSfColBase + 2 * kSfwCols <= static_cast<int>(kTmemAllocCols), "TMEM");
  static constexpr int kBarrierBytes =
      8 * (2 * STAGES + 2 * kAccStages + 1 + 2 * kSchedSlots) + 16 + 16 * kSchedSlots;
  static constexpr int kSmemBytes = 1024 + STAGES * kStageBytes + kBarrierBytes + kTileEndBytes;
  static_assert(kSmemBytes <= 232448, "exceeds 227 KB of shared memory per CTA");
  static constexpr uint32_t kIdesc = ptx::make_idesc_mxf4nvf4(128, kTokens);
};

template <int STAGES>
__global__ void __launch_bounds__(kNumThreads, 1)
    nvfp4_grouped_gemm_swap_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = SwapConfig<STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stage_base = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;
  uint64_t* acce_bar = accf_bar + Cfg::kAccStages;
  uint64_t* drain_bar = acce_bar + Cfg::kAccStages;
  uint64_t* sched_full = drain_bar + 1;
  uint64_t* sched_empty = sched_full + kSchedSlots;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sched_empty + kSchedSlots);
  volatile uint32_t* abort_flag = tmem_holder + 1;
  // Slot i: {tile, group, K, token scale-column offset}; tile >= total_tiles ends the schedule.
  volatile int32_t* sched_info = reinterpret_cast<volatile int32_t*>(tmem_holder + 4);
  int32_t* tile_ends = const_cast<int32_t*>(sched_info + 4 * kSchedSlots);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const GroupDev* __restrict__ groups = p.groups;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full_bar[s], 1);
      ptx::mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < Cfg::kAccStages; ++a) {
      ptx::mbar_init(&accf_bar[a], 1);
      ptx::mbar_init(&acce_bar[a], kEpilogueWarps);
    }
    ptx::mbar_init(drain_bar, 1);
    for (int i = 0; i < kSchedSlots; ++i) {
      ptx::mbar_init(&sched_full[i], 1);
      ptx::mbar_init(&sched_empty[i], kSchedConsumers);
    }
    *abort_flag = 0u;
    ptx::fence_mbarrier_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_holder, Cfg::kTmemAllocCols);
    ptx::tmem_relinquish_alloc_permit();
  }
  // Everything above is local to the CTA. Group records, tensor maps, operands and the
  // tile counter may come from the previous kernels in the stream: wait for them here,
  // then let the next launch be scheduled onto SMs as this grid's CTAs retire.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  stage_tile_ends(tile_ends, groups, p.num_groups);
  ptx::tcgen05_fence_before_sync();
  __syncthreads();
  ptx::tcgen05_fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (ptx::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      auto acquire_maps = [&](int grp) {
        const TmaDesc* m = p.maps + static_cast<size_t>(grp) * kMapsPerGroup;
        ptx::tensormap_fence_acquire(&m[kMapA64]);
        ptx::tensormap_fence_acquire(&m[kMapB]);
      };
      int tile = blockIdx.x;  // grid <= total_tiles: every CTA has a first tile
      int g = advance_group(tile_ends, groups, p.num_groups, 0, tile);
      GroupDev gd = groups[g];
      acquire_maps(g);
      for (uint32_t seq = 0;; ++seq) {
        const int slot = static_cast<int>(seq % kSchedSlots);
        if (!wait_phase(&sched_empty[slot], ((seq / kSchedSlots) & 1u) ^ 1u, abort_flag,
                        p.error_bits, kDevErrProducerTimeout))
          break;
        const int local = tile - gd.tile_start;
        const int mt = tile < p.total_tiles ? local % gd.tiles_m : 0;  // 64-token chunk
        sched_info[4 * slot + 0] = tile;
        sched_info[4 * slot + 1] = g;
        sched_info[4 * slot + 2] = gd.k;
        sched_info[4 * slot + 3] = 2 * (mt & 1);  // rows 64..127 of the scale block: columns 2, 3
        ptx::mbar_arrive(&sched_full[slot]);
        if (tile >= p.total_tiles) break;
        const TmaDesc* maps = p.maps + static_cast<size_t>(g) * kMapsPerGroup;
        const int nt = local / gd.tiles_m;  // 128-row weight block
        const int ktiles = gd.k / kBlockK;
        const int rest_k = gd.k / 64;
        const uint8_t* sfw_blk = gd.sfb + static_cast<size_t>(nt) * rest_k * kSfBlockBytes;
        const uint8_t* sfx_blk = gd.sfa + static_cast<size_t>(mt >> 1) * rest_k * kSfBlockBytes;
        const int claim_kt = ktiles > kClaimLeadKTiles ? ktiles - kClaimLeadKTiles : 0;
        int next_tile = p.total_tiles;
        int g_next = g;
        GroupDev next_gd = gd;
        bool resolved = false;
        auto resolve_next = [&]() {
          resolved = true;
          if (next_tile >= p.total_tiles) return;
          g_next = advance_group(tile_ends, groups, p.num_groups, g, next_tile);
          next_gd = groups[g_next];
          if (g_next != g) acquire_maps(g_next);
        };
        for (int kt = 0; kt < ktiles; ++kt) {
          if (!wait_phase(&empty_bar[stage], phase ^ 1u, abort_flag, p.error_bits,
                          kDevErrProducerTimeout)) {
            ok = false;
            break;
          }
          uint8_t* sW = stage_base + stage * Cfg::kStageBytes;
          uint8_t* sX = sW + Cfg::kWBytes;
          uint8_t* sSFW = sX + Cfg::kXBytes;
          uint8_t* sSFX = sSFW + Cfg::kSfwBytes;
          ptx::mbar_arrive_expect_tx(&full_bar[stage], Cfg::kTxBytes);
          const int kx = kt * kRowBytesPerStage;
          ptx::tma_load_2d(sW, &maps[kMapB], &full_bar[stage], kx, nt * 128);
          ptx::tma_load_2d(sX, &maps[kMapA64], &full_bar[stage], kx, mt * Cfg::kTokens);
          const size_t sf_off = static_cast<size_t>(kt) * 4 * kSfBlockBytes;
          ptx::bulk_load(sSFW, sfw_blk + sf_off, 4 * kSfBlockBytes, &full_bar[stage]);
          ptx::bulk_load(sSFX, sfx_blk + sf_off, 4 * kSfBlockBytes, &full_bar[stage]);
          // Claim the next tile a few k-tiles before the end of this one and resolve it
          // one k-tile later, behind loads already in flight (as in the single-CTA kernel).
          if (kt == claim_kt)
            next_tile = p.dynamic_schedule
                            ? static_cast<int>(gridDim.x + atomicAdd(p.tile_counter, 1u))
                            : tile + static_cast<int>(gridDim.x);
          if (kt == claim_kt + 1) resolve_next();
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (!resolved) resolve_next();
        tile = next_tile;
        g = g_next;
        gd = next_gd;
      }
      // No copy into this CTA's shared memory may still be in flight at exit.
      const uint32_t recent = issued < static_cast<uint32_t>(STAGES) ? issued : STAGES;
      for (uint32_t i = 0; i < recent; ++i) {
        const uint32_t n = issued - 1 - i;
        const uint32_t s = n % STAGES;
        const uint32_t ph = (n / STAGES) & 1u;
        uint64_t t0 = ptx::globaltimer_ns();
        while (!ptx::mbar_try_wait(&full_bar[s], ph)) {
          if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
            atomicOr(p.error_bits, kDevErrDrainTimeout);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (ptx::elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_parity = 0x3u;  // disjoint double buffer: the first two tiles pass
      bool ok = p.diag_skip_mma == 0;
      const uint32_t sfw_t = tmem_base + Cfg::kSfColBase;
      const uint32_t sfx_t = sfw_t + Cfg::kSfwCols;
      for (uint32_t local = 0; ok; ++local) {
        const int slot = static_cast<int>(local % kSchedSlots);
        if (!wait_phase(&sched_full[slot], (local / kSchedSlots) & 1u, abort_flag, p.error_bits,
                        kDevErrMmaTimeout))
          break;
        const int tile = sched_info[4 * slot + 0];
        const int ktiles = sched_info[4 * slot + 2] / kBlockK;
        const uint32_t sfx_shift = static_cast<uint32_t>(sched_info[4 * slot + 3]);
        ptx::mbar_arrive(&sched_empty[slot]);
        if (tile >= p.total_tiles) break;
        const int acc = static_cast<int>(local & 1u);
        if (!wait_phase(&acce_bar[acc], (acc_parity >> acc) & 1u, abort_flag, p.error_bits,
                        kDevErrAccTimeout))
          break;
        acc_parity ^= 1u << acc;
        ptx::tcgen05_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kTokens;
        for (int kt = 0; kt < ktiles; ++kt) {
          if (!wait_phase(&full_bar[stage], phase, abort_flag, p.error_bits, kDevErrMmaTimeout)) {
            ok = false;
            break;
          }
          ptx::tcgen05_fence_after_sync();
          const uint32_t sW = ptx::smem_u32(stage_base + stage * Cfg::kStageBytes);
          const uint32_t sX = sW + Cfg::kWBytes;
          const uint32_t sSFW = sX + Cfg::kXBytes;
          const uint32_t sSFX = sSFW + Cfg::kSfwBytes;
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            ptx::tmem_cp_32x128b_warpx4(sfw_t + 4 * kb,
                                        ptx::make_sf_block_desc(sSFW + kb * kSfBlockBytes));
            ptx::tmem_cp_32x128b_warpx4(sfx_t + 4 * kb,
                                        ptx::make_sf_block_desc(sSFX + kb * kSfBlockBytes));
          }
          const uint64_t w_desc = ptx::make_sw128_kmajor_desc(sW);
          const uint64_t x_desc = ptx::make_sw128_kmajor_desc(sX);
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            // Token scales: the N = 64 MMA reads two columns (32 tokens each) starting at
            // the chunk's half of the 128-row scale block.
            ptx::mma_mxf4nvf4(d_tmem, w_desc + 2 * kb, x_desc + 2 * kb, Cfg::kIdesc,
                              sfw_t + 4 * kb, sfx_t + 4 * kb + sfx_shift,
                              (kt | kb) != 0 ? 1u : 0u);
          }
          ptx::tcgen05_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::tcgen05_commit(&accf_bar[acc]);
      }
      ptx::tcgen05_commit(drain_bar);
      uint64_t t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(drain_bar, 0)) {
        if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
          atomicOr(p.error_bits, kDevErrDrainTimeout);
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter: weight rows 32q..32q+31 of the tile
    uint32_t full_parity = 0;
    for (uint32_t local = 0;; ++local) {
      const int slot = static_cast<int>(local % kSchedSlots);
      if (!warp_wait_phase(&sched_full[slot], (local / kSchedSlots) & 1u, abort_flag,
                           p.error_bits, kDevErrEpilogueTimeout, lane))
        break;
      const int tile = sched_info[4 * slot + 0];
      const int g = sched_info[4 * slot + 1];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&sched_empty[slot]);
      if (tile >= p.total_tiles) break;
      const GroupDev gd = groups[g];  // in flight while the accumulator is awaited
      const int acc = static_cast<int>(local & 1u);
      if (!warp_wait_phase(&accf_bar[acc], (full_parity >> acc) & 1u, abort_flag, p.error_bits,
                           kDevErrEpilogueTimeout, lane))
        break;
      full_parity ^= 1u << acc;
      ptx::tcgen05_fence_after_sync();
      const uint32_t t_acc =
          tmem_base + (static_cast<uint32_t>(32 * quarter) << 16) + acc * Cfg::kTokens;
      uint32_t v0[32], v1[32];
      ptx::tmem_ld_32x32b_x32(t_acc, v0);
      ptx::tmem_ld_32x32b_x32(t_acc + 32, v1);
      ptx::tmem_ld_wait();
      ptx::tcgen05_fence_before_sync();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&acce_bar[acc]);  // accumulator back to the MMA issuer
      const int tl = tile - gd.tile_start;
      const int mt = tl % gd.tiles_m;
      const int nt = tl / gd.tiles_m;
      const int n = nt * 128 + 32 * quarter + lane;
      const int m0 = mt * Cfg::kTokens;
      const int rows = min(Cfg::kTokens, gd.m - m0);
      if (n < gd.n) {
        __half* out = reinterpret_cast<__half*>(gd.c) + static_cast<size_t>(m0) * gd.n + n;
#pragma unroll
        for (int j = 0; j < Cfg::kTokens; ++j)
          if (j < rows)
            out[static_cast<size_t>(j) * gd.n] =
                __float2half_rn(__uint_as_float(j < 32 ? v0[j] : v1[j - 32]) * gd.alpha);
      }
    }
  }

  ptx::tcgen05_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    ptx::tcgen05_fence_after_sync();
    ptx::tmem_dealloc(tmem_base, Cfg::kTmemAllocCols);
  }
  if (threadIdx.x == 0 && p.dynamic_schedule) release_tile_counter(p.tile_counter);
}

}  // namespace nvfp4
