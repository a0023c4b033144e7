// Persistent, warp-specialised NVFP4 block-scaled grouped GEMM for sm_100a.
//
//   C_g[m, n] = fp16( alpha_g * sum_k  e2m1(A_g[m, k]) * sfa_g[m, k/16]
//                                     * e2m1(B_g[n, k]) * sfb_g[n, k/16] )
//
// and, when GATED, the fused MoE gate/up form
//
//   C_g = fp16( silu(fp16(alpha_g * A_g Bgate_g^T)) * fp16(alpha2_g * A_g Bup_g^T) )
//
// which keeps the reference's rounding of the two projections to fp16 before the
// SiLU product (submission.py:877-884, :707-710).
//
// One CTA per SM walks a static schedule of (group, m-tile, n-tile) work units;
// inside the CTA:
//   warp 0       TMA producer: A/B tiles by tensor map (128B swizzle), scale-factor
//                blocks by plain bulk copies, into a STAGES-deep mbarrier ring
//   warp 1       TMEM allocator + single-thread tcgen05 issuer: scale factors
//                smem->TMEM (tcgen05.cp), 4 x tcgen05.mma kind::mxf4nvf4 per stage
//   warps 2..5   epilogue: TMEM -> registers -> alpha / SiLU -> fp16 -> swizzled
//                smem -> TMA store (out-of-range rows/columns clipped by the map)
//
// Every mbarrier wait is bounded in time: on timeout the CTA records the reason
// in the workspace error word, drains its in-flight copies and MMAs, frees TMEM
// and returns, so a malformed launch cannot hang the GPU.
#pragma once

#include <cuda_fp16.h>

#include "nvfp4_quant_math.cuh"
#include "nvfp4_types.cuh"
#include "sm100_ptx.cuh"

namespace nvfp4 {

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s per wait
constexpr int kNumThreads = 192;
constexpr int kEpilogueWarp0 = 2;
constexpr int kEpilogueWarps = 4;
constexpr int kTmemCols = 512;
// k-tiles the producer warms in L2 ahead of its TMA loads. CTAs that share an A or B
// tile walk K in lockstep, so without this every one of them waits on the same DRAM
// miss at every k-step; the prefetch turns those misses into L2 hits.
#ifndef NVFP4_L2_PREFETCH_KTILES
#define NVFP4_L2_PREFETCH_KTILES 6
#endif
constexpr int kL2PrefetchKTiles = NVFP4_L2_PREFETCH_KTILES;
// Groups whose tile_end values are staged in shared memory (see advance_group).
constexpr int kSmemGroups = 512;
constexpr int kTileEndBytes = kSmemGroups * 4;
// Dynamic tile schedule: after its first tile (blockIdx.x) a CTA claims each next tile
// from a launch-wide counter, kClaimLeadKTiles k-tiles before it finishes issuing the
// loads of its current one, so that CTAs whose tiles ran faster take more of them.
// The producer hands each claimed (tile, group, K) to the MMA issuer and the epilogue
// through a ring of kSchedSlots shared-memory slots.
constexpr int kSchedSlots = 4;
constexpr int kClaimLeadKTiles = 3;
constexpr uint32_t kSchedConsumers = 1 + kEpilogueWarps;  // MMA issuer + epilogue warps
// Which producers warm L2: 0 none, 1 one per shared tile (B by the CTAs on the first
// m-tile of a group, A by those on its first n-tile), 2 every producer for its own tiles.
// Measured on cfg2 (G=8, 1024 x 4096 x 7168): single-CTA tiles 108.8 / 119.1 / 133.3 us
// with modes 1 / 0 / 2; CTA-pair tiles 97.0 / 96.3 / 111.4 us (their deeper ring needs no
// warm-up, and every prefetch is an extra L2 request).
#ifndef NVFP4_L2_PREFETCH_SINGLE
#define NVFP4_L2_PREFETCH_SINGLE 1
#endif
#ifndef NVFP4_L2_PREFETCH_PAIR
#define NVFP4_L2_PREFETCH_PAIR 0
#endif
constexpr int kL2PrefetchMode = NVFP4_L2_PREFETCH_SINGLE;
constexpr int kL2PrefetchModePair = NVFP4_L2_PREFETCH_PAIR;

// DIRECT: the epilogue stores C from registers (16 bytes per lane, one row per lane)
// instead of staging 64-column boxes in shared memory for TMA stores. That frees the
// 32 KiB of staging space for a fourth pipeline stage at MMA_N = 256, for launches whose
// run time is the weight stream (groups of at most a few hundred rows).
template <int MMA_N, bool GATED, int STAGES, bool DIRECT = false>
struct GemmConfig {
  static constexpr bool kDirectStore = DIRECT;
  static_assert(MMA_N == 128 || MMA_N == 256, "MMA N must be 128 or 256");
  static_assert(!GATED || MMA_N == 256, "gated tiles pair 128 gate + 128 up columns");
  static constexpr int kOutN = GATED ? MMA_N / 2 : MMA_N;  // output columns per tile
  static constexpr int kABytes = kBlockM * kRowBytesPerStage;
  static constexpr int kBBytes = MMA_N * kRowBytesPerStage;
  static constexpr int kSfaBytes = 4 * kSfBlockBytes;                 // 128 rows x 16 scales
  static constexpr int kSfbBlocks = MMA_N / 128;
  static constexpr int kSfbBytes = kSfbBlocks * 4 * kSfBlockBytes;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  // Two accumulator stages. At MMA_N = 256 they overlap by one 64-column epilogue box
  // (stage 1 starts at column 192): the epilogue drains that shared box first and
  // releases it, so the next tile's MMAs start while the other three boxes drain.
  static constexpr bool kOverlapAcc = (MMA_N == 256);
  static constexpr int kAccStages = 2;
  static constexpr int kAccStride = kOverlapAcc ? MMA_N - 64 : MMA_N;
  // Scale factors: one TMEM slot above the accumulators. tcgen05.cp and tcgen05.mma
  // issued by one thread execute in order, so a slot is reused safely every k-tile.
  static constexpr int kSfaCols = 4 * 4;              // 4 MMAs x 4 columns (128 lanes x 4 B)
  static constexpr int kSfbColsPerMma = MMA_N / 32;   // one column per 32 rows of B
  static constexpr int kSfbCols = 4 * kSfbColsPerMma;
  static constexpr int kSfColBase = kAccStride + MMA_N;
  static_assert(kSfColBase + kSfaCols + kSfbCols <= kTmemCols, "TMEM over-subscribed");
  static constexpr int kEpiBufBytes = 32 * 128;  // 32 rows x 64 fp16, one TMA store box
  static constexpr int kEpiBufsPerWarp = 2;
  static constexpr int kEpiBytes = DIRECT ? 0 : kEpilogueWarps * kEpiBufsPerWarp * kEpiBufBytes;
  // mbarriers (stage ring, accumulators, drain, tile-schedule ring), TMEM address and
  // abort flag, tile-schedule slots.
  static constexpr int kBarrierBytes =
      8 * (2 * STAGES + 2 * kAccStages + 1 + 2 * kSchedSlots + 2) + 16 + 16 * kSchedSlots;
  static constexpr int kSmemBytes = 1024 /*alignment slack*/ + STAGES * kStageBytes + kEpiBytes +
                                    kBarrierBytes + kTileEndBytes;
  static_assert(kSmemBytes <= 232448, "exceeds 227 KB of shared memory per CTA");
  static constexpr uint32_t kIdesc = ptx::make_idesc_mxf4nvf4(kBlockM, MMA_N);
  static constexpr int kNTilesPerOut = kOutN;  // output column span of one tile
};

// Bounded wait: true when the phase completed; false after a timeout (reason
// recorded) or when another role of this CTA has already aborted.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity,
                                           volatile uint32_t* abort_flag, uint32_t* error_bits,
                                           uint32_t reason) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((++spins & 31u) == 0) {
      if (*abort_flag) return false;
      if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
        *abort_flag = 1u;
        atomicOr(error_bits, reason);
        return false;
      }
    }
  }
}

// Stream-K hand-off counter: arrivals of a cut tile's two pieces count in the low byte;
// this bit says the first piece's partial rows are stored.
constexpr int32_t kSkPublished = 0x100;

// Bounded wait until bit `bit` of a word that another SM sets (stream-K partial rows
// published); same timeout and abort scheme as wait_phase.
__device__ __forceinline__ bool wait_global_bit(const int32_t* word, int bit,
                                                volatile uint32_t* abort_flag,
                                                uint32_t* error_bits, uint32_t reason) {
  const volatile int32_t* w = word;
  const uint64_t t0 = ptx::globaltimer_ns();
  while ((*w & bit) == 0) {
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1u;
      atomicOr(error_bits, reason);
      return false;
    }
    __nanosleep(128);
  }
  return true;
}

// Warp-wide bounded wait with one decision for all lanes (the epilogue's TMEM
// loads are warp-collective, so lanes must never disagree about a timeout).
// Lane 0 waits; once it has seen the phase complete, every lane re-probes the
// same (already completed) phase to take its own acquire.
__device__ __forceinline__ bool warp_wait_phase(uint64_t* bar, uint32_t parity,
                                                volatile uint32_t* abort_flag,
                                                uint32_t* error_bits, uint32_t reason, int lane) {
  int ok = 1;
  if (lane == 0) ok = wait_phase(bar, parity, abort_flag, error_bits, reason) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) {
    for (uint32_t i = 0; i < (1u << 20) && !ptx::mbar_try_wait(bar, parity); ++i) {
    }
  }
  return ok != 0;
}

// Gated epilogue value of one output element: fp16(silu(fp16(alpha * gate)) * fp16(alpha2 *
// up)). Gate and up are rounded to fp16 first, as the reference's two-GEMM path does; SiLU
// and the product are fp32.
__device__ __forceinline__ float gated_value(uint32_t gate_bits, uint32_t up_bits, float alpha,
                                             float alpha2) {
  const float gte = __half2float(__float2half_rn(__uint_as_float(gate_bits) * alpha));
  const float up = __half2float(__float2half_rn(__uint_as_float(up_bits) * alpha2));
  return __fdividef(gte, 1.0f + __expf(-gte)) * up;
}

// NVFP4 output of one row's 64-column box of a gated tile: the fp16 values the fp16 output
// would hold, quantised in blocks of 16 exactly as nvfp4_quantize quantises that output.
// Writes 32 bytes of codes at `codes` (16-byte aligned) and the four scale codes as one
// 4-byte store at `sf`.
__device__ __forceinline__ void store_gated_box_nvfp4(const uint32_t* v0, const uint32_t* v1,
                                                      const uint32_t* u0, const uint32_t* u1,
                                                      float alpha, float alpha2, float sg,
                                                      float d6, uint8_t* codes, uint8_t* sf) {
  uint32_t sf4 = 0;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t* v = half ? v1 : v0;
    const uint32_t* u = half ? u1 : u0;
    float hv[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      hv[i] = __half2float(__float2half_rn(gated_value(v[i], u[i], alpha, alpha2)));
    uint32_t c0, c1;
    const uint2 q0 = quantize16(hv, sg, d6, c0);
    const uint2 q1 = quantize16(hv + 16, sg, d6, c1);
    sf4 |= (c0 | (c1 << 8)) << (16 * half);
    *reinterpret_cast<uint4*>(codes + 16 * half) = make_uint4(q0.x, q0.y, q1.x, q1.y);
  }
  *reinterpret_cast<uint32_t*>(sf) = sf4;
}

// Scattered output of one staged box: the warp's 32 rows x 64 fp16 columns sit in shared
// memory (row i at box + 128 * i, 16-byte chunks XOR-swizzled by (i & 7)); `dst` is this
// lane's row destination (nullptr: not stored). Each store instruction writes four whole
// 128-byte row pieces (eight lanes per row), so remote (NVLink) writes go out as full lines
// instead of 32 separate 16-byte pieces.
__device__ __forceinline__ void store_box_rows(const uint8_t* box, uint8_t* dst, int col0, int n,
                                               int lane) {
  const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
  const int c = lane & 7;  // 16-byte chunk = 8 columns
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = 4 * k + (lane >> 3);
    uint8_t* row = reinterpret_cast<uint8_t*>(__shfl_sync(0xffffffffu, mine, r));
    const uint4 v = *reinterpret_cast<const uint4*>(box + r * 128 + ((c ^ (r & 7)) * 16));
    const int col = col0 + 8 * c;
    if (row != nullptr && col < n)
      *reinterpret_cast<uint4*>(row + static_cast<size_t>(col) * sizeof(__half)) = v;
  }
}

// Tile -> group lookup. Tiles are numbered group by group and every CTA meets its
// tiles in increasing order, so the lookup starts from the previous answer `g`.
// Launches of up to kSmemGroups groups first copy each group's tile_end into shared
// memory (one parallel load at kernel start) and search that copy; larger launches
// search the records in global memory. A CTA passes ~grid/tiles-per-group groups
// between two of its tiles (about 20 for 64 groups of 7 tiles): a linear walk cost
// one dependent load per group and stalled the start of every tile, so the lookup
// checks the current group and otherwise bisects the rest.
__device__ __forceinline__ void stage_tile_ends(int32_t* ends, const GroupDev* groups,
                                                int num_groups) {
  if (num_groups <= kSmemGroups)
    for (int i = threadIdx.x; i < num_groups; i += blockDim.x) ends[i] = groups[i].tile_end;
}

__device__ __forceinline__ int advance_group(const int32_t* ends, const GroupDev* groups,
                                             int num_groups, int g, int tile) {
  const bool in_smem = num_groups <= kSmemGroups;
  auto end_of = [&](int i) { return in_smem ? ends[i] : groups[i].tile_end; };
  if (g + 1 >= num_groups || tile < end_of(g)) return g;
  // First group in (g, num_groups - 1] whose tile_end exceeds `tile` (tile_end is
  // non-decreasing); the last group when none does.
  int lo = g + 1, hi = num_groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (tile >= end_of(mid)) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Work units: tiles [0, split_first_tile) are one unit each; every later tile is split into
// split_parts units along K (split s takes k-tiles [s*kt/S, (s+1)*kt/S)), which come last
// in the unit order. split = -1 marks an unsplit tile.
__device__ __forceinline__ void unit_tile(const GemmParams& p, int unit, int& tile, int& split) {
  if (unit < p.split_first_tile) {
    tile = unit;
    split = -1;
  } else {
    const int r = unit - p.split_first_tile;
    tile = p.split_first_tile + r / p.split_parts;
    split = r % p.split_parts;
  }
}

__device__ __forceinline__ void unit_krange(const GemmParams& p, int split, int ktiles, int& k0,
                                            int& k1) {
  if (split < 0) {
    k0 = 0;
    k1 = ktiles;
  } else {
    k0 = split * ktiles / p.split_parts;
    k1 = (split + 1) * ktiles / p.split_parts;
  }
}

// Dynamic schedule bookkeeping in the workspace header: counter[0] hands out tiles,
// counter[1] counts CTAs that have finished. The last CTA to finish sets both back to
// zero, so the next launch on the same workspace starts from zero without a memset.
// Every CTA calls this once, after all of its roles are done with counter[0].
__device__ __forceinline__ void release_tile_counter(uint32_t* counter) {
  __threadfence();
  if (atomicAdd(&counter[1], 1u) == gridDim.x - 1) {
    __threadfence();
    atomicExch(&counter[0], 0u);
    atomicExch(&counter[1], 0u);
  }
}

// STREAMK: the instantiation that runs the stream-K schedule (p.stream_k_iters > 0); the
// others compile without its code (its epilogue hand-off cost the weight-streaming kernel
// 77 registers and ~4 % per call when it was always built in).
template <int MMA_N, bool GATED, int STAGES, bool DIRECT = false, bool STREAMK = false>
__global__ void __launch_bounds__(kNumThreads, 1)
    nvfp4_grouped_gemm_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = GemmConfig<MMA_N, GATED, STAGES, DIRECT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stage_base = smem;
  uint8_t* epi_base = smem + STAGES * Cfg::kStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_base + Cfg::kEpiBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;
  uint64_t* acce_bar = accf_bar + Cfg::kAccStages;
  uint64_t* drain_bar = acce_bar + Cfg::kAccStages;
  uint64_t* sched_full = drain_bar + 1;
  uint64_t* sched_empty = sched_full + kSchedSlots;
  uint64_t* split_arrive = sched_empty + kSchedSlots;  // epilogue warps wrote their partials
  uint64_t* split_result = split_arrive + 1;           // the leader published "last part"
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(split_result + 1);
  volatile uint32_t* abort_flag = tmem_holder + 1;
  volatile uint32_t* split_last = tmem_holder + 2;
  // Slot i: {unit, group, first k-tile, end k-tile}; a unit >= total_units ends the schedule.
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
    ptx::mbar_init(split_arrive, kEpilogueWarps);
    ptx::mbar_init(split_result, 1);
    *abort_flag = 0u;
    ptx::fence_mbarrier_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_holder, kTmemCols);
    ptx::tmem_relinquish_alloc_permit();
  }
  // Everything above is local to the CTA. Group records, tensor maps, operands and the
  // tile counter may come from the previous kernels in the stream: wait for them here,
  // then let the next launch be scheduled onto SMs as this grid's CTAs retire.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  stage_tile_ends(tile_ends, groups, p.num_groups);
  // Segment launches learn their tile count from the workspace (written by the segment
  // set-up kernel); the grid may then have CTAs without a tile, which end at once.
  const int total_tiles = p.seg_total_tiles != nullptr ? *p.seg_total_tiles : p.total_tiles;
  const int total_units = p.seg_total_tiles != nullptr ? total_tiles : p.total_units;
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
        ptx::tensormap_fence_acquire(&m[kMapA]);
        ptx::tensormap_fence_acquire(&m[kMapB]);
        if (GATED) ptx::tensormap_fence_acquire(&m[kMapB2]);
        if (DIRECT) ptx::tensormap_fence_acquire(&m[kMapA64]);
      };
      // Stream-K: whole tiles blockIdx.x, + grid, ... below stream_k_first_tile, then this
      // CTA's k-iterations [sk_pos, sk_end) of the stream-K tiles (tile sk_first + it / kt).
      const bool sk = STREAMK && p.stream_k_iters > 0;
      const int sk_first = sk ? p.stream_k_first_tile : 0;
      const int sk_kt = sk ? p.stream_k_ktiles : 1;
      int64_t sk_pos = sk ? static_cast<int64_t>(blockIdx.x) * p.stream_k_iters : 0;
      const int64_t sk_end =
          sk ? (sk_pos + p.stream_k_iters < p.stream_k_total_iters ? sk_pos + p.stream_k_iters
                                                                   : p.stream_k_total_iters)
             : 0;
      bool sk_whole = sk && static_cast<int>(blockIdx.x) < sk_first;  // in the round-robin part
      auto sk_unit = [&](int64_t it) -> int {
        return it < sk_end ? sk_first + static_cast<int>(it / sk_kt) : total_units;
      };
      int unit = !sk ? static_cast<int>(blockIdx.x)  // >= total_units only in segment launches
                     : (sk_whole ? static_cast<int>(blockIdx.x) : sk_unit(sk_pos));
      int tile, split;
      unit_tile(p, unit, tile, split);
      int g = advance_group(tile_ends, groups, p.num_groups, 0, tile);
      GroupDev gd = groups[g];
      int rb = seg_row(p, g);  // first row of the group's segment (0 outside segment launches)
      acquire_maps(g);
      for (uint32_t seq = 0;; ++seq) {
        // Publish this CTA's seq-th unit (or the end marker) to the MMA issuer and epilogue:
        // {unit, group, first k-tile, end k-tile}.
        const int slot = static_cast<int>(seq % kSchedSlots);
        if (!wait_phase(&sched_empty[slot], ((seq / kSchedSlots) & 1u) ^ 1u, abort_flag,
                        p.error_bits, kDevErrProducerTimeout))
          break;
        int k0 = 0, k1 = 0;
        if (unit < total_units) {
          if (sk && !sk_whole) {
            k0 = static_cast<int>(sk_pos - static_cast<int64_t>(unit - sk_first) * sk_kt);
            const int64_t left = sk_end - sk_pos;
            k1 = left < sk_kt - k0 ? k0 + static_cast<int>(left) : sk_kt;
          } else {
            unit_krange(p, split, gd.k / kBlockK, k0, k1);
          }
        }
        sched_info[4 * slot + 0] = unit;
        sched_info[4 * slot + 1] = g;
        sched_info[4 * slot + 2] = k0;
        sched_info[4 * slot + 3] = k1;
        ptx::mbar_arrive(&sched_full[slot]);
        if (unit >= total_units) break;
        const TmaDesc* maps = p.maps + static_cast<size_t>(g) * kMapsPerGroup;
        const int local = tile - gd.tile_start;
        const int mt = local % gd.tiles_m;
        const int nt = local / gd.tiles_m;
        const int ktiles = gd.k / kBlockK;
        const int rest_k = gd.k / 64;  // 4-scale column blocks along K
        const int rest_n = (gd.n + 127) / 128;
        // Scale-factor blocks of B for this tile (each 128 rows x 16 scales = 2 KiB per stage).
        const uint8_t* sfb_blk0;
        const uint8_t* sfb_blk1 = nullptr;
        if (GATED) {
          sfb_blk0 = gd.sfb + static_cast<size_t>(nt) * rest_k * kSfBlockBytes;
          sfb_blk1 = gd.sfb2 + static_cast<size_t>(nt) * rest_k * kSfBlockBytes;
        } else if (MMA_N == 256) {
          sfb_blk0 = gd.sfb + static_cast<size_t>(2 * nt) * rest_k * kSfBlockBytes;
          if (2 * nt + 1 < rest_n)
            sfb_blk1 = gd.sfb + static_cast<size_t>(2 * nt + 1) * rest_k * kSfBlockBytes;
        } else {
          sfb_blk0 = gd.sfb + static_cast<size_t>(nt) * rest_k * kSfBlockBytes;
        }
        const int row_a = rb + mt * kBlockM;
        const uint8_t* sfa_blk =
            gd.sfa + static_cast<size_t>(rb / kBlockM + mt) * rest_k * kSfBlockBytes;
        // Weight-streaming tiles of at most 64 rows load A through the 64-row box: rows
        // 64-127 of the stage's A tile then keep stale bytes, which only feed accumulator
        // rows that are never stored, and the TMA unit fills 8 KiB less per stage.
        const bool a_half = DIRECT && gd.m - mt * kBlockM <= 64;
        const uint32_t tx = (a_half ? Cfg::kABytes / 2 : Cfg::kABytes) + Cfg::kBBytes +
                            Cfg::kSfaBytes + (sfb_blk1 != nullptr ? 2 : 1) * 4 * kSfBlockBytes;
        // L2 warm-up of k-tile `kp` of this tile (A, B halves, scale blocks). In mode 1 only
        // operands that other CTAs also read are warmed (A when the group has several
        // n-tiles, B when it has several m-tiles): every prefetch box is TMA work, and on
        // weight-streaming shapes (one m-tile per group) warming unshared B only delayed
        // the loads behind it.
        const int tiles_n = (gd.tile_end - gd.tile_start) / gd.tiles_m;
        const bool warm_a =
            kL2PrefetchMode == 2 || (kL2PrefetchMode == 1 && nt == 0 && tiles_n > 1);
        const bool warm_b =
            kL2PrefetchMode == 2 || (kL2PrefetchMode == 1 && mt == 0 && gd.tiles_m > 1);
        auto prefetch_ktile = [&](int kp) {
          const int px = kp * kRowBytesPerStage;
          const size_t psf = static_cast<size_t>(kp) * 4 * kSfBlockBytes;
          if (warm_a) {
            ptx::tma_prefetch_l2_2d(&maps[kMapA], px, row_a);
            ptx::bulk_prefetch_l2(sfa_blk + psf, 4 * kSfBlockBytes);
          }
          if (warm_b) {
            if (GATED) {
              ptx::tma_prefetch_l2_2d(&maps[kMapB], px, nt * 128);
              ptx::tma_prefetch_l2_2d(&maps[kMapB2], px, nt * 128);
            } else if (MMA_N == 256) {
              ptx::tma_prefetch_l2_2d(&maps[kMapB], px, nt * 256);
              ptx::tma_prefetch_l2_2d(&maps[kMapB], px, nt * 256 + 128);
            } else {
              ptx::tma_prefetch_l2_2d(&maps[kMapB], px, nt * 128);
            }
            ptx::bulk_prefetch_l2(sfb_blk0 + psf, 4 * kSfBlockBytes);
            if (sfb_blk1 != nullptr) ptx::bulk_prefetch_l2(sfb_blk1 + psf, 4 * kSfBlockBytes);
          }
        };
        const int claim_kt = k1 - k0 > kClaimLeadKTiles ? k1 - kClaimLeadKTiles : k0;
        int next_unit = total_units;
        int next_tile = total_tiles, next_split = -1;
        int g_next = g;
        GroupDev next_gd = gd;
        int next_rb = rb;
        bool resolved = false;
        auto claim_next = [&]() -> int {
          if (sk) {
            if (sk_whole) {
              const int nu = unit + static_cast<int>(gridDim.x);
              return nu < sk_first ? nu : sk_unit(sk_pos);
            }
            return sk_unit(sk_pos + (k1 - k0));
          }
          if (p.dynamic_schedule)
            return static_cast<int>(gridDim.x + atomicAdd(p.tile_counter, 1u));
          return unit + static_cast<int>(gridDim.x);
        };
        auto resolve_next = [&]() {
          resolved = true;
          if (next_unit >= total_units) return;
          unit_tile(p, next_unit, next_tile, next_split);
          g_next = advance_group(tile_ends, groups, p.num_groups, g, next_tile);
          next_gd = groups[g_next];
          next_rb = seg_row(p, g_next);
          if (g_next != g) acquire_maps(g_next);
        };
        (void)ktiles;
        for (int kt = k0; kt < k1; ++kt) {
          if ((warm_a || warm_b) && kt > k0 && kt + kL2PrefetchKTiles < k1)
            prefetch_ktile(kt + kL2PrefetchKTiles);
          if (!wait_phase(&empty_bar[stage], phase ^ 1u, abort_flag, p.error_bits,
                          kDevErrProducerTimeout)) {
            ok = false;
            break;
          }
          uint8_t* sA = stage_base + stage * Cfg::kStageBytes;
          uint8_t* sB = sA + Cfg::kABytes;
          uint8_t* sSFA = sB + Cfg::kBBytes;
          uint8_t* sSFB = sSFA + Cfg::kSfaBytes;
          ptx::mbar_arrive_expect_tx(&full_bar[stage], tx);
          const int kx = kt * kRowBytesPerStage;
          ptx::tma_load_2d(sA, &maps[a_half ? kMapA64 : kMapA], &full_bar[stage], kx, row_a);
          if (GATED) {
            ptx::tma_load_2d(sB, &maps[kMapB], &full_bar[stage], kx, nt * 128);
            ptx::tma_load_2d(sB + 128 * kRowBytesPerStage, &maps[kMapB2], &full_bar[stage], kx,
                             nt * 128);
          } else if (MMA_N == 256) {
            ptx::tma_load_2d(sB, &maps[kMapB], &full_bar[stage], kx, nt * 256);
            ptx::tma_load_2d(sB + 128 * kRowBytesPerStage, &maps[kMapB], &full_bar[stage], kx,
                             nt * 256 + 128);
          } else {
            ptx::tma_load_2d(sB, &maps[kMapB], &full_bar[stage], kx, nt * 128);
          }
          const size_t sf_off = static_cast<size_t>(kt) * 4 * kSfBlockBytes;
          ptx::bulk_load(sSFA, sfa_blk + sf_off, 4 * kSfBlockBytes, &full_bar[stage]);
          ptx::bulk_load(sSFB, sfb_blk0 + sf_off, 4 * kSfBlockBytes, &full_bar[stage]);
          if (sfb_blk1 != nullptr)
            ptx::bulk_load(sSFB + 4 * kSfBlockBytes, sfb_blk1 + sf_off, 4 * kSfBlockBytes,
                           &full_bar[stage]);
          // The first warm-up prefetches go behind the tile's first loads, which would
          // otherwise wait for the TMA unit to work through them.
          if (kt == k0 && (warm_a || warm_b))
            for (int kp = k0 + 1; kp <= k0 + kL2PrefetchKTiles && kp < k1; ++kp) prefetch_ktile(kp);
          // Claim the next tile a few k-tiles before the end of this one; one k-tile
          // later (the claim's atomic has returned by then) look up its group, load its
          // record and acquire its tensor maps (about a microsecond per group switch),
          // all behind loads already in flight.
          if (kt == claim_kt) next_unit = claim_next();
          if (kt == claim_kt + 1) resolve_next();
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (!resolved) resolve_next();
        if (sk_whole) {
          if (unit + static_cast<int>(gridDim.x) >= sk_first) sk_whole = false;
        } else {
          sk_pos += k1 - k0;
        }
        unit = next_unit;
        tile = next_tile;
        split = next_split;
        g = g_next;
        gd = next_gd;
        rb = next_rb;
      }
      // Make sure no copy into this CTA's shared memory is still in flight at exit:
      // wait for the most recent fill of every stage (already complete on the normal path).
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
      // Parity to wait for on acce_bar[s] before tile t (stage s = t & 1) may write its
      // accumulator. Overlapped stages: tile t needs tile t-1's shared box drained
      // (arrived on acce_bar[t & 1] by the epilogue of tile t-1); the first tile passes.
      // Plain double buffer: tile t needs tile t-2 drained; the first two tiles pass.
      uint32_t acc_parity = Cfg::kOverlapAcc ? 0x1u : 0x3u;  // bit s: parity for stage s
      bool ok = p.diag_skip_mma == 0;
      for (uint32_t local = 0; ok; ++local) {
        // This CTA's local-th tile, as published by the producer.
        const int slot = static_cast<int>(local % kSchedSlots);
        if (!wait_phase(&sched_full[slot], (local / kSchedSlots) & 1u, abort_flag, p.error_bits,
                        kDevErrMmaTimeout))
          break;
        const int unit = sched_info[4 * slot + 0];
        const int ktiles = sched_info[4 * slot + 3] - sched_info[4 * slot + 2];  // this unit's
        ptx::mbar_arrive(&sched_empty[slot]);
        if (unit >= total_units) break;
        const int acc = static_cast<int>(local & 1u);
        if (!wait_phase(&acce_bar[acc], (acc_parity >> acc) & 1u, abort_flag, p.error_bits,
                        kDevErrAccTimeout)) {
          break;
        }
        acc_parity ^= 1u << acc;
        ptx::tcgen05_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccStride;
        for (int kt = 0; kt < ktiles; ++kt) {
          if (!wait_phase(&full_bar[stage], phase, abort_flag, p.error_bits, kDevErrMmaTimeout)) {
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
          // Scale factors: each 512-byte block (128 rows x 4 scales) becomes 4 TMEM
          // columns, replicated to all four lane quarters.
#pragma unroll
          for (int kb = 0; kb < 4; ++kb)
            ptx::tmem_cp_32x128b_warpx4(sfa_t + 4 * kb,
                                        ptx::make_sf_block_desc(sSFA + kb * kSfBlockBytes));
#pragma unroll
          for (int j = 0; j < Cfg::kSfbBlocks; ++j) {
#pragma unroll
            for (int kb = 0; kb < 4; ++kb)
              ptx::tmem_cp_32x128b_warpx4(
                  sfb_t + Cfg::kSfbColsPerMma * kb + 4 * j,
                  ptx::make_sf_block_desc(sSFB + j * 4 * kSfBlockBytes + kb * kSfBlockBytes));
          }
          const uint64_t a_desc = ptx::make_sw128_kmajor_desc(sA);
          const uint64_t b_desc = ptx::make_sw128_kmajor_desc(sB);
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            // 64 e2m1 values = 32 bytes along K inside the 128-byte swizzle row.
            ptx::mma_mxf4nvf4(d_tmem, a_desc + 2 * kb, b_desc + 2 * kb, Cfg::kIdesc,
                              sfa_t + 4 * kb, sfb_t + Cfg::kSfbColsPerMma * kb,
                              (kt | kb) != 0 ? 1u : 0u);
          }
          ptx::tcgen05_commit(&empty_bar[stage]);  // frees the smem stage when the MMAs finish
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::tcgen05_commit(&accf_bar[acc]);  // accumulator complete -> epilogue
      }
      // Wait for every MMA / TMEM copy this thread issued before TMEM is freed.
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
    const int ew = warp - kEpilogueWarp0;   // 0..3
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    uint8_t* my_bufs = epi_base + ew * Cfg::kEpiBufsPerWarp * Cfg::kEpiBufBytes;
    const uint32_t my_bufs_s = ptx::smem_u32(my_bufs);
    uint32_t full_parity = 0;  // bit s: parity to wait for on accf_bar[s]
    uint32_t stores = 0;
    uint32_t split_count = 0;  // split-tile parts this CTA has handled (rendezvous parity)
    int acquired_g = -1;
    constexpr int kBoxes = Cfg::kOutN / 64;
    for (uint32_t local = 0;; ++local) {
      // This CTA's local-th tile, as published by the producer.
      const int slot = static_cast<int>(local % kSchedSlots);
      if (!warp_wait_phase(&sched_full[slot], (local / kSchedSlots) & 1u, abort_flag,
                           p.error_bits, kDevErrEpilogueTimeout, lane))
        break;
      const int unit = sched_info[4 * slot + 0];
      const int g = sched_info[4 * slot + 1];
      const int piece_k0 = sched_info[4 * slot + 2];
      const int piece_k1 = sched_info[4 * slot + 3];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&sched_empty[slot]);
      if (unit >= total_units) break;
      int tile, split;
      unit_tile(p, unit, tile, split);
      const GroupDev gd = groups[g];
      const int rb = seg_row(p, g);  // C rows of the group start here
      const TmaDesc* map_c = p.maps + static_cast<size_t>(g) * kMapsPerGroup + kMapC;
      if (!DIRECT && split < 0 && g != acquired_g) {
        if (lane == 0) ptx::tensormap_fence_acquire(map_c);
        acquired_g = g;
      }
      const int acc = static_cast<int>(local & 1u);
      // The group record's load is in flight while the accumulator is awaited.
      if (!warp_wait_phase(&accf_bar[acc], (full_parity >> acc) & 1u, abort_flag, p.error_bits,
                           kDevErrEpilogueTimeout, lane)) {
        break;
      }
      full_parity ^= 1u << acc;
      ptx::tcgen05_fence_after_sync();
      const int tl = tile - gd.tile_start;
      const int mt = tl % gd.tiles_m;
      const int nt = tl / gd.tiles_m;
      // Which barrier hands this accumulator (or its shared box) back to the MMA issuer.
      uint64_t* release_bar = Cfg::kOverlapAcc ? &acce_bar[acc ^ 1] : &acce_bar[acc];
      // With overlapped stages the box holding TMEM columns [192, 256) goes first:
      // stage 0 -> its last box (up-projection half of box 1 when gated), stage 1 -> box 0.
      const int first_box = (Cfg::kOverlapAcc && acc == 0) ? kBoxes - 1 : 0;
      const int row0 = mt * kBlockM + 32 * quarter;
      const int row = row0 + lane;
      // Split units write their fp32 partial rows here (slot = part of a split tile).
      float* part_row = nullptr;
      if (split >= 0)
        part_row = p.split_partials +
                   (static_cast<size_t>((tile - p.split_first_tile) * p.split_parts + split) *
                        kBlockM + 32 * quarter + lane) * MMA_N;
      // Convert one 64-column box (accumulator bits v0/v1, up-projection bits u0/u1 when
      // gated) to fp16 and store it: straight from registers (DIRECT, and the final sum of
      // split tiles) or through the swizzled staging box and a TMA store.
      // Where this thread's row goes when stored from registers (or, for a scattered output,
      // from the staged box): its C row, or the row it maps to (nullptr: not stored).
      const bool scatter = !GATED && p.row_dest != nullptr;
      uint8_t* out_row = nullptr;
      if (row < gd.m)
        out_row = scatter ? scatter_row(p, static_cast<int64_t>(rb) + row)
                          : gd.c + static_cast<size_t>(rb + row) * gd.n * sizeof(__half);
      auto emit_box = [&](const uint32_t* v0, const uint32_t* v1, const uint32_t* u0,
                          const uint32_t* u1, int box, bool direct) {
        if (GATED && p.out_sf != nullptr) {
          // NVFP4 output (codes and blocked scales; no fp16 staging).
          if (row < gd.m) {
            const int col0 = nt * Cfg::kOutN + box * 64;
            const int64_t r = static_cast<int64_t>(rb) + row;
            store_gated_box_nvfp4(v0, v1, u0, u1, gd.alpha, gd.alpha2, p.out_scale, p.out_d6,
                                  gd.c + r * (gd.n / 2) + col0 / 2,
                                  p.out_sf + blocked_sf_offset(r, col0 / 16, (gd.n + 63) / 64));
          }
          return;
        }
        const uint32_t buf = my_bufs_s + (stores & 1u) * Cfg::kEpiBufBytes;
        if (!direct) {
          // The store that last read this staging buffer (two boxes ago) must be done with it.
          if (lane == 0) ptx::bulk_wait_group_read<1>();
          __syncwarp();
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t* v = half ? v1 : v0;
          uint32_t packed[16];
          if (GATED) {
            const uint32_t* u = half ? u1 : u0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              __half2 hv = __floats2half2_rn(gated_value(v[2 * i], u[2 * i], gd.alpha, gd.alpha2),
                                             gated_value(v[2 * i + 1], u[2 * i + 1], gd.alpha,
                                                         gd.alpha2));
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
          if (direct) {
            // Row row0 + lane, columns [col, col + 32): four 16-byte stores (N is a
            // multiple of 8, so a chunk is either inside the row or past its end).
            const int col = nt * Cfg::kOutN + box * 64 + half * 32;
            if (out_row != nullptr) {
              // The local row, then each replica of it (replicas only without scattering).
              for (int r = -1; r < (scatter ? 0 : p.num_replicas); ++r) {
                uint4* dst = reinterpret_cast<uint4*>(
                    out_row + (r < 0 ? 0 : p.replica_offset[r]) +
                    static_cast<size_t>(col) * sizeof(__half));
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  if (col + 8 * c < gd.n)
                    dst[c] = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                                        packed[4 * c + 3]);
              }
            }
          } else {
            // Row `lane` of the 32 x 128 B box, 16-byte chunks XOR-swizzled by (row & 7)
            // to match the map's 128B swizzle (and to spread the stores over all banks).
            const uint32_t row_addr = buf + lane * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t chunk = static_cast<uint32_t>(half * 4 + c) ^ (lane & 7);
              ptx::st_shared_v4(row_addr + chunk * 16, packed[4 * c], packed[4 * c + 1],
                                packed[4 * c + 2], packed[4 * c + 3]);
            }
          }
        }
        if (!direct && scatter) {
          __syncwarp();
          store_box_rows(my_bufs + (stores & 1u) * Cfg::kEpiBufBytes, out_row,
                         nt * Cfg::kOutN + box * 64, gd.n, lane);
          __syncwarp();  // the box is read before it is written again
          ++stores;
        } else if (!direct) {
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d(map_c, my_bufs + (stores & 1u) * Cfg::kEpiBufBytes,
                              nt * Cfg::kOutN + box * 64, rb + row0);
            ptx::bulk_commit_group();
          }
          // Replicas: the same staged box, four 128-byte row pieces per warp store (whole
          // lines over NVLink), while the TMA store writes the local copy.
          for (int r = 0; r < p.num_replicas; ++r)
            store_box_rows(my_bufs + (stores & 1u) * Cfg::kEpiBufBytes,
                           out_row != nullptr ? out_row + p.replica_offset[r] : nullptr,
                           nt * Cfg::kOutN + box * 64, gd.n, lane);
          ++stores;
        }
      };
      bool released = false;
      // Stream-K piece of a tile cut by the range boundary of CTA sk_b (its later k-tiles
      // are this CTA's first piece, its first k-tiles the previous CTA's last piece). Per
      // warp quarter, the piece that counts in first (arrivals in the counter's low byte)
      // stores its fp32 rows to slot sk_b and then publishes them (kSkPublished, set with
      // atomicOr so that no arrival can carry into it); the other waits for that bit, adds the
      // stored rows to its own (a two-term fp32 sum: the same bits whichever piece comes
      // second) and stores C.
      int sk_role = 0;  // 0: whole tile; 1: store the partial rows; 2: add them and store C
      int32_t* sk_ctr = nullptr;
      const float* sk_src = nullptr;
      float* sk_dst = nullptr;
      if (STREAMK && !GATED && p.stream_k_iters > 0 && row0 < gd.m &&
          (piece_k0 > 0 || piece_k1 < gd.k / kBlockK)) {
        const int sk_b = piece_k0 > 0 ? static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x) + 1;
        sk_ctr = p.split_counters + 4 * sk_b + quarter;
        int old = 0;
        if (lane == 0) old = atomicAdd(sk_ctr, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        sk_role = (old & 0xff) == 0 ? 1 : 2;
        sk_dst = p.split_partials +
                 (static_cast<size_t>(sk_b) * kBlockM + 32 * quarter + lane) * MMA_N;
        sk_src = sk_dst;
        if (sk_role == 2) {
          int ready = 1;
          if (lane == 0)
            ready = wait_global_bit(sk_ctr, kSkPublished, abort_flag, p.error_bits,
                                    kDevErrEpilogueTimeout)
                        ? 1 : 0;
          ready = __shfl_sync(0xffffffffu, ready, 0);
          if (!ready) break;
          __threadfence();
        }
      }
      if (row0 < gd.m) {
        const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(32 * quarter) << 16) +
                               acc * Cfg::kAccStride;
#pragma unroll 1
        for (int bi = 0; bi < kBoxes; ++bi) {
          const int box = (first_box + bi) % kBoxes;
          // 64 output columns: issue every TMEM load of the box, then wait once.
          uint32_t v0[32], v1[32];
          ptx::tmem_ld_32x32b_x32(t_acc + box * 64, v0);
          ptx::tmem_ld_32x32b_x32(t_acc + box * 64 + 32, v1);
          uint32_t u0[32], u1[32];
          if (GATED) {
            ptx::tmem_ld_32x32b_x32(t_acc + 128 + box * 64, u0);
            ptx::tmem_ld_32x32b_x32(t_acc + 128 + box * 64 + 32, u1);
          }
          ptx::tmem_ld_wait();
          if (Cfg::kOverlapAcc ? bi == 0 : bi == kBoxes - 1) {
            ptx::tcgen05_fence_before_sync();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(release_bar);
            released = true;
          }
          if (split >= 0) {
            // A part of a split tile: its fp32 sums go to the tile's partial slot.
            float4* dv = reinterpret_cast<float4*>(part_row + box * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              dv[c] = make_float4(__uint_as_float(v0[4 * c]), __uint_as_float(v0[4 * c + 1]),
                                  __uint_as_float(v0[4 * c + 2]), __uint_as_float(v0[4 * c + 3]));
              dv[8 + c] = make_float4(__uint_as_float(v1[4 * c]), __uint_as_float(v1[4 * c + 1]),
                                      __uint_as_float(v1[4 * c + 2]), __uint_as_float(v1[4 * c + 3]));
            }
            if (GATED) {
              float4* du = reinterpret_cast<float4*>(part_row + 128 + box * 64);
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                du[c] = make_float4(__uint_as_float(u0[4 * c]), __uint_as_float(u0[4 * c + 1]),
                                    __uint_as_float(u0[4 * c + 2]), __uint_as_float(u0[4 * c + 3]));
                du[8 + c] = make_float4(__uint_as_float(u1[4 * c]), __uint_as_float(u1[4 * c + 1]),
                                        __uint_as_float(u1[4 * c + 2]), __uint_as_float(u1[4 * c + 3]));
              }
            }
            continue;
          }
          if (sk_role == 1) {
            // First piece of a cut tile: its fp32 rows go to the boundary's slot.
            if (row < gd.m) {
              float4* dv = reinterpret_cast<float4*>(sk_dst + box * 64);
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                dv[c] = make_float4(__uint_as_float(v0[4 * c]), __uint_as_float(v0[4 * c + 1]),
                                    __uint_as_float(v0[4 * c + 2]), __uint_as_float(v0[4 * c + 3]));
                dv[8 + c] = make_float4(__uint_as_float(v1[4 * c]), __uint_as_float(v1[4 * c + 1]),
                                        __uint_as_float(v1[4 * c + 2]), __uint_as_float(v1[4 * c + 3]));
              }
            }
            continue;
          }
          if (sk_role == 2 && row < gd.m) {
            // Second piece: add the stored rows (written by another SM: read through L2).
            const float4* sv = reinterpret_cast<const float4*>(sk_src + box * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const float4 f = __ldcg(sv + c);
              v0[4 * c] = __float_as_uint(__uint_as_float(v0[4 * c]) + f.x);
              v0[4 * c + 1] = __float_as_uint(__uint_as_float(v0[4 * c + 1]) + f.y);
              v0[4 * c + 2] = __float_as_uint(__uint_as_float(v0[4 * c + 2]) + f.z);
              v0[4 * c + 3] = __float_as_uint(__uint_as_float(v0[4 * c + 3]) + f.w);
              const float4 h = __ldcg(sv + 8 + c);
              v1[4 * c] = __float_as_uint(__uint_as_float(v1[4 * c]) + h.x);
              v1[4 * c + 1] = __float_as_uint(__uint_as_float(v1[4 * c + 1]) + h.y);
              v1[4 * c + 2] = __float_as_uint(__uint_as_float(v1[4 * c + 2]) + h.z);
              v1[4 * c + 3] = __float_as_uint(__uint_as_float(v1[4 * c + 3]) + h.w);
            }
          }
          emit_box(v0, v1, u0, u1, box, DIRECT);
        }
        if (sk_role == 1) {
          // Publish the stored rows to the other piece's warp.
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicOr(sk_ctr, kSkPublished);
        } else if (sk_role == 2) {
          __syncwarp();
          if (lane == 0) atomicExch(sk_ctr, 0);  // 0 again for the next launch
        }
      }
      if (!released) {
        ptx::tcgen05_fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(release_bar);
      }
      if (split >= 0) {
        // Rendezvous of the four epilogue warps (bounded waits), then one thread counts this
        // part in; the part that arrives last sums all parts in split order (so the result
        // does not depend on arrival order), writes C and resets the counter. No CTA ever
        // waits for another CTA.
        const uint32_t par = split_count & 1u;
        ++split_count;
        __threadfence();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(split_arrive);
        if (ew == 0 && lane == 0) {
          uint32_t last = 0;
          if (wait_phase(split_arrive, par, abort_flag, p.error_bits, kDevErrEpilogueTimeout)) {
            __threadfence();
            int32_t* counter = p.split_counters + (tile - p.split_first_tile);
            last = atomicAdd(counter, 1) == p.split_parts - 1 ? 1u : 0u;
            if (last) {
              __threadfence();
              *counter = 0;
            }
          }
          *split_last = last;
          ptx::mbar_arrive(split_result);
        }
        if (!warp_wait_phase(split_result, par, abort_flag, p.error_bits, kDevErrEpilogueTimeout,
                             lane))
          break;
        if (*split_last && row0 < gd.m) {
          __threadfence();
          const float* base = p.split_partials +
                              (static_cast<size_t>((tile - p.split_first_tile) * p.split_parts) *
                                   kBlockM + 32 * quarter + lane) * MMA_N;
          const size_t part_stride = static_cast<size_t>(kBlockM) * MMA_N;
#pragma unroll 1
          for (int box = 0; box < kBoxes; ++box) {
            uint32_t v0[32], v1[32], u0[32], u1[32];
            float sv[64], su[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) sv[i] = su[i] = 0.0f;
#pragma unroll 1
            for (int sp = 0; sp < p.split_parts; ++sp) {
              const float4* src = reinterpret_cast<const float4*>(base + sp * part_stride + box * 64);
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const float4 f = __ldcg(src + c);  // written by other SMs: read through L2
                sv[4 * c] += f.x;
                sv[4 * c + 1] += f.y;
                sv[4 * c + 2] += f.z;
                sv[4 * c + 3] += f.w;
              }
              if (GATED) {
                const float4* srcu =
                    reinterpret_cast<const float4*>(base + sp * part_stride + 128 + box * 64);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                  const float4 f = __ldcg(srcu + c);
                  su[4 * c] += f.x;
                  su[4 * c + 1] += f.y;
                  su[4 * c + 2] += f.z;
                  su[4 * c + 3] += f.w;
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v0[i] = __float_as_uint(sv[i]);
              v1[i] = __float_as_uint(sv[32 + i]);
              u0[i] = __float_as_uint(su[i]);
              u1[i] = __float_as_uint(su[32 + i]);
            }
            emit_box(v0, v1, u0, u1, box, true);
          }
        }
      }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

  ptx::tcgen05_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    ptx::tcgen05_fence_after_sync();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && p.dynamic_schedule) release_tile_counter(p.tile_counter);
}

}  // namespace nvfp4
