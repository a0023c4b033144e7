// Expert-parallel MoE exchange over NVLink peer memory (one process per GPU, up to
// kEpMaxRanks ranks; rank p owns experts [p * E/P, (p + 1) * E/P)).
//
// Every buffer named "peer" is one allocation that exists on every rank at the same size
// (symmetric memory or CUDA IPC), seen here through the address each rank's copy has in
// this process. Steps, with a cross-rank barrier where marked (|):
//
//   publish counts:  rank q writes its per-expert pair counts into row q of every rank's
//                    [P, E] count matrix                                             |
//   layout:          every rank derives, from the same matrix, each owner's 128-row-aligned
//                    expert segments (rows from rank 0 first, then rank 1, ...) and where
//                    its own rows for each expert start in the owner's receive slab
//   dispatch:        rank q writes each routed token row (NVFP4 codes + plain scale row)
//                    straight into the owner's receive slab, and the row's return address
//                    (q << 40 | pair index) into the owner's recv_meta                |
//   (owner: scales plain -> blocked, expert GEMMs over its segments; the down GEMM's
//    epilogue stores every output row into its token's rank's return buffer)        |
//   combine:         rank q sums its pairs' returned rows (local reads)
//
// Or, with owner-side sums (return_sums): after dispatch rank q also publishes, into every
// owner's [P, tokens * topk] pair tables, each pair's slab row there (-1 when the pair went
// elsewhere) and its routing weight; the owner's down GEMM writes its rows locally, and
// return_sums adds each source token's rows of this owner (slot order, fp32) and stores one
// fp16 row per (token, owner) into the token's rank                                 |
//   combine_sums:    rank q adds its tokens' per-owner rows in owner order (local reads)
// A token whose slots meet on one owner then sends one row back instead of one per slot.
//
// The kernels only load and store: no kernel waits on another rank, so the barriers (a
// one-element NCCL all-reduce on the same stream) carry all cross-rank ordering.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "row_ops.cuh"
#include "nvfp4_quant_math.cuh"

namespace nvfp4 {

constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxExperts = 1024;

struct EpPeers {
  void* ptr[kEpMaxRanks];
};

// Device error bit of the exchange: a segment would not fit the owner's receive slab (its
// rows are dropped, consistently on every rank).
constexpr uint32_t kEpErrCapacity = 1u << 0;

// counts[e] (this rank's pairs routed to expert e) -> row `rank` of every rank's matrix.
__global__ void __launch_bounds__(256) nvfp4_ep_publish_counts_kernel(
    const int32_t* __restrict__ counts, int num_experts, int rank, int world, EpPeers mats) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < world * num_experts;
       i += gridDim.x * blockDim.x) {
    const int p = i / num_experts;
    const int e = i % num_experts;
    static_cast<int32_t*>(mats.ptr[p])[static_cast<int64_t>(rank) * num_experts + e] = counts[e];
  }
  __threadfence_system();
}

// One block. mat [world, E]: pairs of each source rank per expert (this rank's copy).
// Outputs for this rank as owner: seg_offsets/seg_counts [E/world] (its local experts'
// segments in its receive slab); as source: send_base[E] (first row of this rank's pairs
// for expert e in the owner's slab, -1 when the owner's slab cannot hold the segment).
__global__ void __launch_bounds__(1024) nvfp4_ep_layout_kernel(
    const int32_t* __restrict__ mat, int num_experts, int rank, int world, int64_t capacity,
    int32_t* __restrict__ seg_offsets, int32_t* __restrict__ seg_counts,
    int32_t* __restrict__ send_base, uint32_t* error_word) {
  __shared__ int32_t total[kEpMaxExperts];   // pairs per expert over all sources
  __shared__ int64_t start[kEpMaxExperts];   // segment start in the owner's slab
  const int epr = num_experts / world;
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) {
    int32_t t = 0;
    for (int q = 0; q < world; ++q) t += mat[q * num_experts + e];
    total[e] = t;
  }
  __syncthreads();
  if (threadIdx.x < world) {  // one thread per owner: scan its experts' padded segments
    const int p = threadIdx.x;
    int64_t acc = 0;
    for (int l = 0; l < epr; ++l) {
      const int e = p * epr + l;
      start[e] = acc;
      acc += (static_cast<int64_t>(total[e]) + 127) / 128 * 128;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) {
    const bool fits = start[e] + total[e] <= capacity;
    if (!fits) atomicOr(error_word, kEpErrCapacity);
    int64_t before = 0;  // pairs of lower source ranks in this segment
    for (int q = 0; q < rank; ++q) before += mat[q * num_experts + e];
    send_base[e] = fits ? static_cast<int32_t>(start[e] + before) : -1;
    if (e / epr == rank) {
      const int l = e - rank * epr;
      seg_offsets[l] = fits ? static_cast<int32_t>(start[e]) : 0;
      seg_counts[l] = fits ? total[e] : 0;
    }
  }
}

// Return address of a received row: the source rank and the pair's index there.
constexpr int kEpRankShift = 40;
constexpr int64_t kEpPairMask = (int64_t{1} << kEpRankShift) - 1;

// One warp per (token, slot) pair. The pair's row in the local dispatched order is dest[i]
// (its rank within expert e is dest[i] - offsets[e]); its row in the owner's slab is
// send_base[e] + that rank. Copies the token's codes (cols/2 bytes) and its scales as a plain
// row (cols/16 bytes, gathered from the blocked layout) into the owner's slabs, writes the
// row's return address (rank << 40 | i) into the owner's recv_meta, and records the row in
// remote_rows[i] (-1 for dropped pairs).
__global__ void __launch_bounds__(256) nvfp4_ep_dispatch_kernel(
    const int32_t* __restrict__ ids, int64_t pairs, int topk, int num_experts, int rank,
    int world, const int32_t* __restrict__ dest, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ send_base, const uint8_t* __restrict__ codes, int64_t ld_codes,
    const uint8_t* __restrict__ sf_blocked, int cols, EpPeers recv_codes, EpPeers recv_sf,
    EpPeers recv_meta, int64_t capacity, int32_t* __restrict__ remote_rows) {
  const int lane = threadIdx.x & 31;
  const int epr = num_experts / world;
  const int code_chunks = cols / 32;   // 16-byte chunks of a codes row
  const int sf_chunks = cols / 256;    // 16-byte chunks of a plain scale row
  const int rest_k = cols / 64;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t i = warp0; i < pairs; i += nwarps) {
    const int e = ids[i];
    const int32_t d = dest[i];
    int64_t row = -1;
    if (e >= 0 && e < num_experts && d >= 0 && send_base[e] >= 0) {
      row = static_cast<int64_t>(send_base[e]) + (d - offsets[e]);
      if (row >= capacity) row = -1;  // cannot happen when the layout fitted; never write past
    }
    if (lane == 0) remote_rows[i] = static_cast<int32_t>(row);
    if (row < 0) continue;
    const int p = e / epr;
    if (lane == 0)
      static_cast<int64_t*>(recv_meta.ptr[p])[row] = (static_cast<int64_t>(rank) << kEpRankShift) | i;
    const int64_t t = i / topk;
    const uint4* src = reinterpret_cast<const uint4*>(codes + t * ld_codes);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(recv_codes.ptr[p]) +
                                          row * (cols / 2));
    copy_row_chunks(src, dst, code_chunks, lane);
    uint4* sdst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(recv_sf.ptr[p]) +
                                           row * (cols / 16));
    for (int c = lane; c < sf_chunks; c += 32) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w[j] = __ldg(reinterpret_cast<const uint32_t*>(
            sf_blocked + blocked_sf_offset(t, 16 * c + 4 * j, rest_k)));
      sdst[c] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  __threadfence_system();
}

// out[t, :] = bf16( sum_j w[t, j] * ret[t*topk + j, :] ) over the pairs that were kept
// (remote_rows >= 0), fp32 products and sums in slot order (the single-GPU combine's
// arithmetic, combine_slots). ret holds each pair's expert output row, returned by its
// owner's down GEMM. One warp per (token, 256-column chunk), 16-byte loads.
__global__ void __launch_bounds__(256) nvfp4_ep_combine_kernel(
    const int32_t* __restrict__ remote_rows, const float* __restrict__ weights, int tokens,
    int topk, const __half* __restrict__ ret, int cols, __nv_bfloat16* __restrict__ out,
    int64_t ldo) {
  const int lane = threadIdx.x & 31;
  const int chunks = (cols + 255) / 256;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t task = warp0; task < static_cast<int64_t>(tokens) * chunks; task += nwarps) {
    const int64_t t = task / chunks;
    const int col = static_cast<int>(task % chunks) * 256 + lane * 8;
    const bool active = col < cols;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    combine_slots(t, topk, col, active, ret, cols, weights,
                  [&](int64_t i) -> int64_t { return __ldg(remote_rows + i) < 0 ? -1 : i; }, acc);
    if (active) store_bf16x8(out + t * ldo + col, acc);
  }
}

// ---- owner-side sums -----------------------------------------------------------------------
// Pair tables (one [world, pairs] int32 and one [world, pairs] fp32 array on every rank, pairs
// = tokens * topk, the same on every rank): row q holds source rank q's pairs. Token slabs
// ([world, tokens] rows of codes and of plain scales on every rank): row q * tokens + t holds
// source rank q's token t.

// One warp per token t of this rank: each slot's row in its owner's slab (remote_rows[i], the
// row nvfp4_ep_dispatch gives pair i; -1 when dropped), then the token's codes (cols/2 bytes)
// and its scales as a plain row (cols/16 bytes) once into each owner that holds a kept pair of
// t, at token-slab row rank * tokens + t: a token whose slots meet on one owner crosses
// NVLink once. The owner places the rows with nvfp4_ep_expand.
__global__ void __launch_bounds__(256) nvfp4_ep_dispatch_tokens_kernel(
    const int32_t* __restrict__ ids, int tokens, int topk, int num_experts, int rank, int world,
    const int32_t* __restrict__ dest, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ send_base, const uint8_t* __restrict__ codes, int64_t ld_codes,
    const uint8_t* __restrict__ sf_blocked, int cols, EpPeers tok_codes, EpPeers tok_sf,
    int64_t capacity, int32_t* __restrict__ remote_rows) {
  const int lane = threadIdx.x & 31;
  const int epr = num_experts / world;
  const int code_chunks = cols / 32;
  const int sf_chunks = cols / 256;
  const int rest_k = cols / 64;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = warp0; t < tokens; t += nwarps) {
    uint32_t owners = 0;
    for (int j0 = 0; j0 < topk; j0 += 32) {
      const int j = j0 + lane;
      int owner = -1;
      if (j < topk) {
        const int64_t i = t * topk + j;
        const int e = ids[i];
        const int32_t d = dest[i];
        int64_t row = -1;
        if (e >= 0 && e < num_experts && d >= 0 && send_base[e] >= 0) {
          row = static_cast<int64_t>(send_base[e]) + (d - offsets[e]);
          if (row >= capacity) row = -1;
        }
        remote_rows[i] = static_cast<int32_t>(row);
        if (row >= 0) owner = e / epr;
      }
      for (int p = 0; p < world; ++p)
        if (__ballot_sync(0xffffffffu, owner == p)) owners |= 1u << p;
    }
    const int64_t slab_row = static_cast<int64_t>(rank) * tokens + t;
    const uint4* src = reinterpret_cast<const uint4*>(codes + t * ld_codes);
    for (int p = 0; p < world; ++p) {
      if (!((owners >> p) & 1u)) continue;
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(tok_codes.ptr[p]) +
                                            slab_row * (cols / 2));
      copy_row_chunks(src, dst, code_chunks, lane);
      uint4* sdst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(tok_sf.ptr[p]) +
                                             slab_row * (cols / 16));
      for (int c = lane; c < sf_chunks; c += 32) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          w[k] = __ldg(reinterpret_cast<const uint32_t*>(
              sf_blocked + blocked_sf_offset(t, 16 * c + 4 * k, rest_k)));
        sdst[c] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  __threadfence_system();
}

// One warp per pair (source rank q, pair i) of the pair table, on the owner: a pair placed
// here (pair_rows[q, i] = r, 0 <= r < capacity) gets its token's codes and plain scale row
// from token-slab row q * tokens + i / topk copied into receive-slab row r (local copies).
__global__ void __launch_bounds__(256) nvfp4_ep_expand_kernel(
    const int32_t* __restrict__ pair_rows, int tokens, int topk, int world,
    const uint8_t* __restrict__ tok_codes, const uint8_t* __restrict__ tok_sf, int cols,
    uint8_t* __restrict__ recv_codes, uint8_t* __restrict__ recv_sf, int64_t capacity) {
  const int lane = threadIdx.x & 31;
  const int64_t pairs = static_cast<int64_t>(tokens) * topk;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t qi = warp0; qi < static_cast<int64_t>(world) * pairs; qi += nwarps) {
    const int64_t r = __ldg(pair_rows + qi);
    if (r < 0 || r >= capacity) continue;
    const int64_t q = qi / pairs;
    const int64_t src_row = q * tokens + (qi % pairs) / topk;
    copy_row_chunks(reinterpret_cast<const uint4*>(tok_codes + src_row * (cols / 2)),
                    reinterpret_cast<uint4*>(recv_codes + r * (cols / 2)), cols / 32, lane);
    const uint4* ssrc = reinterpret_cast<const uint4*>(tok_sf + src_row * (cols / 16));
    uint4* sdst = reinterpret_cast<uint4*>(recv_sf + r * (cols / 16));
    for (int c = lane; c < cols / 256; c += 32) sdst[c] = __ldg(ssrc + c);
  }
}

// One thread per pair of this rank: in every owner's table, the pair's slab row there (-1 on
// the owners it did not go to, and everywhere for dropped pairs), and on its owner its
// routing weight. The tables are rewritten in full on every call, so no entry is stale.
__global__ void __launch_bounds__(256) nvfp4_ep_publish_pairs_kernel(
    const int32_t* __restrict__ ids, const int32_t* __restrict__ remote_rows,
    const float* __restrict__ weights, int64_t pairs, int num_experts, int rank, int world,
    EpPeers pair_rows, EpPeers pair_weights) {
  const int epr = num_experts / world;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = ids[i];
    const int32_t row = remote_rows[i];
    const int owner = (row >= 0 && e >= 0 && e < num_experts) ? e / epr : -1;
    const int64_t at = static_cast<int64_t>(rank) * pairs + i;
    for (int p = 0; p < world; ++p)
      static_cast<int32_t*>(pair_rows.ptr[p])[at] = p == owner ? row : -1;
    if (owner >= 0) static_cast<float*>(pair_weights.ptr[owner])[at] = weights[i];
  }
  __threadfence_system();
}

// Adds one fp16x8 word group, scaled by w (w = 1: unscaled), to acc (fp32 products and sums).
__device__ __forceinline__ void add_half8(float* acc, const uint4& raw, float w, bool scale) {
  const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&words[k]));
    acc[2 * k] = __fadd_rn(acc[2 * k], scale ? __fmul_rn(w, f.x) : f.x);
    acc[2 * k + 1] = __fadd_rn(acc[2 * k + 1], scale ? __fmul_rn(w, f.y) : f.y);
  }
}

// Columns per warp task of the two kernels below: 256-column parts (8 columns per lane
// each), and the window of a token's slots whose rows return_sums loads before adding them,
// so a lane keeps up to parts x window x 16 bytes in flight. Build constants; at cfg5's
// shape on 2 GPUs (return_sums / combine_sums, µs): 4 x 4 453 / 160, 2 x 8 502 / 164,
// 2 x 4 483 / 167, 4 x 2 520 / 160, 1 x 8 640 / 264, 7 x 2 680 / 190, 7 x 4 637 / 193.
#ifndef NVFP4_EP_SUM_PARTS
#define NVFP4_EP_SUM_PARTS 4
#endif
constexpr int kEpSumParts = NVFP4_EP_SUM_PARTS;
#ifndef NVFP4_EP_SUM_WINDOW
#define NVFP4_EP_SUM_WINDOW 4
#endif
constexpr int kEpSumWindow = NVFP4_EP_SUM_WINDOW;

// One warp per (token t, source rank q, group of kEpSumParts 256-column parts), on the owner, tasks ordered token
// first so that stores to every rank run side by side: the fp32 sum, in slot order, of
// w_j * y[row_j] over t's pairs that came here (each product and each sum rounded to fp32,
// as in the slot-order combine), rounded to fp16 and stored as row (t * world + rank) of rank
// q's [tokens, world, cols] return buffer. Tokens with no pair here store nothing (their rank
// knows and skips the row). Per window of kEpSumWindow slots, the rows' indices and
// weights, then every row load of every part are issued before the first add.
__global__ void __launch_bounds__(256) nvfp4_ep_return_sums_kernel(
    const int32_t* __restrict__ pair_rows, const float* __restrict__ pair_weights, int tokens,
    int topk, int rank, int world, const __half* __restrict__ y, int64_t ldy, int cols,
    EpPeers ret) {
  const int lane = threadIdx.x & 31;
  const int groups = (cols + 256 * kEpSumParts - 1) / (256 * kEpSumParts);
  const int64_t pairs = static_cast<int64_t>(tokens) * topk;
  const int64_t tasks = static_cast<int64_t>(tokens) * world * groups;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t task = warp0; task < tasks; task += nwarps) {
    const int64_t tq = task / groups;  // t * world + q
    const int64_t t = tq / world;
    const int q = static_cast<int>(tq % world);
    const int col0 = static_cast<int>(task % groups) * 256 * kEpSumParts + lane * 8;
    const int32_t* rows = pair_rows + static_cast<int64_t>(q) * pairs + t * topk;
    const float* wts = pair_weights + static_cast<int64_t>(q) * pairs + t * topk;
    float acc[kEpSumParts][8];
#pragma unroll
    for (int u = 0; u < kEpSumParts; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[u][i] = 0.0f;
    bool any = false;
    for (int j0 = 0; j0 < topk; j0 += kEpSumWindow) {
      const int jn = topk - j0 < kEpSumWindow ? topk - j0 : kEpSumWindow;
      int32_t r[kEpSumWindow];
      float w[kEpSumWindow];
#pragma unroll
      for (int j = 0; j < kEpSumWindow; ++j) r[j] = j < jn ? __ldg(rows + j0 + j) : -1;
#pragma unroll
      for (int j = 0; j < kEpSumWindow; ++j) w[j] = r[j] >= 0 ? __ldg(wts + j0 + j) : 0.0f;
      uint4 raw[kEpSumWindow][kEpSumParts];
#pragma unroll
      for (int j = 0; j < kEpSumWindow; ++j)
#pragma unroll
        for (int u = 0; u < kEpSumParts; ++u) {
          const int col = col0 + 256 * u;
          raw[j][u] = (r[j] >= 0 && col < cols)
                          ? __ldg(reinterpret_cast<const uint4*>(y + r[j] * ldy + col))
                          : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
      for (int j = 0; j < kEpSumWindow; ++j) {
        if (r[j] < 0) continue;
        any = true;
#pragma unroll
        for (int u = 0; u < kEpSumParts; ++u) add_half8(acc[u], raw[j][u], w[j], true);
      }
    }
    if (!any) continue;
    __half* dst_row = static_cast<__half*>(ret.ptr[q]) + (t * world + rank) * cols;
#pragma unroll
    for (int u = 0; u < kEpSumParts; ++u) {
      const int col = col0 + 256 * u;
      if (col >= cols) continue;
      uint32_t packed[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __half2 h = __floats2half2_rn(acc[u][2 * k], acc[u][2 * k + 1]);
        packed[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(dst_row + col) =
          make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
  }
  __threadfence_system();
}

// out[t, :] = bf16( sum over owners p (ascending) that hold at least one kept pair of t of
// fp32(ret[t, p, :]) ), fp32 sums. One warp per task: groups_per_task consecutive groups of
// kEpSumParts 256-column parts of one token (all of them when the launch has enough tokens
// to fill the GPU), so the token's owner mask is read once per task; within a group the rows
// of two owners (every part) are loaded before they are added.
__global__ void __launch_bounds__(256) nvfp4_ep_combine_sums_kernel(
    const int32_t* __restrict__ ids, const int32_t* __restrict__ remote_rows, int tokens,
    int topk, int num_experts, int world, const __half* __restrict__ ret, int cols,
    __nv_bfloat16* __restrict__ out, int64_t ldo, int groups_per_task) {
  const int lane = threadIdx.x & 31;
  const int groups = (cols + 256 * kEpSumParts - 1) / (256 * kEpSumParts);
  const int chunks = (groups + groups_per_task - 1) / groups_per_task;  // tasks per token
  const int epr = num_experts / world;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t task = warp0; task < static_cast<int64_t>(tokens) * chunks; task += nwarps) {
    const int64_t t = task / chunks;
    const int g0 = static_cast<int>(task % chunks) * groups_per_task;
    const int g1 = min(groups, g0 + groups_per_task);
    // Bit p: owner p holds a kept pair of t. The lanes read the token's slots side by side,
    // once per task (a task covers groups_per_task column groups of the token).
    uint32_t bit = 0;
    for (int j = lane; j < topk; j += 32) {
      const int e = __ldg(ids + t * topk + j);
      if (__ldg(remote_rows + t * topk + j) >= 0 && e >= 0 && e < num_experts)
        bit |= 1u << (e / epr);
    }
    const uint32_t owners = __reduce_or_sync(0xffffffffu, bit);
#pragma unroll 2
    for (int g = g0; g < g1; ++g) {
      const int col0 = g * 256 * kEpSumParts + lane * 8;
      float acc[kEpSumParts][8];
#pragma unroll
      for (int u = 0; u < kEpSumParts; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[u][i] = 0.0f;
      for (int p0 = 0; p0 < world; p0 += 2) {
        uint4 raw[2][kEpSumParts];
#pragma unroll
        for (int v = 0; v < 2; ++v)
#pragma unroll
          for (int u = 0; u < kEpSumParts; ++u) {
            const int p = p0 + v;
            const int col = col0 + 256 * u;
            raw[v][u] = (p < world && ((owners >> p) & 1u) && col < cols)
                            ? __ldg(reinterpret_cast<const uint4*>(ret + (t * world + p) * cols + col))
                            : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          const int p = p0 + v;
          if (p >= world || !((owners >> p) & 1u)) continue;
#pragma unroll
          for (int u = 0; u < kEpSumParts; ++u) add_half8(acc[u], raw[v][u], 1.0f, false);
        }
      }
#pragma unroll
      for (int u = 0; u < kEpSumParts; ++u) {
        const int col = col0 + 256 * u;
        if (col < cols) store_bf16x8(out + t * ldo + col, acc[u]);
      }
    }
  }
}

}  // namespace nvfp4
