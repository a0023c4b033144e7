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

}  // namespace nvfp4
