// MoE token dispatch and combine around the grouped GEMM.
//
// Routing (deterministic stable counting sort of the (token, slot) pairs by expert):
//   1. nvfp4_route_histogram_kernel: per chunk of kRouteChunk pairs, a histogram per expert.
//   2. nvfp4_route_scan_kernel: per expert, the running base of every chunk and the total;
//      padded row offsets (every expert's rows start on a 128-row boundary, so the blocked
//      scale layout of the whole dispatched buffer is the concatenation of the experts'
//      blocked layouts). The row -> token map is set to -1 (a memset) before the scatter.
//   3. nvfp4_route_scatter_kernel: the destination row of every pair, in token order within
//      each expert: chunk base + rank within the chunk (warp match_any for the rank inside a
//      warp's 32 pairs, per-warp expert counts for the rank across a chunk's warps).
// Combine: out[t] = sum_j w[t, j] * Y[dest[t, j]] in fp32 (slot order, each product and sum
// rounded to nearest), written as bf16.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "row_ops.cuh"

namespace nvfp4 {

constexpr int kRouteChunk = 2048;       // pairs per chunk
constexpr int kRouteThreads = 256;      // 8 warps; a warp owns 256 consecutive pairs of a chunk
constexpr int kRouteMaxExperts = 1024;

__global__ void __launch_bounds__(kRouteThreads) nvfp4_route_histogram_kernel(
    const int32_t* __restrict__ ids, int64_t pairs, int num_experts, int32_t* __restrict__ hist) {
  __shared__ int32_t h[kRouteMaxExperts];
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kRouteChunk;
  for (int i = threadIdx.x; i < kRouteChunk; i += blockDim.x) {
    const int64_t p = base + i;
    if (p < pairs) {
      const int e = ids[p];
      if (e >= 0 && e < num_experts) atomicAdd(&h[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x)
    hist[static_cast<int64_t>(blockIdx.x) * num_experts + e] = h[e];
}

// One block of kRouteMaxExperts threads, thread e for expert e. hist[c][e] becomes the
// exclusive running count of expert e before chunk c; counts[e] the total; offsets[e] the
// padded first row of expert e (offsets[num_experts] = padded total), from a block-wide
// exclusive scan of the padded counts. (Padding rows are marked -1 in the row -> token map
// by a memset before the scatter writes the real rows.)
__global__ void __launch_bounds__(kRouteMaxExperts) nvfp4_route_scan_kernel(
    int32_t* __restrict__ hist, int chunks, int num_experts, int32_t* __restrict__ counts,
    int32_t* __restrict__ offsets) {
  __shared__ int32_t warp_sums[kRouteMaxExperts / 32];
  const int e = threadIdx.x;
  const int lane = e & 31;
  const int warp = e >> 5;
  int32_t run = 0;
  if (e < num_experts) {
    int c = 0;
    for (; c + 4 <= chunks; c += 4) {  // four independent loads in flight
      int32_t* slot = hist + static_cast<int64_t>(c) * num_experts + e;
      int32_t v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = slot[static_cast<int64_t>(u) * num_experts];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        slot[static_cast<int64_t>(u) * num_experts] = run;
        run += v[u];
      }
    }
    for (; c < chunks; ++c) {
      int32_t* slot = hist + static_cast<int64_t>(c) * num_experts + e;
      const int32_t v = *slot;
      *slot = run;
      run += v;
    }
    counts[e] = run;
  }
  const int32_t padded = e < num_experts ? (run + 127) / 128 * 128 : 0;
  int32_t incl = padded;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int32_t t = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += t;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int32_t w = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t t = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += t;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  incl += warp > 0 ? warp_sums[warp - 1] : 0;
  if (e < num_experts) offsets[e] = incl - padded;
  if (e == num_experts - 1) offsets[num_experts] = incl;
}

__global__ void __launch_bounds__(kRouteThreads) nvfp4_route_scatter_kernel(
    const int32_t* __restrict__ ids, int64_t pairs, int topk, int num_experts,
    const int32_t* __restrict__ hist, const int32_t* __restrict__ offsets,
    int32_t* __restrict__ dest, int32_t* __restrict__ src_rows) {
  constexpr int kWarps = kRouteThreads / 32;
  constexpr int kPerWarp = kRouteChunk / kWarps;  // 256 consecutive pairs per warp
  __shared__ int32_t wcount[kWarps][kRouteMaxExperts];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kWarps * num_experts; i += blockDim.x)
    wcount[i / num_experts][i % num_experts] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kRouteChunk + warp * kPerWarp;
  // Pass 1: each warp counts its pairs per expert (lane 0 of each peer set adds the set).
  for (int s = 0; s < kPerWarp; s += 32) {
    const int64_t p = base + s + lane;
    int e = p < pairs ? ids[p] : -1;
    if (e >= num_experts) e = -1;
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) wcount[warp][e] += __popc(peers);
  }
  __syncthreads();
  // Exclusive prefix over the chunk's warps, per expert.
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) {
    int32_t run = 0;
    for (int w = 0; w < kWarps; ++w) {
      const int32_t v = wcount[w][e];
      wcount[w][e] = run;
      run += v;
    }
  }
  __syncthreads();
  // Pass 2: destination rows in pair order.
  const int32_t* chunk_base = hist + static_cast<int64_t>(blockIdx.x) * num_experts;
  for (int s = 0; s < kPerWarp; s += 32) {
    const int64_t p = base + s + lane;
    int e = p < pairs ? ids[p] : -1;
    if (e >= num_experts) e = -1;
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0) {
      const int32_t row = offsets[e] + chunk_base[e] + wcount[warp][e] + rank;
      dest[p] = row;
      src_rows[row] = static_cast<int32_t>(p / topk);
    } else if (p < pairs) {
      dest[p] = -1;
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) wcount[warp][e] += __popc(peers);
    __syncwarp();
  }
}

// out[t, :] = bf16( sum_j w[t, j] * y[dest[t*topk + j], :] ), fp32 products and sums in slot
// order; pairs with dest < 0 contribute nothing. One warp per (token, 256-column chunk):
// lane l handles 8 consecutive columns (16-byte loads of fp16, 16-byte stores of bf16).
__global__ void __launch_bounds__(256) nvfp4_moe_combine_kernel(
    const __half* __restrict__ y, int64_t ldy, const int32_t* __restrict__ dest,
    const float* __restrict__ weights, int tokens, int topk, int cols,
    __nv_bfloat16* __restrict__ out, int64_t ldo) {
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
    combine_slots(t, topk, col, active, y, ldy, weights,
                  [&](int64_t i) -> int64_t { return __ldg(dest + i); }, acc);
    if (active) store_bf16x8(out + t * ldo + col, acc);
  }
}

// Dispatch of already-quantised rows: dispatched row r takes packed row src_rows[r] and its
// scales (zeros where src_rows[r] < 0). Quantisation is row-local, so quantising each token
// once and gathering is bit-identical to quantising the gathered bf16 rows, with a quarter of
// the bytes moved per dispatched row (K/2 + K/16 instead of 2K read).
// Packed rows: one warp per dispatched row, 16 bytes per lane.
__global__ void __launch_bounds__(256) nvfp4_gather_packed_rows_kernel(
    const uint8_t* __restrict__ src, int64_t ld_src, const int32_t* __restrict__ src_rows,
    int rows, int row_bytes, uint8_t* __restrict__ dst, int64_t ld_dst) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int chunks = row_bytes / 16;
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const int32_t s = __ldg(src_rows + r);
    uint4* d = reinterpret_cast<uint4*>(dst + r * ld_dst);
    if (s >= 0) {
      const uint4* q = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(s) * ld_src);
      copy_row_chunks(q, d, chunks, lane);
    } else {
      for (int c = lane; c < chunks; c += 32) d[c] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// Blocked scales: one warp per destination 512-byte block (128 rows mm, 4 scale columns kk);
// lane i0 assembles the block's 16-byte row i0 from the four rows 32*i1 + i0 (their 4-byte
// groups in the source blocked layout) and stores it in one piece.
__global__ void __launch_bounds__(256) nvfp4_gather_blocked_scales_kernel(
    const uint8_t* __restrict__ sf_src, const int32_t* __restrict__ src_rows, int rows,
    int rest_k, uint8_t* __restrict__ sf_dst) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int row_blocks = (rows + 127) / 128;
  const int64_t tasks = static_cast<int64_t>(row_blocks) * rest_k;
  for (int64_t task = warp0; task < tasks; task += nwarps) {
    const int mm = static_cast<int>(task / rest_k);
    const int kk = static_cast<int>(task % rest_k);
    uint32_t w[4];
#pragma unroll
    for (int i1 = 0; i1 < 4; ++i1) {
      const int r = mm * 128 + i1 * 32 + lane;
      const int32_t s = r < rows ? __ldg(src_rows + r) : -1;
      w[i1] = 0u;
      if (s >= 0) {
        const int64_t off = ((static_cast<int64_t>(s >> 7) * rest_k + kk) * 32 + (s & 31)) * 16 +
                            ((s & 127) >> 5) * 4;
        w[i1] = __ldg(reinterpret_cast<const uint32_t*>(sf_src + off));
      }
    }
    *reinterpret_cast<uint4*>(sf_dst + (task * 32 + lane) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace nvfp4
