// Warp-level row operations shared by the MoE and expert-parallel kernels: the weighted
// slot-order combine of a token's expert output rows, and a row copy with several 16-byte
// chunks in flight per lane.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace nvfp4 {

// Weighted fp32 sum, in slot order, of a token's expert output rows at 8 columns per lane:
// acc[c] += w_j * y[row_j * ld + col + c] for the token's slots j with row_of(pair) >= 0
// (each product and each sum rounded to fp32). Per 8 slots, the row indices and weights
// (the same addresses for every lane: one transaction each) and then all 8 row loads are
// issued before the first add, so a lane keeps 8 x 16 bytes in flight.
template <typename RowOf>
__device__ __forceinline__ void combine_slots(int64_t t, int topk, int col, bool active,
                                              const __half* __restrict__ y, int64_t ld,
                                              const float* __restrict__ weights, RowOf row_of,
                                              float* acc) {
  for (int j0 = 0; j0 < topk; j0 += 8) {
    const int jn = topk - j0 < 8 ? topk - j0 : 8;
    int64_t r[8];
    float w[8];
    uint4 raw[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = j < jn ? row_of(t * topk + j0 + j) : -1;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      raw[j] = (active && r[j] >= 0) ? __ldg(reinterpret_cast<const uint4*>(y + r[j] * ld + col))
                                     : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = j < jn ? __ldg(weights + t * topk + j0 + j) : 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (r[j] < 0) continue;
      const uint32_t words[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&words[k]));
        acc[2 * k] = __fadd_rn(acc[2 * k], __fmul_rn(w[j], f.x));
        acc[2 * k + 1] = __fadd_rn(acc[2 * k + 1], __fmul_rn(w[j], f.y));
      }
    }
  }
}

__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* dst, const float* acc) {
  uint32_t packed[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
    packed[k] = *reinterpret_cast<const uint32_t*>(&b);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
}

// Row copy by one warp, 16 bytes per lane per chunk: four chunks' loads are issued before
// their stores, so a lane has 64 bytes in flight.
__device__ __forceinline__ void copy_row_chunks(const uint4* __restrict__ src, uint4* dst,
                                                int chunks, int lane) {
  for (int c0 = lane; c0 < chunks; c0 += 128) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + 32 * u;
      v[u] = c < chunks ? __ldg(src + c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c0 + 32 * u < chunks) dst[c0 + 32 * u] = v[u];
  }
}

}  // namespace nvfp4
