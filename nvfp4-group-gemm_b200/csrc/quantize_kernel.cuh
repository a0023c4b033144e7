// NVFP4 activation quantiser: bf16/fp16 [rows, cols] -> packed e2m1 [rows, cols/2] and
// E4M3 block scales written straight into the 128x4-blocked layout the GEMM consumes.
//
// Two-level scaling (nvfp4_quant_math.cuh); s_g = amax_tensor / (6 * 448) keeps every
// block scale in E4M3's range.
//
// Memory-bound: 2 bytes in, 0.5 + 1/16 bytes out per element. A first version gave each
// lane whole rows (so each warp load touched 32 rows): L1 ran at 94 % of its peak and the
// kernel reached 0.66 of HBM on 3.8 GB of activations.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "nvfp4_quant_math.cuh"
#include "sm100_ptx.cuh"

namespace nvfp4 {

// Sixteen elements held as eight 32-bit words (two 16-byte loads) -> fp32 (exact).
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& lo, const uint4& hi, float* v) {
  const uint32_t words[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      v[2 * j] = __uint_as_float(words[j] << 16);
      v[2 * j + 1] = __uint_as_float(words[j] & 0xFFFF0000u);
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&words[j]);
      const float2 f = __half22float2(h);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// One warp per 512-byte scale block, i.e. per (128-row block mm, 64-column chunk kk).
// Lane l covers elements 8 * (l % 8) .. + 7 of the chunk in rows 4 * it + l / 8
// (it = 0..31), so every load covers four whole 128-byte row chunks and every store four
// whole 32-byte packed chunks. A 16-element block spans a lane pair, which exchanges its
// half-block amax with one shuffle. Scale codes are gathered in shared memory and the
// block is written as 32 x 16 bytes at the end.
constexpr int kQuantWarps = 8;
constexpr int kQuantUnroll = 8;  // rows in flight per lane

// Row maps: output row r reads input row r (kQuantRowsPlain), input row src_rows[r]
// (kQuantRowsGather: MoE dispatch; -1 = a padding row, quantised as zeros), or input row r
// only where src_rows[r] >= 0 (kQuantRowsMask: rows of a dispatched buffer that hold data).
enum : int { kQuantRowsPlain = 0, kQuantRowsGather = 1, kQuantRowsMask = 2 };

template <typename T>
__global__ void __launch_bounds__(32 * kQuantWarps, 4) nvfp4_quantize_kernel(
    const T* __restrict__ x, int rows, int64_t ld, float sg, uint8_t* __restrict__ packed,
    int64_t packed_ld, uint8_t* __restrict__ sf, int row_blocks, int rest_k,
    const int32_t* __restrict__ src_rows, int row_mode) {
  __shared__ __align__(16) uint8_t sf_stage[kQuantWarps][512];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int sub = lane & 7;   // 16-byte segment of the 128-byte row chunk
  const int rgrp = lane >> 3;  // row within a group of four
  uint8_t* stage = sf_stage[wib];
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t tasks = static_cast<int64_t>(row_blocks) * rest_k;
  const float d6 = __fmul_rn(6.0f, sg);
  for (int64_t task = warp0; task < tasks; task += nwarps) {
    const int mm = static_cast<int>(task / rest_k);
    const int kk = static_cast<int>(task % rest_k);
#pragma unroll 1
    for (int it0 = 0; it0 < 32; it0 += kQuantUnroll) {
      uint4 raw[kQuantUnroll];
#pragma unroll
      for (int u = 0; u < kQuantUnroll; ++u) {
        const int row = mm * 128 + (it0 + u) * 4 + rgrp;
        int in_row = row < rows ? row : -1;
        if (row_mode != kQuantRowsPlain && in_row >= 0) {
          const int32_t m = __ldg(src_rows + row);
          in_row = m < 0 ? -1 : (row_mode == kQuantRowsGather ? m : row);
        }
        raw[u] = in_row >= 0 ? __ldg(reinterpret_cast<const uint4*>(
                                   x + static_cast<int64_t>(in_row) * ld +
                                   static_cast<int64_t>(kk) * 64) + sub)
                             : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kQuantUnroll; ++u) {
        const int r = (it0 + u) * 4 + rgrp;  // row within the 128-row block
        const int row = mm * 128 + r;
        float v[8];
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        float v16[16];
        unpack16<T>(raw[u], z, v16);  // first 8 values are this lane's elements
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = v16[i];
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        float enc;
        const uint32_t code = block_scale(amax, sg, d6, enc);
        float q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = __fmul_rn(v[i], enc);
        const uint32_t bytes = cvt_e2m1x8(q);
        if (row < rows)
          *reinterpret_cast<uint32_t*>(packed + static_cast<int64_t>(row) * packed_ld +
                                       static_cast<int64_t>(kk) * 32 + sub * 4) = bytes;
        // Scale j = sub / 2 of row r: byte (r % 32) * 16 + (r / 32) * 4 + j of the block.
        if ((sub & 1) == 0) stage[(r & 31) * 16 + (r >> 5) * 4 + (sub >> 1)] = static_cast<uint8_t>(code);
      }
    }
    __syncwarp();
    *reinterpret_cast<uint4*>(sf + ((static_cast<int64_t>(mm) * rest_k + kk) * 32 + lane) * 16) =
        *reinterpret_cast<const uint4*>(stage + lane * 16);
    __syncwarp();
  }
}

}  // namespace nvfp4
