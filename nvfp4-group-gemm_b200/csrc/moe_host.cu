// Host entry points of the activation quantiser and the MoE routing, dispatch and combine
// kernels (nvfp4_quantize*, nvfp4_moe_*).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstddef>

#include "../../include/nvfp4_group_gemm.h"
#include "host_common.cuh"
#include "moe_kernels.cuh"
#include "quantize_kernel.cuh"

namespace nvfp4 {
namespace {

int quantize_impl(const void* x, int rows, int cols, int64_t ld, int dtype, float global_scale,
                  const int32_t* src_rows, int row_mode, void* packed, int64_t packed_ld,
                  void* sf_blocked, void* stream) {
  if (dtype != NVFP4_DTYPE_BF16 && dtype != NVFP4_DTYPE_FP16)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "dtype=%d (expected NVFP4_DTYPE_BF16 or _FP16)", dtype);
  if (!(global_scale > 0.0f) || !std::isfinite(global_scale))
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "global_scale must be finite and > 0");
  if (rows < 0 || cols <= 0 || cols % 64 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "rows=%d cols=%d (cols must be a positive multiple of 64)",
                rows, cols);
  if (rows == 0) return NVFP4_OK;
  if (x == nullptr || packed == nullptr || sf_blocked == nullptr ||
      (row_mode != kQuantRowsPlain && src_rows == nullptr))
    return fail(NVFP4_ERR_NULL_POINTER, "x, packed, sf_blocked or src_rows is NULL");
  if (ld < cols || packed_ld < cols / 2)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "ld=%lld packed_ld=%lld too small for cols=%d",
                static_cast<long long>(ld), static_cast<long long>(packed_ld), cols);
  if (!aligned16(x) || !aligned16(packed) || !aligned16(sf_blocked) || ld % 8 != 0 ||
      packed_ld % 16 != 0)
    return fail(NVFP4_ERR_MISALIGNED,
                "x, packed and sf_blocked must be 16-byte aligned, ld a multiple of 8 elements "
                "and packed_ld a multiple of 16 bytes");
  DeviceState* dsp = nullptr;
  const int dst = current_device_state(&dsp);
  if (dst != NVFP4_OK) return dst;
  const DeviceState& ds = *dsp;
  const int row_blocks = (rows + 127) / 128;
  const int rest_k = cols / 64;
  const int64_t warps = static_cast<int64_t>(row_blocks) * rest_k;
  const int threads = 32 * kQuantWarps;
  const int64_t blocks = std::min<int64_t>((warps + kQuantWarps - 1) / kQuantWarps,
                                           static_cast<int64_t>(ds.num_sms) * 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == NVFP4_DTYPE_BF16)
    nvfp4_quantize_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), rows, ld, global_scale,
        static_cast<uint8_t*>(packed), packed_ld, static_cast<uint8_t*>(sf_blocked), row_blocks,
        rest_k, src_rows, row_mode);
  else
    nvfp4_quantize_kernel<__half><<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        static_cast<const __half*>(x), rows, ld, global_scale, static_cast<uint8_t*>(packed),
        packed_ld, static_cast<uint8_t*>(sf_blocked), row_blocks, rest_k, src_rows, row_mode);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return NVFP4_OK;
}

int64_t route_chunks(int64_t pairs) { return (pairs + kRouteChunk - 1) / kRouteChunk; }

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

NVFP4_API int nvfp4_quantize(const void* x, int rows, int cols, int64_t ld, int dtype,
                             float global_scale, void* packed, int64_t packed_ld, void* sf_blocked,
                             void* stream) {
  g_last_error.clear();
  return quantize_impl(x, rows, cols, ld, dtype, global_scale, nullptr, kQuantRowsPlain, packed,
                       packed_ld, sf_blocked, stream);
}

NVFP4_API int nvfp4_quantize_rows(const void* x, int rows, int cols, int64_t ld, int dtype,
                                  float global_scale, const int32_t* src_rows, int mode,
                                  void* packed, int64_t packed_ld, void* sf_blocked,
                                  void* stream) {
  g_last_error.clear();
  if (mode != NVFP4_ROWS_GATHER && mode != NVFP4_ROWS_MASK)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "mode=%d (expected NVFP4_ROWS_GATHER or _MASK)", mode);
  return quantize_impl(x, rows, cols, ld, dtype, global_scale, src_rows,
                       mode == NVFP4_ROWS_GATHER ? kQuantRowsGather : kQuantRowsMask, packed,
                       packed_ld, sf_blocked, stream);
}

NVFP4_API size_t nvfp4_moe_route_workspace_size(int64_t pairs, int num_experts) {
  if (pairs <= 0 || num_experts <= 0) return 0;
  return static_cast<size_t>(route_chunks(pairs)) * static_cast<size_t>(num_experts) * 4u;
}

NVFP4_API int nvfp4_moe_route(const int32_t* topk_ids, int tokens, int topk, int num_experts,
                              int32_t* counts, int32_t* offsets, int32_t* dest, int32_t* src_rows,
                              int64_t rows_capacity, void* workspace, size_t workspace_bytes,
                              void* stream) {
  g_last_error.clear();
  if (num_experts <= 0 || num_experts > kRouteMaxExperts)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "num_experts=%d must be in [1, %d]", num_experts,
                kRouteMaxExperts);
  if (tokens < 0 || topk <= 0) return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d", tokens, topk);
  const int64_t pairs = static_cast<int64_t>(tokens) * topk;
  if (pairs > (int64_t{1} << 30)) return fail(NVFP4_ERR_BAD_SHAPE, "too many pairs");
  if (counts == nullptr || offsets == nullptr ||
      (pairs > 0 && (topk_ids == nullptr || dest == nullptr || src_rows == nullptr)))
    return fail(NVFP4_ERR_NULL_POINTER, "a routing buffer is NULL");
  const int64_t need_rows = pairs + static_cast<int64_t>(num_experts) * 127;
  if (rows_capacity < need_rows)
    return fail(NVFP4_ERR_INVALID_ARGUMENT,
                "rows_capacity=%lld < tokens*topk + 127*num_experts = %lld",
                static_cast<long long>(rows_capacity), static_cast<long long>(need_rows));
  const size_t ws_need = nvfp4_moe_route_workspace_size(pairs, num_experts);
  if (ws_need > 0 && (workspace == nullptr || workspace_bytes < ws_need))
    return fail(NVFP4_ERR_WORKSPACE, "routing workspace has %zu bytes, needs %zu", workspace_bytes,
                ws_need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t chunks = route_chunks(pairs);
  int32_t* hist = static_cast<int32_t*>(workspace);
  if (chunks > 0) {
    nvfp4_route_histogram_kernel<<<static_cast<unsigned>(chunks), kRouteThreads, 0, s>>>(
        topk_ids, pairs, num_experts, hist);
  }
  // Every row of the map starts as padding (-1); the scatter writes the real rows.
  if (src_rows != nullptr) {
    cudaError_t me = cudaMemsetAsync(src_rows, 0xFF, static_cast<size_t>(rows_capacity) * 4, s);
    if (me != cudaSuccess) return cuda_fail(me, "routing map reset");
  }
  nvfp4_route_scan_kernel<<<1, kRouteMaxExperts, 0, s>>>(hist, static_cast<int>(chunks),
                                                         num_experts, counts, offsets);
  if (chunks > 0) {
    nvfp4_route_scatter_kernel<<<static_cast<unsigned>(chunks), kRouteThreads, 0, s>>>(
        topk_ids, pairs, topk, num_experts, hist, offsets, dest, src_rows);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "routing launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_moe_gather_quantized(const void* packed_src, int64_t ld_src,
                                         const void* sf_src, const int32_t* src_rows, int rows,
                                         int cols, void* packed_dst, int64_t ld_dst, void* sf_dst,
                                         void* stream) {
  g_last_error.clear();
  if (rows < 0 || cols <= 0 || cols % 64 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "rows=%d cols=%d (cols a positive multiple of 64)", rows, cols);
  if (rows == 0) return NVFP4_OK;
  if (packed_src == nullptr || sf_src == nullptr || src_rows == nullptr || packed_dst == nullptr ||
      sf_dst == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a gather buffer is NULL");
  if (ld_src < cols / 2 || ld_dst < cols / 2)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "row strides smaller than cols/2 bytes");
  if (!aligned16(packed_src) || !aligned16(packed_dst) || !aligned16(sf_src) || !aligned16(sf_dst) ||
      ld_src % 16 != 0 || ld_dst % 16 != 0)
    return fail(NVFP4_ERR_MISALIGNED, "buffers must be 16-byte aligned, row strides multiples of 16");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t row_blocks = std::min<int64_t>((static_cast<int64_t>(rows) + 7) / 8, 148 * 16);
  nvfp4_gather_packed_rows_kernel<<<static_cast<unsigned>(row_blocks), 256, 0, s>>>(
      static_cast<const uint8_t*>(packed_src), ld_src, src_rows, rows, cols / 2,
      static_cast<uint8_t*>(packed_dst), ld_dst);
  const int rest_k = cols / 64;
  const int64_t sf_tasks = static_cast<int64_t>((rows + 127) / 128) * rest_k;
  const int64_t sf_blocks = std::min<int64_t>((sf_tasks + 7) / 8, 148 * 16);
  nvfp4_gather_blocked_scales_kernel<<<static_cast<unsigned>(sf_blocks), 256, 0, s>>>(
      static_cast<const uint8_t*>(sf_src), src_rows, rows, rest_k, static_cast<uint8_t*>(sf_dst));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gather launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_moe_combine(const void* y, int64_t ldy, const int32_t* dest,
                                const float* weights, int tokens, int topk, int cols, void* out,
                                int64_t ldo, void* stream) {
  g_last_error.clear();
  if (tokens < 0 || topk <= 0 || cols <= 0 || cols % 8 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d cols=%d (cols a multiple of 8)", tokens,
                topk, cols);
  if (tokens == 0) return NVFP4_OK;
  if (y == nullptr || dest == nullptr || weights == nullptr || out == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a combine buffer is NULL");
  if (ldy < cols || ldo < cols) return fail(NVFP4_ERR_INVALID_ARGUMENT, "ldy/ldo < cols");
  if (!aligned16(y) || !aligned16(out) || ldy % 8 != 0 || ldo % 8 != 0)
    return fail(NVFP4_ERR_MISALIGNED, "y and out must be 16-byte aligned, ldy and ldo multiples of 8");
  const int chunks = (cols + 255) / 256;
  const int64_t warps = static_cast<int64_t>(tokens) * chunks;
  const int64_t blocks = std::min<int64_t>((warps + 7) / 8, 148 * 16);
  nvfp4_moe_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(y), ldy, dest, weights, tokens, topk, cols,
      static_cast<__nv_bfloat16*>(out), ldo);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  return NVFP4_OK;
}

}  // extern "C"
