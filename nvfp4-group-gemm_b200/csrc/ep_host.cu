// Host entry points of the expert-parallel exchange (nvfp4_ep_*).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>

#include "../../include/nvfp4_group_gemm.h"
#include "ep_kernels.cuh"
#include "host_common.cuh"

using namespace nvfp4;

extern "C" {

// ---------------------------------------------------------------------------- expert parallel
static_assert(sizeof(nvfp4_ep_peers) == sizeof(EpPeers), "peer table layouts differ");
static_assert(NVFP4_EP_MAX_RANKS == kEpMaxRanks, "header and library disagree");

namespace {
EpPeers to_peers(const nvfp4_ep_peers& p) {
  EpPeers out;
  for (int i = 0; i < kEpMaxRanks; ++i) out.ptr[i] = p.ptr[i];
  return out;
}

int check_ep_world(int num_experts, int rank, int world) {
  if (world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "rank %d of world %d (1..%d ranks)", rank, world,
                kEpMaxRanks);
  if (num_experts <= 0 || num_experts > kEpMaxExperts || num_experts % world != 0)
    return fail(NVFP4_ERR_INVALID_ARGUMENT,
                "num_experts=%d must be in 1..%d and a multiple of the world size %d",
                num_experts, kEpMaxExperts, world);
  return NVFP4_OK;
}

int check_peers(const nvfp4_ep_peers& p, int world, const char* name, bool align16) {
  for (int i = 0; i < world; ++i) {
    if (p.ptr[i] == nullptr) return fail(NVFP4_ERR_NULL_POINTER, "%s[%d] is NULL", name, i);
    if (align16 ? !aligned16(p.ptr[i]) : (reinterpret_cast<uintptr_t>(p.ptr[i]) & 3u) != 0)
      return fail(NVFP4_ERR_MISALIGNED, "%s[%d] misaligned", name, i);
  }
  return NVFP4_OK;
}
}  // namespace

NVFP4_API int nvfp4_ep_publish_counts(const int32_t* counts, int num_experts, int rank, int world,
                                      nvfp4_ep_peers count_mats, void* stream) {
  g_last_error.clear();
  int st = check_ep_world(num_experts, rank, world);
  if (st != NVFP4_OK) return st;
  if (counts == nullptr) return fail(NVFP4_ERR_NULL_POINTER, "counts is NULL");
  if ((st = check_peers(count_mats, world, "count_mats", false)) != NVFP4_OK) return st;
  const int n = world * num_experts;
  nvfp4_ep_publish_counts_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      counts, num_experts, rank, world, to_peers(count_mats));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "publish counts launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_layout(const int32_t* count_mat, int num_experts, int rank, int world,
                              int64_t recv_capacity, int32_t* seg_offsets, int32_t* seg_counts,
                              int32_t* send_base, unsigned int* error_word, void* stream) {
  g_last_error.clear();
  int st = check_ep_world(num_experts, rank, world);
  if (st != NVFP4_OK) return st;
  if (count_mat == nullptr || seg_offsets == nullptr || seg_counts == nullptr ||
      send_base == nullptr || error_word == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a layout buffer is NULL");
  if (recv_capacity < 0 || recv_capacity > INT32_MAX)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "recv_capacity=%lld",
                static_cast<long long>(recv_capacity));
  nvfp4_ep_layout_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      count_mat, num_experts, rank, world, recv_capacity, seg_offsets, seg_counts, send_base,
      error_word);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "layout launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_dispatch(const int32_t* topk_ids, int tokens, int topk, int num_experts,
                                int rank, int world, const int32_t* dest, const int32_t* offsets,
                                const int32_t* send_base, const void* codes, int64_t ld_codes,
                                const void* sf_blocked, int cols, nvfp4_ep_peers recv_codes,
                                nvfp4_ep_peers recv_sf, nvfp4_ep_peers recv_meta,
                                int64_t recv_capacity, int32_t* remote_rows, void* stream) {
  g_last_error.clear();
  int st = check_ep_world(num_experts, rank, world);
  if (st != NVFP4_OK) return st;
  if (tokens < 0 || topk <= 0 || cols <= 0 || cols % 256 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d cols=%d (cols a multiple of 256)",
                tokens, topk, cols);
  if (tokens == 0) return NVFP4_OK;
  if (topk_ids == nullptr || dest == nullptr || offsets == nullptr || send_base == nullptr ||
      codes == nullptr || sf_blocked == nullptr || remote_rows == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a dispatch buffer is NULL");
  if (!aligned16(codes) || ld_codes % 16 != 0 || ld_codes < cols / 2 ||
      (reinterpret_cast<uintptr_t>(sf_blocked) & 3u) != 0)
    return fail(NVFP4_ERR_MISALIGNED, "codes 16-byte aligned with ld a multiple of 16 >= cols/2, "
                "scales 4-byte aligned");
  if ((st = check_peers(recv_codes, world, "recv_codes", true)) != NVFP4_OK) return st;
  if ((st = check_peers(recv_sf, world, "recv_sf", true)) != NVFP4_OK) return st;
  if ((st = check_peers(recv_meta, world, "recv_meta", true)) != NVFP4_OK) return st;
  const int64_t pairs = static_cast<int64_t>(tokens) * topk;
  const int64_t blocks = std::min<int64_t>((pairs + 7) / 8, 148 * 16);
  nvfp4_ep_dispatch_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                             static_cast<cudaStream_t>(stream)>>>(
      topk_ids, pairs, topk, num_experts, rank, world, dest, offsets, send_base,
      static_cast<const uint8_t*>(codes), ld_codes, static_cast<const uint8_t*>(sf_blocked), cols,
      to_peers(recv_codes), to_peers(recv_sf), to_peers(recv_meta), recv_capacity, remote_rows);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dispatch launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_combine(const int32_t* remote_rows, const float* weights, int tokens,
                               int topk, const void* ret, int cols, void* out, int64_t ldo,
                               void* stream) {
  g_last_error.clear();
  if (tokens < 0 || topk <= 0 || cols <= 0 || cols % 8 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d cols=%d (cols a multiple of 8)", tokens,
                topk, cols);
  if (tokens == 0) return NVFP4_OK;
  if (remote_rows == nullptr || weights == nullptr || ret == nullptr || out == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a combine buffer is NULL");
  if (!aligned16(out) || !aligned16(ret) || ldo % 8 != 0 || ldo < cols)
    return fail(NVFP4_ERR_MISALIGNED, "ret and out 16-byte aligned, ldo a multiple of 8 >= cols");
  const int chunks = (cols + 255) / 256;
  const int64_t warps = static_cast<int64_t>(tokens) * chunks;
  const int64_t blocks = std::min<int64_t>((warps + 7) / 8, 148 * 16);
  nvfp4_ep_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                            static_cast<cudaStream_t>(stream)>>>(
      remote_rows, weights, tokens, topk, static_cast<const __half*>(ret), cols,
      static_cast<__nv_bfloat16*>(out), ldo);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_dispatch_tokens(const int32_t* topk_ids, int tokens, int topk,
                                       int num_experts, int rank, int world, const int32_t* dest,
                                       const int32_t* offsets, const int32_t* send_base,
                                       const void* codes, int64_t ld_codes, const void* sf_blocked,
                                       int cols, nvfp4_ep_peers tok_codes, nvfp4_ep_peers tok_sf,
                                       int64_t recv_capacity, int32_t* remote_rows, void* stream) {
  g_last_error.clear();
  int st = check_ep_world(num_experts, rank, world);
  if (st != NVFP4_OK) return st;
  if (tokens < 0 || topk <= 0 || cols <= 0 || cols % 256 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d cols=%d (cols a multiple of 256)",
                tokens, topk, cols);
  if (tokens == 0) return NVFP4_OK;
  if (topk_ids == nullptr || dest == nullptr || offsets == nullptr || send_base == nullptr ||
      codes == nullptr || sf_blocked == nullptr || remote_rows == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a dispatch buffer is NULL");
  if (!aligned16(codes) || ld_codes % 16 != 0 || ld_codes < cols / 2 ||
      (reinterpret_cast<uintptr_t>(sf_blocked) & 3u) != 0)
    return fail(NVFP4_ERR_MISALIGNED, "codes 16-byte aligned with ld a multiple of 16 >= cols/2, "
                "scales 4-byte aligned");
  if ((st = check_peers(tok_codes, world, "tok_codes", true)) != NVFP4_OK) return st;
  if ((st = check_peers(tok_sf, world, "tok_sf", true)) != NVFP4_OK) return st;
  const int64_t blocks = std::min<int64_t>((static_cast<int64_t>(tokens) + 7) / 8, 148 * 16);
  nvfp4_ep_dispatch_tokens_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                                    static_cast<cudaStream_t>(stream)>>>(
      topk_ids, tokens, topk, num_experts, rank, world, dest, offsets, send_base,
      static_cast<const uint8_t*>(codes), ld_codes, static_cast<const uint8_t*>(sf_blocked), cols,
      to_peers(tok_codes), to_peers(tok_sf), recv_capacity, remote_rows);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dispatch tokens launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_expand(const int32_t* pair_rows, int tokens, int topk, int world,
                              const void* tok_codes, const void* tok_sf, int cols,
                              void* recv_codes, void* recv_sf, int64_t recv_capacity,
                              void* stream) {
  g_last_error.clear();
  if (world < 1 || world > kEpMaxRanks)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "world %d (1..%d ranks)", world, kEpMaxRanks);
  if (tokens < 0 || topk <= 0 || cols <= 0 || cols % 256 != 0 || recv_capacity < 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d cols=%d (cols a multiple of 256)",
                tokens, topk, cols);
  if (tokens == 0) return NVFP4_OK;
  if (pair_rows == nullptr || tok_codes == nullptr || tok_sf == nullptr ||
      recv_codes == nullptr || recv_sf == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "an expand buffer is NULL");
  if (!aligned16(tok_codes) || !aligned16(tok_sf) || !aligned16(recv_codes) ||
      !aligned16(recv_sf))
    return fail(NVFP4_ERR_MISALIGNED, "token and receive slabs must be 16-byte aligned");
  const int64_t warps = static_cast<int64_t>(world) * tokens * topk;
  const int64_t blocks = std::min<int64_t>((warps + 7) / 8, 148 * 16);
  nvfp4_ep_expand_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      pair_rows, tokens, topk, world, static_cast<const uint8_t*>(tok_codes),
      static_cast<const uint8_t*>(tok_sf), cols, static_cast<uint8_t*>(recv_codes),
      static_cast<uint8_t*>(recv_sf), recv_capacity);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "expand launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_publish_pairs(const int32_t* topk_ids, const int32_t* remote_rows,
                                     const float* weights, int tokens, int topk, int num_experts,
                                     int rank, int world, nvfp4_ep_peers pair_rows,
                                     nvfp4_ep_peers pair_weights, void* stream) {
  g_last_error.clear();
  int st = check_ep_world(num_experts, rank, world);
  if (st != NVFP4_OK) return st;
  if (tokens < 0 || topk <= 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d", tokens, topk);
  if (tokens == 0) return NVFP4_OK;
  if (topk_ids == nullptr || remote_rows == nullptr || weights == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a pair table input is NULL");
  if ((st = check_peers(pair_rows, world, "pair_rows", false)) != NVFP4_OK) return st;
  if ((st = check_peers(pair_weights, world, "pair_weights", false)) != NVFP4_OK) return st;
  const int64_t pairs = static_cast<int64_t>(tokens) * topk;
  const int64_t blocks = std::min<int64_t>((pairs + 255) / 256, 148 * 8);
  nvfp4_ep_publish_pairs_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                                  static_cast<cudaStream_t>(stream)>>>(
      topk_ids, remote_rows, weights, pairs, num_experts, rank, world, to_peers(pair_rows),
      to_peers(pair_weights));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "publish pairs launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_return_sums(const int32_t* pair_rows, const float* pair_weights,
                                   int tokens, int topk, int rank, int world, const void* y,
                                   int64_t ldy, int cols, nvfp4_ep_peers ret, void* stream) {
  g_last_error.clear();
  if (world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "rank %d of world %d (1..%d ranks)", rank, world,
                kEpMaxRanks);
  if (tokens < 0 || topk <= 0 || cols <= 0 || cols % 8 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d cols=%d (cols a multiple of 8)", tokens,
                topk, cols);
  if (tokens == 0) return NVFP4_OK;
  if (pair_rows == nullptr || pair_weights == nullptr || y == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a return-sum buffer is NULL");
  if (!aligned16(y) || ldy % 8 != 0 || ldy < cols)
    return fail(NVFP4_ERR_MISALIGNED, "y 16-byte aligned, ldy a multiple of 8 >= cols");
  int st = check_peers(ret, world, "ret", true);
  if (st != NVFP4_OK) return st;
  const int groups = (cols + 256 * kEpSumParts - 1) / (256 * kEpSumParts);
  const int64_t warps = static_cast<int64_t>(world) * tokens * groups;
  const int64_t blocks = std::min<int64_t>((warps + 7) / 8, 148 * 16);
  nvfp4_ep_return_sums_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                                static_cast<cudaStream_t>(stream)>>>(
      pair_rows, pair_weights, tokens, topk, rank, world, static_cast<const __half*>(y), ldy,
      cols, to_peers(ret));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "return sums launch");
  return NVFP4_OK;
}

NVFP4_API int nvfp4_ep_combine_sums(const int32_t* topk_ids, const int32_t* remote_rows,
                                    int tokens, int topk, int num_experts, int world,
                                    const void* ret, int cols, void* out, int64_t ldo,
                                    void* stream) {
  g_last_error.clear();
  int st = check_ep_world(num_experts, 0, world);
  if (st != NVFP4_OK) return st;
  if (tokens < 0 || topk <= 0 || cols <= 0 || cols % 8 != 0)
    return fail(NVFP4_ERR_BAD_SHAPE, "tokens=%d topk=%d cols=%d (cols a multiple of 8)", tokens,
                topk, cols);
  if (tokens == 0) return NVFP4_OK;
  if (topk_ids == nullptr || remote_rows == nullptr || ret == nullptr || out == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "a combine buffer is NULL");
  if (!aligned16(out) || !aligned16(ret) || ldo % 8 != 0 || ldo < cols)
    return fail(NVFP4_ERR_MISALIGNED, "ret and out 16-byte aligned, ldo a multiple of 8 >= cols");
  const int groups = (cols + 256 * kEpSumParts - 1) / (256 * kEpSumParts);
  // A warp task covers a run of a token's column groups, so the token's owner mask (one
  // round trip to the routing ids) is read once per run; launches with few tokens keep one
  // group per task, so that every SM still gets warps.
  const int per_task = static_cast<int64_t>(tokens) * groups > 148 * 64 ? groups : 1;
  const int64_t warps =
      static_cast<int64_t>(tokens) * ((groups + per_task - 1) / per_task);
  const int64_t blocks = std::min<int64_t>((warps + 7) / 8, 148 * 16);
  nvfp4_ep_combine_sums_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                                 static_cast<cudaStream_t>(stream)>>>(
      topk_ids, remote_rows, tokens, topk, num_experts, world, static_cast<const __half*>(ret),
      cols, static_cast<__nv_bfloat16*>(out), ldo, per_task);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "combine sums launch");
  return NVFP4_OK;
}

}  // extern "C"
