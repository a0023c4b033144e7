// C ABI implementation: host-side validation and scheduling, tensor-map encoding
// (driver encoder, cached per tensor) and upload into the workspace, the
// scale-factor layout converter, and the launch of the persistent tcgen05
// grouped GEMM.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/nvfp4_group_gemm.h"
#include "grouped_gemm_kernel.cuh"
#include "host_common.cuh"
#include "grouped_gemm_pair_kernel.cuh"
#include "grouped_gemm_swap_kernel.cuh"
#include "nvfp4_types.cuh"
#include "sm100_ptx.cuh"

namespace nvfp4 {

// ============================================================================
// Descriptor upload
// ============================================================================
// Copies host-encoded group records and tensor maps (carried in the kernel's
// parameter block) into the workspace, then releases the maps to the
// tensor-map proxy. One warp per group moves the group's 1 KiB of maps in 16-byte
// pieces; lane 0 also writes the record.
__global__ void __launch_bounds__(32) nvfp4_upload_descriptors_kernel(
    const __grid_constant__ UploadParams p) {
  const int gi = blockIdx.x;
  const int lane = threadIdx.x;
  if (gi == 0 && p.zero_counters != nullptr)
    for (int i = lane; i < static_cast<int>(kSplitCounterBytes / 4); i += 32) p.zero_counters[i] = 0;
  if (gi >= p.count) return;
  const int g = p.first_group + gi;
  const uint4* src = reinterpret_cast<const uint4*>(&p.maps[gi][0]);
  uint4* dst = reinterpret_cast<uint4*>(p.maps_out + static_cast<size_t>(g) * kMapsPerGroup);
#pragma unroll
  for (int i = lane; i < kMapsPerGroup * 8; i += 32) dst[i] = src[i];  // 8 maps x 128 B
  if (lane == 0) p.groups_out[g] = p.rec[gi];
  ptx::tensormap_fence_release();
}

// ============================================================================
// Segment launches: group sizes read on the device
// ============================================================================
// One block. Group g multiplies rows [seg_offsets[g], seg_offsets[g] + seg_counts[g]) of
// a slab of `capacity` rows, as the routing step left them in device memory. The kernel
// checks each segment (offset a multiple of 128, inside the slab; a group that fails is
// skipped and kDevErrBadSegment is set), writes the group's m, tiles_m and tile range
// into its record and its first row into seg_rows, and the launch's tile count into the
// workspace header. Tile ranges follow group order: a block-wide exclusive scan of each
// group's tile count, 1024 groups per pass.
constexpr int kSegSetupThreads = 1024;

__global__ void __launch_bounds__(kSegSetupThreads) nvfp4_segments_setup_kernel(
    GroupDev* __restrict__ groups, int num_groups, const int32_t* __restrict__ seg_offsets,
    const int32_t* __restrict__ seg_counts, int capacity, int tile_m, int out_n,
    int32_t* __restrict__ seg_rows, int32_t* __restrict__ total_tiles, uint32_t* error_bits) {
  __shared__ int32_t warp_sums[kSegSetupThreads / 32];
  __shared__ int32_t carry;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < num_groups; base += kSegSetupThreads) {
    const int g = base + static_cast<int>(threadIdx.x);
    int32_t m = 0, off = 0, tiles_m = 1, tiles = 0;
    if (g < num_groups) {
      const int32_t n = groups[g].n;
      const int32_t cnt = seg_counts[g];
      off = seg_offsets[g];
      const bool ok = cnt >= 0 && off >= 0 && off % kBlockM == 0 &&
                      static_cast<int64_t>(off) + cnt <= capacity;
      if (!ok) {
        atomicOr(error_bits, kDevErrBadSegment);
        off = 0;
      } else if (cnt > 0 && n > 0) {
        m = cnt;
        tiles_m = (cnt + tile_m - 1) / tile_m;
        tiles = tiles_m * ((n + out_n - 1) / out_n);
      }
    }
    // Inclusive scan of `tiles` over the block: within each warp, then over warp totals.
    int32_t v = tiles;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t t = __shfl_up_sync(0xffffffffu, v, d);
      if (lane >= d) v += t;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int32_t w = warp_sums[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t t = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += t;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int32_t incl = carry + v + (warp > 0 ? warp_sums[warp - 1] : 0);
    if (g < num_groups) {
      GroupDev& d = groups[g];
      d.m = m;
      d.tiles_m = tiles_m;
      d.tile_start = incl - tiles;
      d.tile_end = incl;
      seg_rows[g] = off;
    }
    __syncthreads();  // every thread has read carry and warp_sums
    if (threadIdx.x == kSegSetupThreads - 1) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total_tiles = carry;
}

// ============================================================================
// Scale-factor layout: plain [rows, cols] -> 128x4 blocks
// ============================================================================
// Output byte ((mm * rest_k + kk) * 32 + i0) * 16 + i1 * 4 + j holds
// plain[mm*128 + i1*32 + i0][kk*4 + j] (zero outside the input), i.e. the
// to_blocked permutation (REFERENCE_IMPL.md:19-42). One thread writes one
// 16-byte row (i0) of a 512-byte block.
__global__ void __launch_bounds__(256) nvfp4_sf_to_blocked_kernel(const uint8_t* __restrict__ plain,
                                                                  uint8_t* __restrict__ blocked,
                                                                  int rows, int cols, int64_t ld,
                                                                  int rest_k, int64_t chunks) {
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < chunks;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i0 = static_cast<int>(idx & 31);
    const int64_t blk = idx >> 5;
    const int kk = static_cast<int>(blk % rest_k);
    const int64_t mm = blk / rest_k;
    uint32_t w[4];
#pragma unroll
    for (int i1 = 0; i1 < 4; ++i1) {
      const int64_t r = mm * 128 + i1 * 32 + i0;
      uint32_t word = 0;
      if (r < rows) {
        const uint8_t* src = plain + r * ld;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = kk * 4 + j;
          if (c < cols) word |= static_cast<uint32_t>(src[c]) << (8 * j);
        }
      }
      w[i1] = word;
    }
    reinterpret_cast<uint4*>(blocked)[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// The same permutation, tiled for rows whose scale bytes come in whole 16-byte chunks
// (sf_cols and ld multiples of 16, both pointers 16-byte aligned): one CTA takes 128 rows x
// 32 blocks' columns (128 bytes of each row), loads them with 16-byte loads (8 lanes per
// row, so every load instruction covers whole rows) into shared memory, and writes the 32
// output blocks -- 16 KiB, contiguous -- one 16-byte output row (i0) per thread. The shared
// copy is kept as 4-byte words with a row stride of 33 words, so that both the stores (rows
// r..r+3, chunks 0..7 per warp) and the loads (i0 = 0..31 of one block per warp) fall on 32
// different banks. The byte-wise kernel above gathers each output row from four plain rows
// one byte at a time and reached about 0.9 TB/s on a B200.
constexpr int kSfTileBlocks = 32;                  // output blocks (4 columns each) per CTA
constexpr int kSfTileStride = kSfTileBlocks + 1;   // words per staged row
__global__ void __launch_bounds__(256) nvfp4_sf_to_blocked_tiled_kernel(
    const uint8_t* __restrict__ plain, uint8_t* __restrict__ blocked, int rows, int cols,
    int64_t ld, int rest_k) {
  __shared__ uint32_t tile[128 * kSfTileStride];
  const int64_t mm = blockIdx.y;
  const int kk0 = static_cast<int>(blockIdx.x) * kSfTileBlocks;
  const int nblk = min(kSfTileBlocks, rest_k - kk0);  // blocks of this tile (>= 1)
  const int t = static_cast<int>(threadIdx.x);
  // Load: row (t / 8) + 32 i, 16-byte chunk t % 8 of this tile's 128 bytes.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = t / 8 + 32 * i;
    const int c = t % 8;
    const int64_t row = mm * 128 + r;
    const int col = kk0 * 4 + c * 16;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < rows && col < cols)
      v = __ldg(reinterpret_cast<const uint4*>(plain + row * ld + col));
    uint32_t* dst = &tile[r * kSfTileStride + c * 4];
    dst[0] = v.x;
    dst[1] = v.y;
    dst[2] = v.z;
    dst[3] = v.w;
  }
  __syncthreads();
  // Store: output row u = (block b, i0) of this tile holds the words of rows i0, 32 + i0,
  // 64 + i0, 96 + i0 in column b.
  uint4* out = reinterpret_cast<uint4*>(blocked + (mm * rest_k + kk0) * kSfBlockBytes);
  for (int u = t; u < nblk * 32; u += blockDim.x) {
    const int b = u / 32;
    const int i0 = u % 32;
    out[u] = make_uint4(tile[i0 * kSfTileStride + b], tile[(32 + i0) * kSfTileStride + b],
                        tile[(64 + i0) * kSfTileStride + b], tile[(96 + i0) * kSfTileStride + b]);
  }
}

// ============================================================================
// Host side
// ============================================================================
thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(NVFP4_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

namespace {

// Kernel variants. Single CTA: <MMA N, gated, stages>; CTA pair: <gated, stages>.
using Kn128 = GemmConfig<128, false, 5>;
using Kn256 = GemmConfig<256, false, 3>;
using Kgated = GemmConfig<256, true, 3>;
using Kstream = GemmConfig<256, false, 4, true>;  // weight-streaming shapes
constexpr int kPairStages = 5 * kPairStagesPerKTile;  // 190 KiB of operands in flight
using Kpair = PairConfig<false, kPairStages>;
using KpairGated = PairConfig<true, kPairStages>;
constexpr int kSwapStages = 7;
using Kswap = SwapConfig<kSwapStages>;

DeviceState g_dev[kMaxDevices];

int max_pair_clusters(const void* fn, int smem, int num_sms) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms, 1, 1);
  cfg.blockDim = dim3(kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();  // clear the error; fall back to pairs of all SMs
    n = num_sms / 2;
  }
  return n;
}

void init_device(int dev, DeviceState& st) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) {
    st.status = NVFP4_ERR_CUDA;
    st.detail = std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e);
    return;
  }
  if (prop.major != 10 || prop.minor != 0) {
    st.status = NVFP4_ERR_UNSUPPORTED_DEVICE;
    char buf[512];
    snprintf(buf, sizeof(buf), "device %d is %.200s (sm_%d%d); this library is built for sm_100a",
             dev, prop.name, prop.major, prop.minor);
    st.detail = buf;
    return;
  }
  st.num_sms = prop.multiProcessorCount;
  struct {
    const void* fn;
    int smem;
  } kernels[] = {
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_kernel<128, false, 5>), Kn128::kSmemBytes},
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_kernel<256, false, 3>), Kn256::kSmemBytes},
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_kernel<256, true, 3>), Kgated::kSmemBytes},
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_kernel<256, false, 4, true>),
       Kstream::kSmemBytes},
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_kernel<256, false, 4, true, true>),
       Kstream::kSmemBytes},
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_pair_kernel<false, kPairStages>),
       Kpair::kSmemBytes},
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_pair_kernel<true, kPairStages>),
       KpairGated::kSmemBytes},
      {reinterpret_cast<const void*>(&nvfp4_grouped_gemm_swap_kernel<kSwapStages>),
       Kswap::kSmemBytes},
  };
  for (auto& k : kernels) {
    e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
    if (e != cudaSuccess) {
      st.status = NVFP4_ERR_CUDA;
      st.detail = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
      return;
    }
  }
  st.pair_clusters = max_pair_clusters(
      reinterpret_cast<const void*>(&nvfp4_grouped_gemm_pair_kernel<false, kPairStages>),
      Kpair::kSmemBytes, st.num_sms);
  st.pair_clusters_gated = max_pair_clusters(
      reinterpret_cast<const void*>(&nvfp4_grouped_gemm_pair_kernel<true, kPairStages>),
      KpairGated::kSmemBytes, st.num_sms);
}

}  // namespace

int current_device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NVFP4_ERR_INVALID_ARGUMENT, "device %d", dev);
  DeviceState& ds = g_dev[dev];
  std::call_once(ds.once, init_device, dev, std::ref(ds));
  if (ds.status != NVFP4_OK) return fail(ds.status, "%s", ds.detail.c_str());

  *out = &ds;
  return NVFP4_OK;
}

namespace {

// cuTensorMapEncodeTiled, resolved once through the runtime (no libcuda link).
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
struct Encoder {
  std::once_flag once;
  EncodeFn fn = nullptr;
};
Encoder g_encoder;

void init_encoder(Encoder& e) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) e.fn = reinterpret_cast<EncodeFn>(fn);
}

// Encoded maps are cached by (kind, address, rows, row elements): weights keep
// their maps across calls, so steady-state calls encode only what changed.
struct MapKey {
  uint64_t addr;
  uint32_t rows;
  uint32_t row_bytes;
  uint32_t kind;
  bool operator==(const MapKey& o) const {
    return addr == o.addr && rows == o.rows && row_bytes == o.row_bytes && kind == o.kind;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = k.addr * 0x9E3779B97F4A7C15ull;
    h ^= (static_cast<uint64_t>(k.rows) << 32 | k.row_bytes) + 0x632BE59BD9B4E019ull + (h << 6);
    return static_cast<size_t>(h ^ (static_cast<uint64_t>(k.kind) << 61));
  }
};
std::mutex g_map_cache_mu;
std::unordered_map<MapKey, TmaDesc, MapKeyHash> g_map_cache;
constexpr size_t kMapCacheMax = 1 << 14;

enum : uint32_t {
  kKindOperand = 0, kKindOutput = 1, kKindScales = 2, kKindOperand64 = 3,
  kKindOperandHalf = 4, kKindScalesHalf = 5
};

// kKindOperand: e2m1 operand [rows, row_elems bytes] (uint8 view), box 128 B x 128 rows,
//   128B swizzle, zero fill outside the tensor; kKindOperand64: the same with 64-row boxes;
//   kKindOperandHalf: box 64 B x 128 rows with the 64B swizzle (pair kernels with half-k-tile
//   stages).
// kKindOutput:  fp16 output [rows, row_elems], box 64 x 32, 128B swizzle.
// kKindScales:  blocked scale bytes as `rows` rows of 128 bytes, box 128 B x 16 rows =
//   one 2-KiB k-tile chunk of a 128-row block, zero fill outside.
bool encode_map_uncached(uint32_t kind, const void* addr, uint32_t rows, uint32_t row_elems,
                         TmaDesc* out) {
  CUtensorMap m;
  cuuint32_t estr[2] = {1, 1};
  CUresult r;
  if (kind == kKindOperand || kind == kKindOperand64 || kind == kKindOperandHalf) {
    const bool half = kind == kKindOperandHalf;
    cuuint64_t dims[2] = {row_elems, rows};
    cuuint64_t strides[1] = {row_elems};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(half ? 64 : kRowBytesPerStage),
                         static_cast<cuuint32_t>(kind == kKindOperand64 ? 64 : kBlockM)};
    r = g_encoder.fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(addr), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     half ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (kind == kKindOutput) {
    cuuint64_t dims[2] = {row_elems, rows};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_elems) * 2u};
    cuuint32_t box[2] = {64, 32};
    r = g_encoder.fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(addr), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {128, rows};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {128, kind == kKindScalesHalf ? 8u : 16u};
    r = g_encoder.fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(addr), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return false;
  memcpy(out, &m, sizeof(TmaDesc));
  return true;
}

bool encode_map(uint32_t kind, const void* addr, uint32_t rows, uint32_t row_elems, TmaDesc* out,
                bool use_cache) {
  if (!use_cache) return encode_map_uncached(kind, addr, rows, row_elems, out);
  const MapKey key{reinterpret_cast<uint64_t>(addr), rows, row_elems, kind};
  {
    std::lock_guard<std::mutex> lk(g_map_cache_mu);
    auto it = g_map_cache.find(key);
    if (it != g_map_cache.end()) {
      *out = it->second;
      return true;
    }
  }
  if (!encode_map_uncached(kind, addr, rows, row_elems, out)) return false;
  std::lock_guard<std::mutex> lk(g_map_cache_mu);
  if (g_map_cache.size() >= kMapCacheMax) g_map_cache.clear();
  g_map_cache.emplace(key, *out);
  return true;
}


// Single-CTA launches hand out tiles dynamically (see kClaimLeadKTiles); building with
// -DNVFP4_DYNAMIC_SCHEDULE=0 restores the static round-robin order.
#ifndef NVFP4_DYNAMIC_SCHEDULE
#define NVFP4_DYNAMIC_SCHEDULE 1
#endif
constexpr bool kDynamicSchedule = NVFP4_DYNAMIC_SCHEDULE != 0;

// Non-gated launches whose non-empty groups average at most this many rows use the
// weight-stationary kernel. Off by default: on the shapes measured (64 experts, N = 1536,
// K = 4096, 8 and 64 rows per expert on average) the single-CTA row tiles were as fast
// or faster (43.3 vs 44.2 us and 55 vs 59 us per call), both being bound by the weight
// stream; the kernel stays available through NVFP4_FLAG_WEIGHT_STATIONARY.
#ifndef NVFP4_SWAP_MAX_AVG_ROWS
#define NVFP4_SWAP_MAX_AVG_ROWS 0
#endif
constexpr int kSwapMaxAvgRows = NVFP4_SWAP_MAX_AVG_ROWS;

// Non-gated 128 x 256 single-CTA launches whose non-empty groups average at most this
// many rows are bound by the weight stream: they use the variant with four pipeline
// stages and register-direct output stores (their C writes are small). Measured per
// call, 4 vs 3 stages: 64 experts x N 1536 x K 4096 with 64 rows each 52.0 vs 53.1 us,
// with 8 rows each 42.0 vs 44.0 us; but 8 groups of 128 rows, N 7168, K 2048, 34.6 vs
// 32.0 us (there the row-per-lane stores of the larger C cost more than the deeper ring
// gains). Taller groups keep the three-stage variant whose TMA stores write whole rows.
#ifndef NVFP4_STREAM_MAX_AVG_ROWS
#define NVFP4_STREAM_MAX_AVG_ROWS 64
#endif
constexpr int kStreamMaxAvgRows = NVFP4_STREAM_MAX_AVG_ROWS;

// Split-K of a single-CTA launch's last partial wave (NVFP4_FLAG_SPLIT_K): at least
// kSplitMinKTiles k-tiles per part. -DNVFP4_SPLIT_K=0 compiles it out.
#ifndef NVFP4_SPLIT_K
#define NVFP4_SPLIT_K 1
#endif
constexpr bool kSplitEnabled = NVFP4_SPLIT_K != 0;
// Stream-K schedule of weight-streaming launches (NVFP4_FLAG_STREAM_K, see
// grouped_gemm_impl); -DNVFP4_STREAM_K=0 compiles the option out.
#ifndef NVFP4_STREAM_K
#define NVFP4_STREAM_K 1
#endif
constexpr bool kStreamK = NVFP4_STREAM_K != 0;
constexpr int kSplitMinKTiles = 2;
static_assert(NVFP4_SPLIT_SCRATCH_BYTES == kSplitScratchBytes, "header and library disagree");

// GEMM kernels are launched with programmatic stream serialization: a launch may be
// scheduled while the previous kernel in the stream is still finishing, and waits
// (griddepcontrol.wait) before reading anything that kernel may have written.
#ifndef NVFP4_PDL
#define NVFP4_PDL 1
#endif

template <typename Kernel>
cudaError_t launch_gemm(Kernel kernel, const GemmParams& gp, int grid, int smem, int cluster,
                        cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (NVFP4_PDL) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, gp);
}

template <int MMA_N, bool GATED, int STAGES, bool DIRECT = false, bool STREAMK = false>
cudaError_t launch_single(const GemmParams& gp, int grid, cudaStream_t stream) {
  using Cfg = GemmConfig<MMA_N, GATED, STAGES, DIRECT>;
  return launch_gemm(nvfp4_grouped_gemm_kernel<MMA_N, GATED, STAGES, DIRECT, STREAMK>, gp, grid,
                     Cfg::kSmemBytes, 1, stream);
}

template <bool GATED>
cudaError_t launch_pair(const GemmParams& gp, int clusters, cudaStream_t stream) {
  using Cfg = PairConfig<GATED, kPairStages>;
  return launch_gemm(nvfp4_grouped_gemm_pair_kernel<GATED, kPairStages>, gp, 2 * clusters,
                     Cfg::kSmemBytes, 2, stream);
}

// Everything a launch needs once descriptors are in the workspace: the kernel variant, its
// grid and its parameters. grouped_gemm_impl builds one per call; a prepared plan
// (nvfp4_plan_create) keeps it and replays only the launch.
enum class KernelKind : int {
  kSwap, kPair, kPairGated, kSingleGated, kSingle128, kStream, kSingle256, kStreamK
};
struct LaunchSpec {
  GemmParams gp;
  KernelKind kind;
  int grid;  // CTAs (single-CTA and swap kernels) or clusters (pair kernels)
};

cudaError_t run_spec(const LaunchSpec& sp, cudaStream_t s) {
  switch (sp.kind) {
    case KernelKind::kSwap:
      return launch_gemm(nvfp4_grouped_gemm_swap_kernel<kSwapStages>, sp.gp, sp.grid,
                         Kswap::kSmemBytes, 1, s);
    case KernelKind::kPair: return launch_pair<false>(sp.gp, sp.grid, s);
    case KernelKind::kPairGated: return launch_pair<true>(sp.gp, sp.grid, s);
    case KernelKind::kSingleGated: return launch_single<256, true, 3>(sp.gp, sp.grid, s);
    case KernelKind::kSingle128: return launch_single<128, false, 5>(sp.gp, sp.grid, s);
    case KernelKind::kStream: return launch_single<256, false, 4, true>(sp.gp, sp.grid, s);
    case KernelKind::kStreamK: return launch_single<256, false, 4, true, true>(sp.gp, sp.grid, s);
    case KernelKind::kSingle256: return launch_single<256, false, 3>(sp.gp, sp.grid, s);
  }
  return cudaErrorInvalidValue;
}

// Row segments of a segment launch (nvfp4_grouped_gemm_segments): device arrays of
// per-group first rows and row counts, and the host's estimate of their total.
struct SegmentArgs {
  const int32_t* offsets;
  const int32_t* counts;
  int64_t expected_rows;
  const nvfp4_segment_output* output;  // nullptr: fp16 rows into c
};

// Shared implementation of the grouped entry points: validate, schedule, encode
// and upload descriptors into `ws`, launch. `rec` holds num_groups records of host
// scratch; `use_cache` selects the cached tensor-map encoder. With `seg`, each group's
// m is the slab's row count and the rows it multiplies are read on the device.
// `clear_header` zeroes the workspace header (error word, tile counters) on `s` once the
// table has passed every host-side check, before anything is uploaded or launched.
int grouped_gemm_impl(const nvfp4_group* groups, int num_groups, unsigned int flags, uint8_t* ws,
                      size_t ws_bytes, cudaStream_t s, GroupDev* rec, bool use_cache,
                      const SegmentArgs* seg = nullptr, LaunchSpec* prepared = nullptr,
                      bool clear_header = false, const int64_t* replica_offsets = nullptr,
                      int num_replicas = 0) {
  const bool gated = (flags & NVFP4_FLAG_GATED) != 0;
  // Tile shape: CTA pairs (256-row tiles) when the groups are tall enough to fill
  // them, single CTAs (128-row tiles) otherwise; 256 MMA columns unless asked otherwise.
  int64_t rows = 0, active = 0;  // rows and count of the non-empty groups
  int max_k = 0;
  for (int i = 0; i < num_groups; ++i)
    if (groups[i].m > 0 && groups[i].n > 0) {
      rows += groups[i].m;
      ++active;
      max_k = std::max(max_k, groups[i].k);
    }
  if (seg != nullptr) {
    // The rows are on the device: choose the kernel from the caller's estimate (or the
    // slab), and never the weight-stationary or split-K variants.
    rows = seg->expected_rows > 0 ? seg->expected_rows : (num_groups > 0 ? groups[0].m : 0);
    flags &= ~NVFP4_FLAG_SPLIT_K;
  }
  bool pair = false;
  bool swap = (flags & NVFP4_FLAG_WEIGHT_STATIONARY) != 0 && seg == nullptr;
  if (!swap && (flags & NVFP4_FLAG_TILE_N128) == 0 && (flags & NVFP4_FLAG_SINGLE_CTA) == 0) {
    if (flags & NVFP4_FLAG_CTA_PAIR) {
      pair = true;
    } else {
      // Pairs pay off when the groups fill most of a 256-row tile, or when K is long
      // enough that the halved B traffic outweighs the padding of 128-255-row groups
      // (measured per call, pair vs single CTA: G=8, M 64-248, K=7168 -> 43.2 vs 51.2 us;
      // G=8, M 40-196, N=7168, K=2048 -> 30.7 vs 32.8 us).
      pair = active > 0 && (rows >= 192 * active || (rows >= 96 * active && max_k >= 2048));
      // Small groups: weight-stationary tiles carry no padding rows (non-gated launches
      // without a forced tile width).
      swap = !pair && !gated && seg == nullptr && (flags & NVFP4_FLAG_TILE_N256) == 0 &&
             active > 0 && rows <= static_cast<int64_t>(kSwapMaxAvgRows) * active;
    }
  }
  if (num_replicas > 0) swap = false;  // the weight-stationary kernel has no replicated output
  int mma_n = gated ? 256 : ((flags & NVFP4_FLAG_TILE_N128) ? 128 : 256);
  int out_n = swap ? 128 : (gated ? 128 : mma_n);
  int tile_m = swap ? Kswap::kTokens : (pair ? 256 : kBlockM);
  // Tile shape chosen by the library (no tile or kernel flag): it may still switch to
  // 128 x 128 tiles below, once the device's size is known.
  const bool auto_shape =
      !gated && seg == nullptr &&
      (flags & (NVFP4_FLAG_TILE_N128 | NVFP4_FLAG_TILE_N256 | NVFP4_FLAG_SINGLE_CTA |
                NVFP4_FLAG_CTA_PAIR | NVFP4_FLAG_WEIGHT_STATIONARY | NVFP4_FLAG_SPLIT_K)) == 0;

  int64_t total_tiles = 0;
  for (int i = 0; i < num_groups; ++i) {
    const nvfp4_group& gr = groups[i];
    if (gr.m < 0 || gr.n < 0 || gr.k < 0)
      return fail(NVFP4_ERR_BAD_SHAPE, "group %d: negative size (m=%d n=%d k=%d)", i, gr.m, gr.n, gr.k);
    GroupDev& d = rec[i];
    memset(&d, 0, sizeof(d));
    d.m = gr.m;
    d.n = gr.n;
    d.k = gr.k;
    d.alpha = gr.alpha;
    d.alpha2 = gr.alpha2;
    d.tiles_m = 1;
    d.tile_start = d.tile_end = static_cast<int32_t>(total_tiles);
    if (gr.m == 0 || gr.n == 0) continue;
    if (gr.k <= 0 || gr.k % kBlockK != 0)
      return fail(NVFP4_ERR_BAD_SHAPE, "group %d: k=%d must be a positive multiple of 256", i, gr.k);
    if (gr.n % 8 != 0)
      return fail(NVFP4_ERR_BAD_SHAPE, "group %d: n=%d must be a multiple of 8", i, gr.n);
    const void* ptrs[7] = {gr.a, gr.b, gr.b2, gr.sfa, gr.sfb, gr.sfb2, gr.c};
    const char* names[7] = {"a", "b", "b2", "sfa", "sfb", "sfb2", "c"};
    for (int j = 0; j < 7; ++j) {
      if (!gated && (j == 2 || j == 5)) continue;
      if (ptrs[j] == nullptr) return fail(NVFP4_ERR_NULL_POINTER, "group %d: %s is NULL", i, names[j]);
      if (!aligned16(ptrs[j]))
        return fail(NVFP4_ERR_MISALIGNED, "group %d: %s not 16-byte aligned", i, names[j]);
    }
    d.sfa = static_cast<const uint8_t*>(gr.sfa);
    d.sfb = static_cast<const uint8_t*>(gr.sfb);
    d.sfb2 = gated ? static_cast<const uint8_t*>(gr.sfb2) : nullptr;
    d.c = static_cast<uint8_t*>(gr.c);
    d.tiles_m = (gr.m + tile_m - 1) / tile_m;
    total_tiles += static_cast<int64_t>(d.tiles_m) * ((gr.n + out_n - 1) / out_n);
    if (total_tiles > (int64_t{1} << 30))
      return fail(NVFP4_ERR_BAD_SHAPE, "too many tiles (%lld)", static_cast<long long>(total_tiles));
    d.tile_end = static_cast<int32_t>(total_tiles);
  }
  if (total_tiles == 0) return NVFP4_OK;

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NVFP4_ERR_INVALID_ARGUMENT, "device %d", dev);
  DeviceState& ds = g_dev[dev];
  std::call_once(ds.once, init_device, dev, std::ref(ds));
  if (ds.status != NVFP4_OK) return fail(ds.status, "%s", ds.detail.c_str());

  // Launches too small to give every SM (or CTA pair) a tile are bound by the latency of
  // one tile's k-loop: when 128 x 128 tiles fit in one wave they halve each SM's MMA work
  // per tile and use more SMs (measured per call, auto shape vs 128 x 128: M=128, N=256,
  // K=512 12.3 vs 10.3 us; G=2, M 192/320, N 3072, K 4096 18.4 vs 16.4 us; G=2, M 128/384,
  // N 4096, K 1536 14.3 vs 13.4 us).
  if (auto_shape && !swap && (pair ? total_tiles < ds.pair_clusters : total_tiles < ds.num_sms)) {
    int64_t small_tiles = 0;
    for (int i = 0; i < num_groups; ++i)
      if (rec[i].tile_end > rec[i].tile_start)
        small_tiles += static_cast<int64_t>((groups[i].m + kBlockM - 1) / kBlockM) *
                       ((groups[i].n + 127) / 128);
    if (small_tiles <= ds.num_sms) {
      pair = false;
      mma_n = out_n = 128;
      tile_m = kBlockM;
      total_tiles = 0;  // the same tile bookkeeping as above, for the new tile shape
      for (int i = 0; i < num_groups; ++i) {
        GroupDev& d = rec[i];
        d.tiles_m = 1;
        d.tile_start = static_cast<int32_t>(total_tiles);
        if (groups[i].m > 0 && groups[i].n > 0) {
          d.tiles_m = (groups[i].m + tile_m - 1) / tile_m;
          total_tiles += static_cast<int64_t>(d.tiles_m) * ((groups[i].n + out_n - 1) / out_n);
        }
        d.tile_end = static_cast<int32_t>(total_tiles);
      }
    }
  }
  std::call_once(g_encoder.once, init_encoder, std::ref(g_encoder));
  if (g_encoder.fn == nullptr)
    return fail(NVFP4_ERR_DRIVER, "cuTensorMapEncodeTiled entry point not available from the driver");

  GroupDev* groups_dev = reinterpret_cast<GroupDev*>(ws + ws_groups_offset());
  TmaDesc* maps_dev = reinterpret_cast<TmaDesc*>(ws + ws_maps_offset(num_groups));

  if (clear_header) {
    e = cudaMemsetAsync(ws, 0, offsetof(WorkspaceHeader, reserved), s);
    if (e != cudaSuccess) return cuda_fail(e, "clear workspace header");
  }

  if ((flags & NVFP4_FLAG_REUSE_DESCRIPTORS) == 0) {
    static thread_local UploadParams up;  // ~26 KB: kept off the caller's stack
    up.groups_out = groups_dev;
    up.maps_out = maps_dev;
    // Split-K counters move with the group count: zero them with every new table (when the
    // workspace has the split scratch at all).
    const bool has_split_scratch = ws_bytes >= ws_split_offset(num_groups) + kSplitScratchBytes;
    up.zero_counters = has_split_scratch
                           ? reinterpret_cast<int32_t*>(ws + ws_split_offset(num_groups))
                           : nullptr;
    for (int first = 0; first < num_groups; first += kGroupsPerUpload) {
      const int count = std::min(kGroupsPerUpload, num_groups - first);
      up.first_group = first;
      up.count = count;
      for (int gi = 0; gi < count; ++gi) {
        const int i = first + gi;
        const nvfp4_group& gr = groups[i];
        up.rec[gi] = rec[i];
        TmaDesc* mp = up.maps[gi];
        memset(mp, 0, sizeof(TmaDesc) * kMapsPerGroup);
        if (rec[i].tile_end == rec[i].tile_start) continue;  // empty group: maps never read
        const uint32_t kb = static_cast<uint32_t>(gr.k / 2);
        // Blocked scale bytes of an R-row operand, in rows of 128 bytes.
        const uint32_t sfa_rows = static_cast<uint32_t>(((gr.m + 127) / 128) * (gr.k / 64) * 4);
        const uint32_t sfb_rows = static_cast<uint32_t>(((gr.n + 127) / 128) * (gr.k / 64) * 4);
        // Pair kernels with half-k-tile stages load A/B through 64-byte boxes and scales in
        // 1-KiB chunks; every other kernel uses whole-k-tile boxes.
        const bool half = pair && kPairStagesPerKTile == 2;
        const uint32_t opk = half ? kKindOperandHalf : kKindOperand;
        const uint32_t sfk = half ? kKindScalesHalf : kKindScales;
        bool ok = encode_map(opk, gr.a, gr.m, kb, &mp[kMapA], use_cache) &&
                  encode_map(opk, gr.b, gr.n, kb, &mp[kMapB], use_cache) &&
                  encode_map(kKindOutput, gr.c, gr.m, gr.n, &mp[kMapC], use_cache) &&
                  encode_map(sfk, gr.sfa, sfa_rows, 128, &mp[kMapSfa], use_cache) &&
                  encode_map(sfk, gr.sfb, sfb_rows, 128, &mp[kMapSfb], use_cache) &&
                  (!gated ||
                   (encode_map(opk, gr.b2, gr.n, kb, &mp[kMapB2], use_cache) &&
                    encode_map(sfk, gr.sfb2, sfb_rows, 128, &mp[kMapSfb2], use_cache))) &&
                  // 64-row A boxes: the weight-stationary kernel's token tiles, and the
                  // weight-streaming kernel's tiles of at most 64 rows.
                  (!(swap || (!pair && !gated)) ||
                   encode_map(kKindOperand64, gr.a, gr.m, kb, &mp[kMapA64], use_cache));
        if (!ok) return fail(NVFP4_ERR_DRIVER, "group %d: cuTensorMapEncodeTiled rejected a tensor", i);
      }
      nvfp4_upload_descriptors_kernel<<<count, 32, 0, s>>>(up);
      up.zero_counters = nullptr;  // once per table
      e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(e, "descriptor upload launch");
    }
  }

  GemmParams gp;
  gp.num_replicas = num_replicas;
  for (int i = 0; i < kMaxReplicas; ++i)
    gp.replica_offset[i] = i < num_replicas ? replica_offsets[i] : 0;
  gp.seg_rows = nullptr;
  gp.seg_total_tiles = nullptr;
  const nvfp4_segment_output* out = seg != nullptr ? seg->output : nullptr;
  gp.out_sf = out != nullptr ? static_cast<uint8_t*>(out->sf) : nullptr;
  gp.out_scale = out != nullptr ? out->scale : 0.0f;
  gp.out_d6 = 6.0f * gp.out_scale;
  gp.row_dest = out != nullptr ? out->row_dest : nullptr;
  for (int i = 0; i < 8; ++i)
    gp.dest_base[i] = out != nullptr ? static_cast<uint8_t*>(out->dest_base[i]) : nullptr;
  gp.dest_ld = out != nullptr ? out->dest_ld : 0;
  if (seg != nullptr) {
    int32_t* seg_rows = reinterpret_cast<int32_t*>(ws + ws_seg_rows_offset(num_groups));
    int32_t* seg_total = &reinterpret_cast<WorkspaceHeader*>(ws)->seg_total_tiles;
    nvfp4_segments_setup_kernel<<<1, kSegSetupThreads, 0, s>>>(
        groups_dev, num_groups, seg->offsets, seg->counts, groups[0].m, tile_m, out_n, seg_rows,
        seg_total, reinterpret_cast<uint32_t*>(ws));
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "segment set-up launch");
    gp.seg_rows = seg_rows;
    gp.seg_total_tiles = seg_total;
  }
  gp.groups = groups_dev;
  gp.maps = maps_dev;
  gp.error_bits = reinterpret_cast<uint32_t*>(ws);
  gp.num_groups = num_groups;
  gp.total_tiles = static_cast<int32_t>(total_tiles);
  gp.diag_skip_mma = (flags & NVFP4_FLAG_DIAG_SKIP_MMA) ? 1 : 0;
  gp.dynamic_schedule = (!pair && kDynamicSchedule) ? 1 : 0;  // single-CTA kernels only
  gp.tile_counter = reinterpret_cast<WorkspaceHeader*>(ws)->tile_counter;
  // Split-K of the last partial wave (single-CTA row tiles, when the workspace has room).
  int split_parts = 1;
  int64_t tail = 0;
  if (!pair && !swap && kSplitEnabled && (flags & NVFP4_FLAG_SPLIT_K) &&
      ws_bytes >= ws_split_offset(num_groups) + kSplitScratchBytes) {
    const int64_t sms = ds.num_sms;
    tail = total_tiles >= sms ? total_tiles % sms : total_tiles;
    int min_ktiles = 1 << 30;
    for (int i = 0; i < num_groups; ++i)
      if (rec[i].tile_end > rec[i].tile_start) min_ktiles = std::min(min_ktiles, rec[i].k / kBlockK);
    if (tail > 0) {
      int64_t parts = sms / tail;
      parts = std::min<int64_t>(parts, min_ktiles / kSplitMinKTiles);
      parts = std::min<int64_t>(parts, kSplitMaxSlots / tail);
      if (parts >= 2) split_parts = static_cast<int>(parts);
    }
  }
  gp.split_parts = split_parts;
  gp.split_first_tile = static_cast<int32_t>(split_parts > 1 ? total_tiles - tail : total_tiles);
  gp.total_units = static_cast<int32_t>(gp.split_first_tile + (total_tiles - gp.split_first_tile) *
                                                                  split_parts);
  gp.split_counters = reinterpret_cast<int32_t*>(ws + ws_split_offset(num_groups));
  gp.split_partials = reinterpret_cast<float*>(ws + ws_split_offset(num_groups) + kSplitCounterBytes);
  LaunchSpec sp;
  sp.gp = gp;
  if (swap) {
    sp.kind = KernelKind::kSwap;
    sp.grid = static_cast<int>(std::min<int64_t>(total_tiles, ds.num_sms));
  } else if (pair) {
    const int max_clusters = gated ? ds.pair_clusters_gated : ds.pair_clusters;
    sp.kind = gated ? KernelKind::kPairGated : KernelKind::kPair;
    sp.grid = static_cast<int>(std::min<int64_t>(total_tiles, max_clusters));
  } else {
    sp.grid = static_cast<int>(std::min<int64_t>(gp.total_units, ds.num_sms));
    if (gated)
      sp.kind = KernelKind::kSingleGated;
    else if (mma_n == 128)
      sp.kind = KernelKind::kSingle128;
    else if (rows <= static_cast<int64_t>(kStreamMaxAvgRows) * active && gp.row_dest == nullptr)
      sp.kind = KernelKind::kStream;  // weight-streaming shapes
    else
      sp.kind = KernelKind::kSingle256;
  }
  // A grid with a CTA for every unit needs no tile claims (and so no launch-wide counter
  // to reset at exit, which sits on the critical path of one-tile launches).
  if (sp.gp.dynamic_schedule && sp.gp.total_units <= sp.grid) sp.gp.dynamic_schedule = 0;
  sp.gp.stream_k_iters = 0;
  sp.gp.stream_k_ktiles = 0;
  sp.gp.stream_k_total_iters = 0;
  sp.gp.stream_k_first_tile = 0;
  if ((flags & NVFP4_FLAG_STREAM_K) && sp.kind == KernelKind::kStream && kStreamK &&
      split_parts == 1 && seg == nullptr &&
      ws_bytes >= ws_split_offset(num_groups) + kSplitScratchBytes) {
    // Stream-K: weight-streaming launches are bound by the weight bytes every SM pulls, so
    // a last wave that only some SMs run costs nearly a whole tile's time. All but the last
    // full wave of tiles stay whole (round robin); the last full wave and the partial one
    // are shared out as equal k-iteration ranges, one per CTA; a tile cut by a range
    // boundary is finished by the second of its two CTAs. Needs one K for all groups, at
    // least one full wave (the ranges are then at least one tile long, so a tile spans at
    // most two CTAs) and the split scratch for the cut tiles' fp32 rows. Opt-in
    // (NVFP4_FLAG_STREAM_K): on 64 experts, N 1536, K 4096 it measured 64.2 us per call
    // against 53.0 us with dynamic tile claims, because a tile's cost is not its k-iteration
    // count (m-tiles whose weight tile a neighbour already brought into L2 run much faster)
    // and claims follow the real cost. Ranges over all tiles were slower still (71.8 us):
    // each CTA then ran the m-tiles of a group one after another instead of with its
    // neighbours, which lost the sharing of weight tiles in L2.
    int kt = 0;
    bool uniform = true;
    for (int i = 0; i < num_groups; ++i) {
      if (rec[i].tile_end == rec[i].tile_start) continue;
      const int kti = rec[i].k / kBlockK;
      if (kt == 0) kt = kti; else if (kti != kt) uniform = false;
    }
    const int64_t sms = ds.num_sms;
    const int64_t full = total_tiles / sms;
    if (uniform && kt > 0 && full >= 1 && total_tiles % sms != 0) {
      const int64_t first = (full - 1) * sms;  // whole tiles, round robin
      const int64_t iters = (total_tiles - first) * kt;
      const int64_t w = (iters + sms - 1) / sms;  // >= kt: at least sms tiles are shared out
      sp.gp.stream_k_iters = static_cast<int32_t>(w);
      sp.gp.stream_k_ktiles = kt;
      sp.gp.stream_k_total_iters = iters;
      sp.gp.stream_k_first_tile = static_cast<int32_t>(first);
      sp.gp.dynamic_schedule = 0;
      sp.grid = static_cast<int>(sms);
      sp.kind = KernelKind::kStreamK;
    }
  }
  if (prepared != nullptr) {  // a plan: descriptors uploaded, the launch is replayed later
    *prepared = sp;
    return NVFP4_OK;
  }
  e = run_spec(sp, s);
  if (e != cudaSuccess) return cuda_fail(e, "grouped GEMM launch");
  return NVFP4_OK;
}

int check_common_args(const nvfp4_group* groups, int num_groups, unsigned int flags) {
  const unsigned known = NVFP4_FLAG_GATED | NVFP4_FLAG_TILE_N128 | NVFP4_FLAG_TILE_N256 |
                         NVFP4_FLAG_REUSE_DESCRIPTORS | NVFP4_FLAG_CTA_PAIR |
                         NVFP4_FLAG_SINGLE_CTA | NVFP4_FLAG_DIAG_SKIP_MMA |
                         NVFP4_FLAG_WEIGHT_STATIONARY | NVFP4_FLAG_SPLIT_K |
                         NVFP4_FLAG_STREAM_K;
  if (flags & ~known) return fail(NVFP4_ERR_INVALID_ARGUMENT, "unknown flag bits 0x%x", flags & ~known);
  if (num_groups < 0) return fail(NVFP4_ERR_INVALID_ARGUMENT, "num_groups=%d", num_groups);
  if (num_groups > 0 && groups == nullptr)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "groups table is NULL");
  if ((flags & NVFP4_FLAG_TILE_N128) && (flags & NVFP4_FLAG_TILE_N256))
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "TILE_N128 and TILE_N256 are exclusive");
  if ((flags & NVFP4_FLAG_CTA_PAIR) && (flags & NVFP4_FLAG_SINGLE_CTA))
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "CTA_PAIR and SINGLE_CTA are exclusive");
  if ((flags & NVFP4_FLAG_CTA_PAIR) && (flags & NVFP4_FLAG_TILE_N128))
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "CTA pairs use 256-column tiles");
  if ((flags & NVFP4_FLAG_GATED) && (flags & NVFP4_FLAG_TILE_N128))
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "gated launches use 128 gate + 128 up columns");
  if ((flags & NVFP4_FLAG_WEIGHT_STATIONARY) &&
      (flags & (NVFP4_FLAG_GATED | NVFP4_FLAG_TILE_N128 | NVFP4_FLAG_TILE_N256 |
                NVFP4_FLAG_CTA_PAIR | NVFP4_FLAG_SINGLE_CTA)))
    return fail(NVFP4_ERR_INVALID_ARGUMENT,
                "the weight-stationary kernel is non-gated with its own tile shape");
  return NVFP4_OK;
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

NVFP4_API int nvfp4_abi_version(void) { return NVFP4_ABI_VERSION; }

NVFP4_API const char* nvfp4_strerror(int status) {
  switch (status) {
    case NVFP4_OK: return "success";
    case NVFP4_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NVFP4_ERR_BAD_SHAPE: return "unsupported problem shape";
    case NVFP4_ERR_MISALIGNED: return "tensor address not 16-byte aligned";
    case NVFP4_ERR_NULL_POINTER: return "null tensor pointer";
    case NVFP4_ERR_WORKSPACE: return "workspace missing, too small or misaligned";
    case NVFP4_ERR_CUDA: return "CUDA error";
    case NVFP4_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case NVFP4_ERR_UNSUPPORTED_DEVICE: return "unsupported device (needs sm_100)";
    case NVFP4_ERR_DRIVER: return "driver entry point unavailable";
    default: return "unknown status";
  }
}

NVFP4_API const char* nvfp4_last_error_detail(void) { return g_last_error.c_str(); }

NVFP4_API size_t nvfp4_workspace_size(int num_groups) {
  if (num_groups < 0) return 0;
  return ws_total_bytes(num_groups);
}

NVFP4_API size_t nvfp4_sf_blocked_size(int rows, int sf_cols) {
  if (rows <= 0 || sf_cols <= 0) return 0;
  const size_t rest_m = (static_cast<size_t>(rows) + 127) / 128;
  const size_t rest_k = (static_cast<size_t>(sf_cols) + 3) / 4;
  return rest_m * rest_k * kSfBlockBytes;
}

NVFP4_API int nvfp4_sf_to_blocked(const void* plain, void* blocked, int rows, int sf_cols,
                                  int64_t ld, void* stream) {
  g_last_error.clear();
  if (rows < 0 || sf_cols < 0) return fail(NVFP4_ERR_BAD_SHAPE, "rows=%d sf_cols=%d", rows, sf_cols);
  if (rows == 0 || sf_cols == 0) return NVFP4_OK;
  if (plain == nullptr || blocked == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "plain or blocked pointer is NULL");
  if (ld < sf_cols) return fail(NVFP4_ERR_INVALID_ARGUMENT, "ld=%lld < sf_cols=%d",
                                static_cast<long long>(ld), sf_cols);
  if (!aligned16(blocked)) return fail(NVFP4_ERR_MISALIGNED, "blocked output not 16-byte aligned");
  const int rest_m = (rows + 127) / 128;
  const int rest_k = (sf_cols + 3) / 4;
  if (sf_cols % 16 == 0 && ld % 16 == 0 && aligned16(plain) && rest_m <= 65535) {
    const dim3 grid((rest_k + kSfTileBlocks - 1) / kSfTileBlocks, rest_m);
    nvfp4_sf_to_blocked_tiled_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(plain), static_cast<uint8_t*>(blocked), rows, sf_cols, ld,
        rest_k);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "sf_to_blocked launch");
    return NVFP4_OK;
  }
  const int64_t chunks = static_cast<int64_t>(rest_m) * rest_k * 32;
  const int threads = 256;
  int64_t blocks = (chunks + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  nvfp4_sf_to_blocked_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                               static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(plain), static_cast<uint8_t*>(blocked), rows, sf_cols, ld, rest_k,
      chunks);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "sf_to_blocked launch");
  return NVFP4_OK;
}

}  // extern "C"

extern "C" {

NVFP4_API int nvfp4_workspace_check(void* workspace, void* stream, unsigned int* device_error_bits) {
  g_last_error.clear();
  if (device_error_bits) *device_error_bits = 0;
  if (workspace == nullptr) return fail(NVFP4_ERR_WORKSPACE, "workspace is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t bits = 0;
  e = cudaMemcpy(&bits, workspace, sizeof(bits), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read workspace error word");
  if (bits != 0) {
    const uint32_t zero = 0;
    e = cudaMemcpy(workspace, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "clear workspace error word");
    if (device_error_bits) *device_error_bits = bits;
    if (bits & kDevErrTimeouts)
      return fail(NVFP4_ERR_DEVICE_TIMEOUT, "device error bits 0x%x", bits);
    return fail(NVFP4_ERR_BAD_SHAPE,
                "device error bits 0x%x: a device-side row segment was out of range (skipped)",
                bits);
  }
  return NVFP4_OK;
}

NVFP4_API int nvfp4_grouped_gemm(const nvfp4_group* groups, int num_groups, unsigned int flags,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  int st = check_common_args(groups, num_groups, flags);
  if (st != NVFP4_OK || num_groups == 0) return st;
  if (workspace == nullptr) return fail(NVFP4_ERR_WORKSPACE, "workspace is NULL");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(NVFP4_ERR_WORKSPACE, "workspace not 256-byte aligned");
  if (workspace_bytes < ws_total_bytes(num_groups))
    return fail(NVFP4_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes,
                ws_total_bytes(num_groups));
  std::vector<GroupDev> rec(static_cast<size_t>(num_groups));
  return grouped_gemm_impl(groups, num_groups, flags, static_cast<uint8_t*>(workspace),
                           workspace_bytes, static_cast<cudaStream_t>(stream), rec.data(),
                           /*use_cache=*/true);
}

NVFP4_API int nvfp4_grouped_gemm_replicated(const nvfp4_group* groups, int num_groups,
                                            unsigned int flags, void* workspace,
                                            size_t workspace_bytes,
                                            const int64_t* replica_offsets, int num_replicas,
                                            void* stream) {
  g_last_error.clear();
  int st = check_common_args(groups, num_groups, flags);
  if (st != NVFP4_OK) return st;
  if (num_replicas < 1 || num_replicas > kMaxReplicas)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "num_replicas=%d outside [1, %d]", num_replicas,
                kMaxReplicas);
  if (replica_offsets == nullptr) return fail(NVFP4_ERR_NULL_POINTER, "replica_offsets is NULL");
  for (int i = 0; i < num_replicas; ++i)
    if (replica_offsets[i] == 0 || (replica_offsets[i] & 15) != 0)
      return fail(NVFP4_ERR_MISALIGNED,
                  "replica %d: offset %lld must be a non-zero multiple of 16 bytes", i,
                  static_cast<long long>(replica_offsets[i]));
  if (flags & NVFP4_FLAG_WEIGHT_STATIONARY)
    return fail(NVFP4_ERR_INVALID_ARGUMENT,
                "replicated output is not available with NVFP4_FLAG_WEIGHT_STATIONARY");
  if (num_groups == 0) return NVFP4_OK;
  if (workspace == nullptr) return fail(NVFP4_ERR_WORKSPACE, "workspace is NULL");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(NVFP4_ERR_WORKSPACE, "workspace not 256-byte aligned");
  if (workspace_bytes < ws_total_bytes(num_groups))
    return fail(NVFP4_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes,
                ws_total_bytes(num_groups));
  std::vector<GroupDev> rec(static_cast<size_t>(num_groups));
  return grouped_gemm_impl(groups, num_groups, flags, static_cast<uint8_t*>(workspace),
                           workspace_bytes, static_cast<cudaStream_t>(stream), rec.data(),
                           /*use_cache=*/true, /*seg=*/nullptr, /*prepared=*/nullptr,
                           /*clear_header=*/false, replica_offsets, num_replicas);
}

}  // extern "C"

struct nvfp4_plan {
  LaunchSpec spec;
  int device;
};

extern "C" {

NVFP4_API int nvfp4_plan_create(const nvfp4_group* groups, int num_groups, unsigned int flags,
                                void* workspace, size_t workspace_bytes, void* stream,
                                nvfp4_plan** plan) {
  g_last_error.clear();
  if (plan == nullptr) return fail(NVFP4_ERR_INVALID_ARGUMENT, "plan is NULL");
  *plan = nullptr;
  if (flags & (NVFP4_FLAG_REUSE_DESCRIPTORS | NVFP4_FLAG_SPLIT_K))
    return fail(NVFP4_ERR_INVALID_ARGUMENT,
                "a plan uploads its own descriptors and does not split K");
  int st = check_common_args(groups, num_groups, flags);
  if (st != NVFP4_OK) return st;
  if (num_groups == 0) return fail(NVFP4_ERR_BAD_SHAPE, "a plan needs at least one group");
  if (workspace == nullptr) return fail(NVFP4_ERR_WORKSPACE, "workspace is NULL");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(NVFP4_ERR_WORKSPACE, "workspace not 256-byte aligned");
  if (workspace_bytes < ws_total_bytes(num_groups))
    return fail(NVFP4_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes,
                ws_total_bytes(num_groups));
  std::vector<GroupDev> rec(static_cast<size_t>(num_groups));
  nvfp4_plan* p = new nvfp4_plan();
  p->spec.grid = 0;  // no tiles at all: launching does nothing
  st = grouped_gemm_impl(groups, num_groups, flags, static_cast<uint8_t*>(workspace),
                         workspace_bytes, static_cast<cudaStream_t>(stream), rec.data(),
                         /*use_cache=*/true, nullptr, &p->spec);
  cudaError_t e = cudaSuccess;
  if (st == NVFP4_OK && (e = cudaGetDevice(&p->device)) != cudaSuccess)
    st = cuda_fail(e, "cudaGetDevice");
  if (st != NVFP4_OK) {
    delete p;
    return st;
  }
  *plan = p;
  return NVFP4_OK;
}

NVFP4_API int nvfp4_plan_launch(const nvfp4_plan* plan, void* stream) {
  if (plan == nullptr) return fail(NVFP4_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (plan->spec.grid == 0) return NVFP4_OK;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != plan->device)
    return fail(NVFP4_ERR_INVALID_ARGUMENT, "plan made on device %d, current device %d",
                plan->device, dev);
  const cudaError_t e = run_spec(plan->spec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "grouped GEMM launch");
  return NVFP4_OK;
}

NVFP4_API void nvfp4_plan_destroy(nvfp4_plan* plan) { delete plan; }

NVFP4_API int nvfp4_grouped_gemm_segments(const nvfp4_group* groups, int num_groups,
                                          unsigned int flags, const int32_t* seg_offsets,
                                          const int32_t* seg_counts, int64_t expected_rows,
                                          const nvfp4_segment_output* output, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  int st = check_common_args(groups, num_groups, flags);
  if (st != NVFP4_OK || num_groups == 0) return st;
  if (flags & (NVFP4_FLAG_WEIGHT_STATIONARY | NVFP4_FLAG_SPLIT_K))
    return fail(NVFP4_ERR_INVALID_ARGUMENT,
                "segment launches use row tiles without split-K");
  if (seg_offsets == nullptr || seg_counts == nullptr)
    return fail(NVFP4_ERR_NULL_POINTER, "seg_offsets or seg_counts is NULL");
  if ((reinterpret_cast<uintptr_t>(seg_offsets) & 3u) || (reinterpret_cast<uintptr_t>(seg_counts) & 3u))
    return fail(NVFP4_ERR_MISALIGNED, "seg_offsets and seg_counts must be 4-byte aligned");
  if (output != nullptr && output->sf != nullptr) {
    if ((flags & NVFP4_FLAG_GATED) == 0)
      return fail(NVFP4_ERR_INVALID_ARGUMENT, "NVFP4 output needs NVFP4_FLAG_GATED");
    if (!(output->scale > 0.0f) || !std::isfinite(output->scale))
      return fail(NVFP4_ERR_INVALID_ARGUMENT, "output scale must be finite and > 0");
    if (!aligned16(output->sf)) return fail(NVFP4_ERR_MISALIGNED, "output sf not 16-byte aligned");
    for (int i = 0; i < num_groups; ++i)
      if (groups[i].n % 64 != 0)
        return fail(NVFP4_ERR_BAD_SHAPE,
                    "group %d: n=%d must be a multiple of 64 for NVFP4 output", i, groups[i].n);
  }
  if (output != nullptr && output->row_dest != nullptr) {
    if (flags & NVFP4_FLAG_GATED)
      return fail(NVFP4_ERR_INVALID_ARGUMENT, "scattered output is for non-gated launches");
    if ((reinterpret_cast<uintptr_t>(output->row_dest) & 7u) != 0 || output->dest_ld % 16 != 0)
      return fail(NVFP4_ERR_MISALIGNED, "row_dest 8-byte aligned and dest_ld a multiple of 16");
    int nmax = 0;
    for (int i = 0; i < num_groups; ++i) nmax = std::max(nmax, groups[i].n);
    if (output->dest_ld < static_cast<int64_t>(nmax) * 2)
      return fail(NVFP4_ERR_INVALID_ARGUMENT, "dest_ld=%lld < 2 * n",
                  static_cast<long long>(output->dest_ld));
    for (int i = 0; i < NVFP4_EP_MAX_RANKS; ++i)
      if (output->dest_base[i] != nullptr && !aligned16(output->dest_base[i]))
        return fail(NVFP4_ERR_MISALIGNED, "dest_base[%d] not 16-byte aligned", i);
  }
  for (int i = 1; i < num_groups; ++i)
    if (groups[i].m != groups[0].m)
      return fail(NVFP4_ERR_BAD_SHAPE,
                  "group %d: m=%d differs from group 0's %d (m is the slab's row count, the same "
                  "for every group of a segment launch)", i, groups[i].m, groups[0].m);
  if (workspace == nullptr) return fail(NVFP4_ERR_WORKSPACE, "workspace is NULL");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(NVFP4_ERR_WORKSPACE, "workspace not 256-byte aligned");
  if (workspace_bytes < ws_total_bytes(num_groups))
    return fail(NVFP4_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes,
                ws_total_bytes(num_groups));
  std::vector<GroupDev> rec(static_cast<size_t>(num_groups));
  const SegmentArgs seg{seg_offsets, seg_counts, expected_rows, output};
  return grouped_gemm_impl(groups, num_groups, flags, static_cast<uint8_t*>(workspace),
                           workspace_bytes, static_cast<cudaStream_t>(stream), rec.data(),
                           /*use_cache=*/true, &seg);
}

}  // extern "C"

// ============================================================================
// Allocation-free entry point
// ============================================================================
// Some callers cannot allocate device memory at the point where they run the
// GEMM: frameworks whose memory is owned by their own pool allocator and that
// forbid other device allocations, plugins loaded into a host that only hands
// them the input and output buffers, and latency-critical paths that cannot
// afford the device synchronisation cudaMalloc may imply. For them this entry
// point takes its scratch space (group records, tensor maps and the device error
// word) from a fixed-size array compiled into the library instead of a
// caller-provided workspace. Limits and sharing rules are documented with the
// declaration in nvfp4_group_gemm.h.
namespace {

constexpr size_t kNoAllocScratchBytes = ws_total_bytes(NVFP4_NOALLOC_MAX_GROUPS);

// One copy per GPU that loads the library, kept until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocState {
  std::mutex mu;
  void* scratch = nullptr;  // device address of g_noalloc_scratch on this device, once found
};
NoAllocState g_noalloc[kMaxDevices];

// The device address of the scratch array on the current device. The host-side symbol is
// only a stand-in, so kernels must be given the address looked up here, with the device
// current. Only a successful lookup is kept: a failed one (for example a first call made
// inside a stream capture) is retried by the next call.
int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NVFP4_ERR_INVALID_ARGUMENT, "device %d", dev);
  NoAllocState& na = g_noalloc[dev];
  std::lock_guard<std::mutex> lock(na.mu);
  if (na.scratch == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                       "cudaGetSymbolAddress(scratch)");
    na.scratch = p;
  }
  *out = static_cast<uint8_t*>(na.scratch);
  return NVFP4_OK;
}

}  // namespace

extern "C" NVFP4_API int nvfp4_grouped_gemm_noalloc(const nvfp4_group* groups, int num_groups,
                                                    unsigned int flags, void* stream) {
  g_last_error.clear();
  int st = check_common_args(groups, num_groups, flags);
  if (st != NVFP4_OK) return st;
  if (num_groups > NVFP4_NOALLOC_MAX_GROUPS)
    return fail(NVFP4_ERR_INVALID_ARGUMENT,
                "num_groups=%d exceeds the %d groups the built-in scratch array holds; "
                "use nvfp4_grouped_gemm with a caller-provided workspace",
                num_groups, NVFP4_NOALLOC_MAX_GROUPS);
  if (num_groups == 0) return NVFP4_OK;
  uint8_t* ws = nullptr;
  st = noalloc_scratch(&ws);
  if (st != NVFP4_OK) return st;
  // Fixed-size host staging and uncached encoding: no heap use on this path. The header
  // (device error word, tile counters) keeps what the previous call left; the shared
  // implementation zeroes it on this call's stream once the table has passed its checks,
  // so a rejected call queues no write to the shared array.
  static thread_local GroupDev rec[NVFP4_NOALLOC_MAX_GROUPS];
  return grouped_gemm_impl(groups, num_groups, flags, ws, kNoAllocScratchBytes,
                           static_cast<cudaStream_t>(stream), rec, /*use_cache=*/false,
                           /*seg=*/nullptr, /*prepared=*/nullptr, /*clear_header=*/true);
}

extern "C" NVFP4_API int nvfp4_noalloc_check(void* stream, unsigned int* device_error_bits) {
  g_last_error.clear();
  if (device_error_bits) *device_error_bits = 0;
  uint8_t* ws = nullptr;
  int st = noalloc_scratch(&ws);
  if (st != NVFP4_OK) return st;
  return nvfp4_workspace_check(ws, stream, device_error_bits);
}
