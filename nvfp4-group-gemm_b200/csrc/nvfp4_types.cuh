// Types shared by the host launcher and the device kernels: the per-launch
// workspace layout (group records + tensor maps + error word) and the kernel
// parameter blocks.
#pragma once

#include <cstddef>
#include <cstdint>

namespace nvfp4 {

// Problem constants of the NVFP4 block-scaled format (16 e2m1 values share one
// E4M3 scale; scale factors are stored in 128-row x 4-column blocks of 512 B).
constexpr int kBlockM = 128;          // rows per tile (one tcgen05.mma M)
constexpr int kBlockK = 256;          // K elements per pipeline stage (128 bytes per row)
constexpr int kRowBytesPerStage = 128;
constexpr int kMmaK = 64;             // K per tcgen05.mma kind::mxf4nvf4
constexpr int kSfVec = 16;            // elements per scale factor
constexpr int kSfBlockBytes = 512;    // one 128 x 4 scale-factor block
// Groups whose records and tensor maps one upload launch carries in its parameters.
constexpr int kGroupsPerUpload = 24;

// 128-byte opaque CUtensorMap image (the driver type requires 64-byte alignment).
struct alignas(64) TmaDesc {
  uint64_t raw[16];
};
static_assert(sizeof(TmaDesc) == 128, "tensor map image must be 128 bytes");

// Tensor maps kept per group, in this order. The scale-factor maps view the blocked
// scale bytes as rows of 128 bytes (one box = 16 rows = one 2-KiB k-tile chunk of a
// 128-row block); the CTA-pair kernel loads scales through them.
// kMapA64 views A like kMapA with a 64-row box (the weight-stationary kernel's token tiles).
enum : int {
  kMapA = 0, kMapB = 1, kMapB2 = 2, kMapC = 3, kMapSfa = 4, kMapSfb = 5, kMapSfb2 = 6,
  kMapA64 = 7, kMapsPerGroup = 8
};

// One group as the device sees it (written by the descriptor builder).
struct GroupDev {
  const uint8_t* sfa;   // 128x4-blocked E4M3 scales of A
  const uint8_t* sfb;   // blocked scales of B (gate weights when gated)
  const uint8_t* sfb2;  // blocked scales of the up weights (gated only)
  uint8_t* c;           // fp16 output (the weight-stationary kernel stores without a map)
  int32_t m, n, k;
  int32_t tiles_m;
  int32_t tile_start, tile_end;  // [start, end) in the launch-wide tile order
  float alpha, alpha2;
};
static_assert(sizeof(GroupDev) == 64, "group record must fill its 64-byte workspace slot");

struct WorkspaceHeader {
  uint32_t error_bits;        // OR of device-side failure reasons (see kDevErr*)
  uint32_t tile_counter[2];   // dynamic tile schedule: next tile, finished CTAs (0 between launches)
  int32_t seg_total_tiles;    // segment launches: tiles of the launch, written on the device
  uint32_t reserved[60];
};
static_assert(sizeof(WorkspaceHeader) == 256, "header is 256 bytes");

// Device-side failure reasons (bit positions in WorkspaceHeader::error_bits).
enum : uint32_t {
  kDevErrProducerTimeout = 1u << 0,  // TMA producer gave up waiting for a free stage
  kDevErrMmaTimeout = 1u << 1,       // MMA issuer gave up waiting for a loaded stage
  kDevErrAccTimeout = 1u << 2,       // MMA issuer gave up waiting for a drained accumulator
  kDevErrEpilogueTimeout = 1u << 3,  // epilogue gave up waiting for a finished accumulator
  kDevErrDrainTimeout = 1u << 4,     // in-flight copies or MMAs did not finish at exit
  kDevErrBadSegment = 1u << 5,       // a device-side row segment was out of range (skipped)
};
constexpr uint32_t kDevErrTimeouts = kDevErrProducerTimeout | kDevErrMmaTimeout |
                                     kDevErrAccTimeout | kDevErrEpilogueTimeout |
                                     kDevErrDrainTimeout;

// Workspace layout: header | GroupDev[G] (64 B each) | TmaDesc[G][8] (128 B aligned) |
// int32 segment row offsets[G] (segment launches; 128 B aligned).
__host__ __device__ constexpr size_t ws_groups_offset() { return sizeof(WorkspaceHeader); }
__host__ __device__ constexpr size_t ws_maps_offset(int num_groups) {
  return (ws_groups_offset() + static_cast<size_t>(num_groups) * 64 + 127) &
         ~static_cast<size_t>(127);
}
__host__ __device__ constexpr size_t ws_seg_rows_offset(int num_groups) {
  return ws_maps_offset(num_groups) +
         static_cast<size_t>(num_groups) * kMapsPerGroup * sizeof(TmaDesc);
}
__host__ __device__ constexpr size_t ws_total_bytes(int num_groups) {
  return ws_seg_rows_offset(num_groups) +
         ((static_cast<size_t>(num_groups) * 4 + 127) & ~static_cast<size_t>(127));
}

// Split-K scratch, after the workspace proper (256-byte aligned): split_counters (4 KiB),
// then kSplitMaxSlots partial slots of 128 rows x 256 fp32 (128 KiB each).
constexpr int kSplitMaxSlots = 148;
constexpr size_t kSplitSlotBytes = 128 * 256 * 4;
constexpr size_t kSplitCounterBytes = 4096;
constexpr size_t kSplitScratchBytes = kSplitCounterBytes + kSplitMaxSlots * kSplitSlotBytes;
__host__ __device__ constexpr size_t ws_split_offset(int num_groups) {
  return (ws_total_bytes(num_groups) + 255) & ~static_cast<size_t>(255);
}

// Parameter block of the descriptor upload kernel: host-encoded records and
// tensor maps of up to kGroupsPerUpload groups (about 26 KB of kernel parameters).
struct UploadParams {
  TmaDesc maps[kGroupsPerUpload][kMapsPerGroup];
  GroupDev rec[kGroupsPerUpload];
  GroupDev* groups_out;
  TmaDesc* maps_out;
  int32_t first_group;
  int32_t count;
  // Split-K counters to zero (or nullptr): their place depends on the group count, so a
  // new group table may put them over bytes an earlier launch used for something else.
  int32_t* zero_counters;
};
static_assert(sizeof(UploadParams) <= 32000, "kernel parameter block too large");

// Peer copies an epilogue can replicate its fp16 output into (one box of 8 GPUs).
constexpr int kMaxReplicas = 7;

struct GemmParams {
  const GroupDev* groups;
  const TmaDesc* maps;
  uint32_t* error_bits;
  int32_t num_groups;
  int32_t total_tiles;
  int32_t diag_skip_mma;  // NVFP4_FLAG_DIAG_SKIP_MMA: the MMA issuer does no work
  int32_t dynamic_schedule;  // single-CTA kernel: claim tiles from tile_counter after the first
  uint32_t* tile_counter;    // WorkspaceHeader::tile_counter
  // Split-K of the last tiles (single-CTA kernels): units [0, split_first_tile) are whole
  // tiles; tiles split_first_tile.. are split into split_parts K ranges each. total_units =
  // split_first_tile + (total_tiles - split_first_tile) * split_parts (= total_tiles when
  // split_parts is 1). Partial tiles go to split_partials (one 128 x MMA_N fp32 slot per
  // split unit), split_counters[tile - split_first_tile] counts the parts that arrived.
  int32_t split_first_tile;
  int32_t split_parts;
  int32_t total_units;
  float* split_partials;
  int32_t* split_counters;
  // Segment launches (group rows given on the device): group g's A rows, scale blocks and C
  // rows start at row seg_rows[g] (a multiple of 128) of its operands, and the launch's
  // tile count is *seg_total_tiles (total_tiles and total_units above are then only upper
  // bounds). Both nullptr otherwise.
  const int32_t* seg_rows;
  const int32_t* seg_total_tiles;
  // NVFP4 output of gated launches (out_sf != nullptr): each group's c holds packed e2m1
  // codes [rows, n/2] and out_sf the blocked E4M3 scales of the output slab; out_scale is
  // the output's per-tensor scale and out_d6 = 6 * out_scale (fp32).
  uint8_t* out_sf;
  float out_scale;
  float out_d6;
  // Scattered fp16 output of non-gated segment launches (row_dest != nullptr): slab row r
  // goes to dest_base[row_dest[r] >> 40] + (row_dest[r] & (2^40 - 1)) * dest_ld bytes
  // (row_dest[r] < 0: not stored); c is not written.
  const int64_t* row_dest;
  uint8_t* dest_base[8];
  int64_t dest_ld;
  // Stream-K schedule of the weight-streaming kernel (stream_k_iters > 0; every group has
  // stream_k_ktiles k-tiles). Tiles [0, stream_k_first_tile) are whole units taken round
  // robin (CTA c: c, c + grid, ...), so that the tiles running at any moment are
  // neighbours (the m-tiles that share a weight tile run together and share it in L2).
  // The remaining tiles form a tile-major iteration space of stream_k_total_iters
  // k-iterations (tile stream_k_first_tile + j owns [j * ktiles, (j + 1) * ktiles)); CTA c
  // then runs iterations [c * stream_k_iters, (c + 1) * stream_k_iters) of it, so every CTA
  // ends with the same amount of work. A tile cut by the range boundary of CTA b (b >= 1)
  // is computed in two pieces, its first k-tiles by CTA b - 1 and the rest by CTA b; per
  // epilogue warp, the piece that finishes first stores its fp32 rows to split_partials
  // slot b and the other adds them to its own and stores C (split_counters[4 b + warp
  // quarter] orders the two; 0 between launches).
  int32_t stream_k_iters;
  int32_t stream_k_ktiles;
  int64_t stream_k_total_iters;
  int32_t stream_k_first_tile;
  // Replicated fp16 output (num_replicas > 0): every C row a kernel stores also goes to
  // c_row + replica_offset[i] (byte offsets into other GPUs' copies of the output buffers,
  // mapped into this process), straight from the epilogue, tile by tile.
  int32_t num_replicas;
  int64_t replica_offset[kMaxReplicas];
};

// Destination of slab row r of a scattered output (nullptr: not stored).
__device__ __forceinline__ uint8_t* scatter_row(const GemmParams& p, int64_t r) {
  const int64_t code = p.row_dest[r];
  if (code < 0) return nullptr;
  uint8_t* base = p.dest_base[(code >> 40) & 7];
  if (base == nullptr) return nullptr;
  return base + (code & ((int64_t{1} << 40) - 1)) * p.dest_ld;
}

// First row of group g's segment (0 outside segment launches).
__device__ __forceinline__ int seg_row(const GemmParams& p, int g) {
  return p.seg_rows != nullptr ? p.seg_rows[g] : 0;
}

}  // namespace nvfp4
