/*
 * nvfp4_group_gemm.h - C ABI of the B200 (sm_100a) NVFP4 block-scaled grouped GEMM.
 *
 * Plain pointers and sizes only; no CUDA or framework types appear in the
 * signatures (streams are passed as `void*` holding a cudaStream_t, NULL = the
 * legacy default stream). Every entry point returns an nvfp4_status code and
 * never aborts the process. Launches are asynchronous on the given stream.
 *
 * Reference interfaces replaced (goldbar123467/NVFP4-Group-Gemm):
 *   custom_kernel(data), 4-tuple grouped branch ... submission.py:788-858
 *   run_single_gemm(...) + _fused_silu_gate(...) .. submission.py:742-785, 860-886, 707-710
 *   compile_kernel(problem_sizes) ................. submission.py:715-739 (no JIT here:
 *                                                   kernels are compiled ahead of time)
 *   to_blocked(input_matrix) ...................... REFERENCE_IMPL.md:19-42
 *   create_reordered_scale_factor_tensor(...) ..... REFERENCE_IMPL.md:89-137 (same bytes)
 */
#ifndef NVFP4_GROUP_GEMM_H_
#define NVFP4_GROUP_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NVFP4_API __attribute__((visibility("default")))
#else
#define NVFP4_API
#endif

/* 2: segment launches (nvfp4_grouped_gemm_segments, nvfp4_segment_output), the
 * expert-parallel exchange (nvfp4_ep_*), NVFP4_FLAG_SPLIT_K, a segment-row table in the
 * workspace (nvfp4_workspace_size grew by 4 bytes per group, rounded up to 128). */
#define NVFP4_ABI_VERSION 2

typedef enum nvfp4_status {
  NVFP4_OK = 0,
  NVFP4_ERR_INVALID_ARGUMENT = 1,  /* null table, negative count, bad flags */
  NVFP4_ERR_BAD_SHAPE = 2,         /* K % 256 != 0, K <= 0, N % 8 != 0, negative sizes */
  NVFP4_ERR_MISALIGNED = 3,        /* a tensor base address is not 16-byte aligned */
  NVFP4_ERR_NULL_POINTER = 4,      /* a tensor of a non-empty group is NULL */
  NVFP4_ERR_WORKSPACE = 5,         /* workspace NULL, too small, or not 256-byte aligned */
  NVFP4_ERR_CUDA = 6,              /* a CUDA runtime call or kernel launch failed */
  NVFP4_ERR_DEVICE_TIMEOUT = 7,    /* a kernel gave up waiting (see nvfp4_workspace_check) */
  NVFP4_ERR_UNSUPPORTED_DEVICE = 8,/* current device is not compute capability 10.0 */
  NVFP4_ERR_DRIVER = 9             /* tensor-map encoder entry point unavailable */
} nvfp4_status;

/* Flags for nvfp4_grouped_gemm. */
#define NVFP4_FLAG_GATED 0x1u     /* C = fp16(silu(fp16(a*A.B^T)) * fp16(a2*A.B2^T)) */
#define NVFP4_FLAG_TILE_N128 0x2u /* force 128-column tiles (non-gated only) */
#define NVFP4_FLAG_TILE_N256 0x4u /* force 256-column tiles (non-gated only) */
#define NVFP4_FLAG_REUSE_DESCRIPTORS 0x8u /* workspace already holds this exact group table
                                             (same pointers, sizes, scales, flags) from the
                                             previous call on the same stream: skip rebuilding */
#define NVFP4_FLAG_CTA_PAIR 0x10u   /* force 256-row tiles on CTA pairs (tcgen05 cta_group::2) */
#define NVFP4_FLAG_DIAG_SKIP_MMA 0x40u /* diagnostic, for testing failure detection only: the
                                          MMA issuer issues nothing, so the kernel's bounded
                                          waits run out (about 2 s), it records the reason in
                                          the workspace error word and exits cleanly; the
                                          output is not written */
#define NVFP4_FLAG_SINGLE_CTA 0x20u /* force 128-row tiles on single CTAs.
                                       Default: CTA pairs when the non-empty groups average
                                       at least 192 rows, or at least 96 rows with
                                       K >= 4096; single CTAs otherwise */
#define NVFP4_FLAG_SPLIT_K 0x100u /* allow split-K of a single-CTA launch's last partial wave
                                     (needs the split scratch, see NVFP4_SPLIT_SCRATCH_BYTES) */
#define NVFP4_FLAG_STREAM_K 0x200u /* weight-streaming launches (non-empty groups averaging
                                      at most 64 rows, one K) with at least one full wave of
                                      tiles: share the last full wave and the partial one out
                                      as equal k-iteration ranges, one per CTA (needs the
                                      split scratch). Off by default: measured slower than
                                      dynamic tile claims (64 experts, N 1536, K 4096: 64.2 vs
                                      53.0 us per call), whose balance follows the real cost
                                      of each tile */
#define NVFP4_FLAG_WEIGHT_STATIONARY 0x80u /* force the weight-stationary kernel (non-gated
                                              only): tiles of 128 weight rows x 64 token
                                              rows, computed as C^T so that small groups
                                              carry no padding rows */

/*
 * One GEMM of the group. All matrices are row-major with K innermost ("K-major"),
 * exactly the storage of the reference's tensors (L = 1):
 *   a    : packed e2m1, [m, k/2] bytes     (float4_e2m1fn_x2 [M, K//2, 1]; low nibble = even k)
 *   b    : packed e2m1, [n, k/2] bytes     (gate weights when NVFP4_FLAG_GATED)
 *   b2   : packed e2m1, [n, k/2] bytes     (up weights; gated only, else NULL)
 *   sfa  : E4M3 scales of a in the 128x4-blocked layout, ceil(m/128)*128 * k/16 bytes
 *          (the storage of the reference's sfa_reordered tensor, = to_blocked(sfa))
 *   sfb  : blocked E4M3 scales of b, ceil(n/128)*128 * k/16 bytes
 *   sfb2 : blocked E4M3 scales of b2 (gated only)
 *   c    : fp16 [m, n] output, written in place
 *   alpha, alpha2 : per-tensor fp32 global scales of the (gate, up) products; 1.0 = none
 * Constraints: k > 0 and k % 256 == 0; n % 8 == 0; every pointer 16-byte aligned.
 * Groups with m == 0 or n == 0 are skipped (their pointers are not read).
 */
typedef struct nvfp4_group {
  const void* a;
  const void* b;
  const void* b2;
  const void* sfa;
  const void* sfb;
  const void* sfb2;
  void* c;
  int32_t m;
  int32_t n;
  int32_t k;
  float alpha;
  float alpha2;
} nvfp4_group;

/*
 * Device workspace bytes needed for `num_groups` groups (group records, tensor
 * maps, segment row offsets and a device error word): 256 + 64 * num_groups rounded up
 * to 128, plus 1024 * num_groups, plus 4 * num_groups rounded up to 128. The workspace is owned by the caller, must be
 * 256-byte aligned, must not be shared by calls that may run concurrently, and
 * may be reused by consecutive calls on one stream.
 */
NVFP4_API size_t nvfp4_workspace_size(int num_groups);

/*
 * Grouped GEMM over `num_groups` groups in one persistent launch (replaces
 * custom_kernel's 4-tuple path, submission.py:804-858, and, with
 * NVFP4_FLAG_GATED, the dual GEMM + SiLU path, submission.py:860-886).
 * `groups` is a HOST array read before the call returns.
 */
NVFP4_API int nvfp4_grouped_gemm(const nvfp4_group* groups, int num_groups, unsigned int flags,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Grouped GEMM whose groups' row counts are read on the GPU when the launch runs: group g
 * multiplies rows [seg_offsets[g], seg_offsets[g] + seg_counts[g]) of a slab of
 * groups[g].m rows (a, sfa and c of every group address such a slab; m must be the same
 * for all groups) with its own weights. seg_offsets/seg_counts are device int32 arrays of
 * num_groups entries, e.g. the offsets/counts nvfp4_moe_route writes, so a routed MoE
 * step needs no device-to-host read between routing and the expert GEMMs and can be
 * captured in a CUDA graph whole (no new graph per batch composition).
 *
 * Each offset must be a multiple of 128 and offset + count <= m; a group that breaks this
 * is skipped and nvfp4_workspace_check reports NVFP4_ERR_BAD_SHAPE. Rows of C from
 * offset + count up to the next multiple of 128 (inside the slab) may be overwritten:
 * they are the segment's padding. `expected_rows` is a host estimate of the rows over all
 * groups (tokens x top-k), used like the real rows of nvfp4_grouped_gemm to pick CTA
 * pairs or single CTAs; <= 0 means m. The workspace is that of nvfp4_grouped_gemm and
 * NVFP4_FLAG_REUSE_DESCRIPTORS has the same meaning (the slab addresses, not the
 * segments, are the descriptors). NVFP4_FLAG_WEIGHT_STATIONARY and NVFP4_FLAG_SPLIT_K are
 * rejected. No counterpart in the reference, whose groups are formed on the host.
 *
 * `output` (may be NULL: fp16 rows into c) selects another output form, see below.
 */
#define NVFP4_EP_MAX_RANKS 8
typedef struct nvfp4_segment_output {
  /* NVFP4 output (gated launches, sf != NULL): instead of fp16, c receives packed e2m1
   * codes [m, n/2] and sf the 128x4-blocked E4M3 scales of the [m, n] output slab, as
   * nvfp4_quantize(fp16 output, global_scale = scale) would write them (bit-identical); n a
   * multiple of 64. Saves the fp16 write and the quantiser's read of it. */
  void* sf;
  float scale;
  /* Scattered rows (non-gated launches, row_dest != NULL): the fp16 row of slab row r goes
   * to dest_base[row_dest[r] >> 40] + (row_dest[r] & 0xFFFFFFFFFF) * dest_ld bytes instead
   * of c (row_dest[r] < 0: not stored). The bases may be peer GPUs' memory (P2P stores):
   * the expert-parallel block returns each expert output row to its token's rank this way,
   * from the GEMM's epilogue, overlapping the transfer with the GEMM. dest_ld and the
   * bases 16-byte aligned. */
  const int64_t* row_dest;
  void* dest_base[NVFP4_EP_MAX_RANKS];
  int64_t dest_ld;
} nvfp4_segment_output;

NVFP4_API int nvfp4_grouped_gemm_segments(const nvfp4_group* groups, int num_groups,
                                          unsigned int flags, const int32_t* seg_offsets,
                                          const int32_t* seg_counts, int64_t expected_rows,
                                          const nvfp4_segment_output* output, void* workspace,
                                          size_t workspace_bytes, void* stream);

/*
 * Prepared launches: nvfp4_plan_create validates a group table, uploads its descriptors into
 * `workspace` on `stream` and keeps the launch (kernel, grid, parameters); each
 * nvfp4_plan_launch then only launches the kernel (host work of a plain launch with
 * NVFP4_FLAG_REUSE_DESCRIPTORS, minus the per-group pass over the table). The tensors,
 * the workspace and the device must stay as they were when the plan was made; launches of
 * one plan share its workspace and must be ordered on the GPU. Neither REUSE_DESCRIPTORS nor
 * SPLIT_K may be passed to nvfp4_plan_create. nvfp4_plan_launch is CUDA-graph capturable.
 */
typedef struct nvfp4_plan nvfp4_plan;
NVFP4_API int nvfp4_plan_create(const nvfp4_group* groups, int num_groups, unsigned int flags,
                                void* workspace, size_t workspace_bytes, void* stream,
                                nvfp4_plan** plan);
NVFP4_API int nvfp4_plan_launch(const nvfp4_plan* plan, void* stream);
NVFP4_API void nvfp4_plan_destroy(nvfp4_plan* plan);

/*
 * Extra workspace for split-K: with NVFP4_FLAG_SPLIT_K and workspace_bytes at least
 * nvfp4_workspace_size(num_groups) rounded up to 256, plus this, single-CTA launches split
 * the K loop of the tiles that would otherwise run in a last, partly idle wave (all tiles,
 * when the launch has fewer tiles than the GPU has SMs) into several units; each writes an
 * fp32 partial tile to this space and the last part of a tile to finish sums the parts in a
 * fixed order and writes C (results are bit-identical from run to run). Zero-filled before
 * its first use, like the rest of the workspace. 4 KiB of counters + 148 x 128 KiB. Opt-in:
 * the final sum of a tile runs on one SM, which on the shapes measured cost more than the
 * balanced tail saved (cfg4-like 64 experts: 138 vs 52 us per call).
 */
#define NVFP4_SPLIT_SCRATCH_BYTES (4096u + 148u * 131072u)

/*
 * Convert plain row-major E4M3 scales [rows, sf_cols] (row stride `ld` bytes)
 * into the 128x4-blocked layout the kernel consumes; the output holds
 * nvfp4_sf_blocked_size(rows, sf_cols) bytes, padding rows/columns written as 0.
 * Bit-exact with to_blocked (REFERENCE_IMPL.md:19-42).
 */
NVFP4_API size_t nvfp4_sf_blocked_size(int rows, int sf_cols);
NVFP4_API int nvfp4_sf_to_blocked(const void* plain, void* blocked, int rows, int sf_cols,
                                  int64_t ld, void* stream);

/*
 * NVFP4 activation quantiser: x [rows, cols] (bf16 or fp16, row stride `ld` elements)
 * -> packed e2m1 [rows, cols/2] (row stride `packed_ld` bytes; element 2i in the low
 * nibble) and E4M3 scales per 16 elements, written in the 128x4-blocked layout that
 * nvfp4_group.sfa expects (nvfp4_sf_blocked_size(rows, cols/16) bytes; padding rows 0).
 * Per 16-element block: sf = E4M3(amax / (6 * global_scale)) and
 * q = E2M1(x * (1 / (value(sf) * global_scale))), every step rounded to nearest even and
 * saturated, so x ~= value(q) * value(sf) * global_scale; pass global_scale =
 * amax(|x|) / (6 * 448) and fold it into the GEMM's alpha. The reference has no
 * counterpart: its inputs arrive already quantised (REFERENCE_IMPL.md:143-205 generates
 * e2m1 codes and scales directly); this produces the GEMM's A operand from activations.
 * Requirements: cols a positive multiple of 64; x, packed and sf_blocked 16-byte aligned;
 * ld a multiple of 8 elements, packed_ld a multiple of 16 bytes; global_scale finite > 0;
 * inputs finite. Asynchronous on `stream`.
 */
#define NVFP4_DTYPE_BF16 0
#define NVFP4_DTYPE_FP16 1
NVFP4_API int nvfp4_quantize(const void* x, int rows, int cols, int64_t ld, int dtype,
                             float global_scale, void* packed, int64_t packed_ld, void* sf_blocked,
                             void* stream);

/*
 * nvfp4_quantize with a row map (`src_rows`, device int32 [rows]):
 *   NVFP4_ROWS_GATHER: output row r quantises input row src_rows[r] (MoE dispatch: the row
 *                      map from nvfp4_moe_route); src_rows[r] < 0 gives a zero row.
 *   NVFP4_ROWS_MASK:   output row r quantises input row r where src_rows[r] >= 0, zeros
 *                      elsewhere (a dispatched buffer whose padding rows hold no data).
 * No counterpart in the reference (see nvfp4_quantize).
 */
#define NVFP4_ROWS_GATHER 1
#define NVFP4_ROWS_MASK 2
NVFP4_API int nvfp4_quantize_rows(const void* x, int rows, int cols, int64_t ld, int dtype,
                                  float global_scale, const int32_t* src_rows, int mode,
                                  void* packed, int64_t packed_ld, void* sf_blocked, void* stream);

/*
 * MoE token dispatch metadata (no counterpart in the reference, which receives its groups
 * already formed; this is the routing step before the grouped GEMM). topk_ids: device int32
 * [tokens, topk], expert of each (token, slot) pair (< 0 or >= num_experts: dropped).
 * Outputs (device int32): counts [num_experts] rows per expert; offsets [num_experts + 1]
 * first row of each expert in the dispatched buffers, every expert starting on a 128-row
 * boundary (offsets[num_experts] = padded total), so one blocked scale buffer for all rows is
 * the concatenation of the experts' blocked layouts; dest [tokens * topk] the dispatched row
 * of each pair (-1 if dropped), rows of an expert in token order; src_rows [rows_capacity] the
 * token of each dispatched row (-1 for padding rows and for every row past
 * offsets[num_experts]). rows_capacity >= tokens * topk + 127 * num_experts;
 * num_experts <= 1024.
 * Deterministic. workspace: nvfp4_moe_route_workspace_size(tokens * topk, num_experts) bytes
 * of device memory (no initialisation needed).
 */
NVFP4_API size_t nvfp4_moe_route_workspace_size(int64_t pairs, int num_experts);
NVFP4_API int nvfp4_moe_route(const int32_t* topk_ids, int tokens, int topk, int num_experts,
                              int32_t* counts, int32_t* offsets, int32_t* dest, int32_t* src_rows,
                              int64_t rows_capacity, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * MoE dispatch of quantised rows (no counterpart in the reference): dispatched row r
 * receives packed row src_rows[r] of packed_src ([*, cols/2] bytes, row stride ld_src) and its
 * scales from sf_src (blocked layout of the source rows) into packed_dst (row stride ld_dst)
 * and sf_dst (blocked layout of `rows` rows); rows with src_rows[r] < 0 become zeros.
 * Quantising tokens once with nvfp4_quantize and gathering equals nvfp4_quantize_rows in
 * gather mode bit for bit, with a quarter of the bytes read per dispatched row.
 * cols a multiple of 64; buffers 16-byte aligned; strides multiples of 16 bytes.
 */
NVFP4_API int nvfp4_moe_gather_quantized(const void* packed_src, int64_t ld_src,
                                         const void* sf_src, const int32_t* src_rows, int rows,
                                         int cols, void* packed_dst, int64_t ld_dst, void* sf_dst,
                                         void* stream);

/*
 * MoE combine (no counterpart in the reference): out[t, :] = bf16( sum_j weights[t, j] *
 * y[dest[t * topk + j], :] ), y fp16 [dispatched rows, cols] (row stride ldy elements),
 * weights fp32 [tokens, topk], out bf16 [tokens, cols] (row stride ldo); fp32 products and
 * sums in slot order; pairs with dest < 0 are skipped. cols, ldy, ldo multiples of 8;
 * y and out 16-byte aligned.
 */
NVFP4_API int nvfp4_moe_combine(const void* y, int64_t ldy, const int32_t* dest,
                                const float* weights, int tokens, int topk, int cols, void* out,
                                int64_t ldo, void* stream);

/*
 * Expert-parallel MoE exchange over NVLink peer memory: one process per GPU, `world` ranks
 * (<= NVFP4_EP_MAX_RANKS), rank p owning experts [p * E / world, (p + 1) * E / world).
 * A nvfp4_ep_peers table holds, for every rank i < world, this process's device address of
 * rank i's copy of one symmetric buffer (the same allocation size on every rank, mapped
 * peer-to-peer, e.g. torch symmetric memory or CUDA IPC). The kernels only load and store;
 * the caller orders the steps across ranks with a barrier on the same stream (a one-element
 * NCCL all-reduce) where marked (|). Per MoE layer:
 *
 *   nvfp4_moe_route over all E experts (local pairs), nvfp4_quantize of the local tokens
 *   nvfp4_ep_publish_counts: route counts -> row `rank` of every rank's [world, E] matrix  |
 *   nvfp4_ep_layout: from this rank's copy of the matrix, this rank's expert segments in its
 *     receive slab (rows of rank 0 first, then rank 1, ...; each expert 128-row aligned) and,
 *     per expert, the first row of this rank's pairs in the owner's slab (send_base)
 *   nvfp4_ep_dispatch: each routed token row (codes, and its scales as a plain row of cols/16
 *     bytes) into the owner's receive slabs, with the row's return address (rank << 40 |
 *     pair index) in the owner's recv_meta; remote_rows[pair] = its row there (-1: dropped)  |
 *   owner: nvfp4_sf_to_blocked on the received scales, the gate/up GEMM over its segments
 *     (nvfp4_grouped_gemm_segments, NVFP4 output), the down GEMM with scattered output
 *     (row_dest = recv_meta, dest_base = every rank's return buffer): each output row is
 *     stored by the GEMM's epilogue into its token's rank, [tokens * topk, cols] fp16 there  |
 *   nvfp4_ep_combine: out[t] = bf16(sum_j w[t, j] * ret[t * topk + j]) over kept pairs
 *     (fp32, slot order: bit-identical to nvfp4_moe_combine over the same rows)
 *
 * Owner-side sums (a token's slots that meet on one owner travel as one row each way):
 *
 *   nvfp4_ep_dispatch_tokens instead of nvfp4_ep_dispatch: remote_rows as nvfp4_ep_dispatch
 *     gives them, and each token's codes and plain scale row once into every owner holding
 *     a kept pair of it ([world * tokens] token-slab rows there, row rank * tokens + t);
 *   nvfp4_ep_publish_pairs: into every owner's pair tables ([world, tokens * topk] int32 rows
 *     and fp32 weights, row q = source rank q; every rank has the same tokens * topk) each
 *     pair's slab row there (-1 where it did not go) and, on its owner, its routing weight |
 *   owner: nvfp4_ep_expand copies each received pair's token row from the token slabs into
 *     its receive-slab row (what nvfp4_ep_dispatch would have stored there);
 *   owner: the down GEMM writes its output rows locally ([capacity, cols] fp16, slab order);
 *     nvfp4_ep_return_sums: for every source rank q and token t with pairs here,
 *     fp16(sum_j w[t, j] * y[row_j]) (fp32, slot order) -> row t * world + rank of rank q's
 *     [tokens, world, cols] fp16 return buffer                                             |
 *   nvfp4_ep_combine_sums: out[t] = bf16(sum_p ret[t, p]) over the owners p (ascending) that
 *     hold a kept pair of t (fp32)
 *
 * A segment that does not fit the owner's receive slab is dropped on every rank (its pairs
 * get remote_rows -1) and bit 0x1 is set in the layout's error word. No counterpart in the
 * reference (single GPU).
 */
typedef struct nvfp4_ep_peers {
  void* ptr[NVFP4_EP_MAX_RANKS];
} nvfp4_ep_peers;

NVFP4_API int nvfp4_ep_publish_counts(const int32_t* counts, int num_experts, int rank, int world,
                                      nvfp4_ep_peers count_mats, void* stream);
NVFP4_API int nvfp4_ep_layout(const int32_t* count_mat, int num_experts, int rank, int world,
                              int64_t recv_capacity, int32_t* seg_offsets, int32_t* seg_counts,
                              int32_t* send_base, unsigned int* error_word, void* stream);
NVFP4_API int nvfp4_ep_dispatch(const int32_t* topk_ids, int tokens, int topk, int num_experts,
                                int rank, int world, const int32_t* dest, const int32_t* offsets,
                                const int32_t* send_base, const void* codes, int64_t ld_codes,
                                const void* sf_blocked, int cols, nvfp4_ep_peers recv_codes,
                                nvfp4_ep_peers recv_sf, nvfp4_ep_peers recv_meta,
                                int64_t recv_capacity, int32_t* remote_rows, void* stream);
NVFP4_API int nvfp4_ep_combine(const int32_t* remote_rows, const float* weights, int tokens,
                               int topk, const void* ret, int cols, void* out, int64_t ldo,
                               void* stream);
NVFP4_API int nvfp4_ep_dispatch_tokens(const int32_t* topk_ids, int tokens, int topk,
                                       int num_experts, int rank, int world, const int32_t* dest,
                                       const int32_t* offsets, const int32_t* send_base,
                                       const void* codes, int64_t ld_codes, const void* sf_blocked,
                                       int cols, nvfp4_ep_peers tok_codes, nvfp4_ep_peers tok_sf,
                                       int64_t recv_capacity, int32_t* remote_rows, void* stream);
NVFP4_API int nvfp4_ep_expand(const int32_t* pair_rows, int tokens, int topk, int world,
                              const void* tok_codes, const void* tok_sf, int cols,
                              void* recv_codes, void* recv_sf, int64_t recv_capacity,
                              void* stream);
NVFP4_API int nvfp4_ep_publish_pairs(const int32_t* topk_ids, const int32_t* remote_rows,
                                     const float* weights, int tokens, int topk, int num_experts,
                                     int rank, int world, nvfp4_ep_peers pair_rows,
                                     nvfp4_ep_peers pair_weights, void* stream);
NVFP4_API int nvfp4_ep_return_sums(const int32_t* pair_rows, const float* pair_weights,
                                   int tokens, int topk, int rank, int world, const void* y,
                                   int64_t ldy, int cols, nvfp4_ep_peers ret, void* stream);
NVFP4_API int nvfp4_ep_combine_sums(const int32_t* topk_ids, const int32_t* remote_rows,
                                    int tokens, int topk, int num_experts, int world,
                                    const void* ret, int cols, void* out, int64_t ldo,
                                    void* stream);

/*
 * Synchronise `stream`, then read and clear the device error word of `workspace`.
 * Returns NVFP4_ERR_DEVICE_TIMEOUT if a kernel using it gave up on a wait, else
 * NVFP4_ERR_BAD_SHAPE if a segment launch skipped an out-of-range segment (bit 0x20); the
 * reason bits are stored to *device_error_bits when non-NULL.
 */
NVFP4_API int nvfp4_workspace_check(void* workspace, void* stream, unsigned int* device_error_bits);

/* Human-readable text of a status code, and detail of the last error on this thread. */
NVFP4_API const char* nvfp4_strerror(int status);
NVFP4_API const char* nvfp4_last_error_detail(void);

/*
 * nvfp4_grouped_gemm whose fp16 output is also written, tile by tile from the kernel's
 * epilogue, into num_replicas (1..7) copies of the output buffers on other GPUs: every row
 * stored at c also goes to (uint8_t*)c + replica_offsets[i] for each i. The copies are other
 * GPUs' memory mapped into this process at the same layout as the local outputs (for
 * example one symmetric-memory allocation holding every rank's output slab, offsets = peer
 * base - local base), so an expert-parallel GEMM followed by an all-gather of its outputs is
 * one kernel whose NVLink stores overlap its math. The stores are plain 16-byte stores (no
 * multicast); they are complete when the kernel is, and the caller orders them with the
 * replicas' owners (e.g. a cross-rank barrier on the stream) before those read the rows or
 * the next call writes them again. Offsets must be non-zero multiples of 16;
 * NVFP4_FLAG_WEIGHT_STATIONARY is not accepted. No counterpart in the reference, which runs
 * on one GPU; this is the fused form of the output all-gather of its expert-parallel
 * deployment (north star (5)).
 */
NVFP4_API int nvfp4_grouped_gemm_replicated(const nvfp4_group* groups, int num_groups,
                                            unsigned int flags, void* workspace,
                                            size_t workspace_bytes,
                                            const int64_t* replica_offsets, int num_replicas,
                                            void* stream);

/*
 * Allocation-free variant of nvfp4_grouped_gemm. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory where they run the GEMM:
 * frameworks that own all device memory through their own pool allocator and
 * forbid other allocations, plugins loaded into a host application that only
 * hands them their input and output buffers, and latency-critical paths that
 * cannot afford cudaMalloc's implicit device synchronisation. Instead of a caller-provided
 * workspace it uses a scratch array compiled into the library
 * (nvfp4_workspace_size(NVFP4_NOALLOC_MAX_GROUPS) bytes, about 544 KiB, held on
 * every GPU that loads the library until the process exits). It calls no
 * cudaMalloc/cudaFree and no allocating library routine.
 *
 * - num_groups above NVFP4_NOALLOC_MAX_GROUPS is rejected with
 *   NVFP4_ERR_INVALID_ARGUMENT (use nvfp4_grouped_gemm with a workspace instead).
 * - The first call on a device looks up the device address of the scratch array
 *   (cudaGetSymbolAddress) with that device current; make that first call before
 *   any stream capture. Only a successful lookup is kept: if it fails, the call
 *   returns NVFP4_ERR_CUDA and the next call on that device tries again.
 * - Every call on a device shares the one scratch array, which keeps the last
 *   call's contents. A call that passes its checks first zeroes the array's header
 *   (device error word, tile counters) on its stream; a rejected call writes
 *   nothing to it. Calls that can overlap on the GPU - on different streams, or
 *   from different threads without ordering - race on it and must not be issued.
 * - NVFP4_FLAG_REUSE_DESCRIPTORS means the scratch array holds this exact group
 *   table from the previous call on the device.
 * - Device-side wait timeouts set bits in the scratch array's error word; read
 *   them with nvfp4_noalloc_check after the call (before the next call clears them).
 * Arguments, flags, outputs and other status codes are as in nvfp4_grouped_gemm.
 */
#define NVFP4_NOALLOC_MAX_GROUPS 512
NVFP4_API int nvfp4_grouped_gemm_noalloc(const nvfp4_group* groups, int num_groups,
                                         unsigned int flags, void* stream);

/*
 * nvfp4_workspace_check for the built-in scratch array of nvfp4_grouped_gemm_noalloc
 * on the current device: synchronise `stream`, then read and clear the array's
 * device error word. NVFP4_ERR_DEVICE_TIMEOUT if the last call's kernel gave up on a
 * wait; the reason bits go to *device_error_bits when non-NULL. Allocates nothing.
 * No counterpart in the reference.
 */
NVFP4_API int nvfp4_noalloc_check(void* stream, unsigned int* device_error_bits);

/* NVFP4_ABI_VERSION of the loaded library. */
NVFP4_API int nvfp4_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_GROUP_GEMM_H_ */
