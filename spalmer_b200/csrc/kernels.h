// Internal kernel interfaces of libspx (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "status.h"

namespace spx {

constexpr int kTileRows = 128;         // M of every tcgen05 tile (cta_group::1)
constexpr int kGemmThreads = 320;      // 10 warps: TMA, MMA, 8 x epilogue (2 per TMEM lane quadrant)
// gemm_kernel adds producer warps for gathered BF16 rows (warp 0 and warps
// 10.. each gather an equal share of a tile's rows); idle otherwise.
constexpr int kGemmGatherProducers = 2;
constexpr int kGemmExtraProducerWarp0 = 10;
constexpr int kGemmCopierWarp = 10 + kGemmGatherProducers - 1;  // copies gathered A stages out (copy_out)
constexpr int kGemmKernelThreads = 32 * (kGemmCopierWarp + 1);
constexpr int kGemmEpilogueWarps = 8;
constexpr int kMaxAccBufs = 4;         // TMEM accumulator buffers per CTA (as many as fit in 512 columns)
constexpr size_t kGemmSmemBudget = 227 * 1024;  // sm_100 opt-in maximum per CTA
constexpr int kSliceCols = 64;                  // epilogue staging slice width
constexpr int kStageBytesPerWarp = 32 * kSliceCols * 2;
constexpr int kRouteRows = 128;        // token rows per route_select CTA
constexpr int kTieWarps = 8;           // rows replayed at once per route_ties CTA (one warp each)
constexpr int kRouteWarps = 8;         // warps per small-T route CTA (one token row per warp)
constexpr int kRouteRowsMaxTokens = 4096;  // up to this many rows the warp-per-row route kernel runs
constexpr int kSmallBatchTokens = 256;     // decode-sized batches: narrow GEMM tiles (see make_shape)
constexpr int kMaxTopK = 20;           // MicroExpertsConfig.max_active_experts default
constexpr int kDispatchChunk = 2048;   // pairs per dispatch CTA
constexpr int kDispatchWarps = 4;
constexpr int kDispatchSmallPairs = 4096;  // up to this many pairs one CTA runs the whole dispatch
constexpr int kDispatchThreads = 32 * kDispatchWarps;

// kEpiScatter writes the weighted expert rows in sorted (dispatch) order; the
// combine (pack.cu, or kEpiCombine: the shared down projection's epilogue)
// gathers each token's k rows through the rank array.
enum Epi : int { kEpiStore = 0, kEpiSwiglu = 1, kEpiScatter = 2, kEpiCombine = 3 };
constexpr int kCombineMaxK = 8;  // kEpiCombine: top-k up to this (larger k: separate combine kernel)

// MXFP8 lane: B-operand sources of the pack-time quantiser, and the tensor
// memory plan of the block-scaled GEMM: accumulators in columns [0, 384)
// (three of 128 columns, or one of 256), then eight rotating 16-column
// scale-factor slots (SFA in the first 4 columns, SFB -- up to 256 rows,
// 2 atoms -- in the next 8).
enum MxSource : int { kMxSrcW1 = 0, kMxSrcW2 = 1, kMxSrcRows = 2 };
constexpr int kMxBlock = 32;        // elements per E8M0 scale
constexpr int kMxAtomBytes = 512;   // scale atom: 128 rows x 4 scales (one 128-element K block)
constexpr int kMxMaxBn = 256;
constexpr int kMxDenseBn = 128;              // N tile of the dense MXFP8 matmul
constexpr uint32_t kMxSfColumn = 384;
constexpr int kMxSfSlots = 8;
constexpr uint32_t kMxSfSlotCols = 16;
constexpr uint32_t kMxStageSfBytes = 3 * kMxAtomBytes;  // SFA atom + up to two SFB atoms per stage
// NVFP4 lane: a stage is 128 bytes of K = 256 E2M1 elements = four K-64 MMAs,
// each with its own SFA atom and up to two SFB atoms; their TMEM copies rotate
// through ten 12-column slots from column 384.
constexpr uint32_t kNvStageSfBytes = 12 * kMxAtomBytes;
constexpr uint32_t kNvSfSlots = 10;
constexpr uint32_t kNvSfSlotCols = 12;

struct RouteArgs {
  const uint16_t* logits;    // [T, E] bf16
  const uint16_t* lut;       // softplus table [65536] or null (identity transform)
  const uint8_t* resident;   // [E] or null (full pool)
  uint16_t* scores;          // [T, E] bf16 (router_scores)
  int64_t* ids;              // [T, k]
  uint16_t* weights;         // [T, k] bf16
  int* tie_count;            // zeroed before launch
  int* tie_rows;             // [T]
  float* lb_partial;         // [ceil(T/128), E]
  int64_t tokens;
  int num_experts;
  int top_k;
  int sm_count;
  int* status;
};

struct DispatchArgs {
  const int64_t* ids;        // [P] expert id per pair, pair p = token * k + slot
  int64_t pairs;
  int64_t tokens;
  int num_experts;
  int top_k;
  int* chunk_hist;           // [ceil(P/2048), E]
  int* counts;               // [E]
  int* starts;               // [E]
  int4* tiles;               // [ceil(P/128) + E] {expert, row0, rows, expert}: BF16-lane experts
  int* num_tiles;
  const uint8_t* lane_mx;    // [E] 1 = expert runs the MXFP8 lane, or null (all BF16)
  int4* tiles_mx;            // [ceil(P/128) + E] tiles of MXFP8-lane experts (when lane_mx)
  int* num_tiles_mx;
  int* order;                // [P] argsort(stable) permutation
  int* src_row;              // [P] token row of each sorted position
  int* rank;                 // [P] sorted position of each pair (inverse of order), or null
  const uint16_t* pair_weights;  // [P] routing weights in pair order, or null
  uint16_t* sorted_weights;  // [P] the same weights in sorted (dispatch) order, or null
  // statistics (any may be null)
  float* utilization;        // [E]
  long long* group_stats;    // [6]
  float* group_ratios;       // [2]
  uint16_t* aux_loss;        // [1] bf16
  const float* lb_partial;   // [lb_blocks, E]
  int lb_blocks;
  float* lb_sum;             // [E] workspace: lb_partial summed over blocks (needed with aux_loss)
  int eligible_experts;        // used when resident == null
  const uint8_t* resident;   // [E] resident mask or null
  int execution_loop;        // 1: reference expert_execution == "loop" telemetry
  const float* recon_error;  // [E] each expert's reconstruction error (spx_expert_quant_error), or null
  float* quant_error;        // [E] out: recon_error of the selected experts, 0 elsewhere, or null
  int* status;
};

struct GemmArgs {
  CUtensorMap tma_a;         // A rows: box {64,128} (unused when gather != 0)
  CUtensorMap tma_b;         // B [groups, N, K]: box {64, bn, 1}
  int m_rows;                // uniform tiling: rows of A
  int k_blocks;              // K / 64
  int bn;                    // N per tile: multiple of 16, 16..256
  int stages;
  uint32_t tmem_cols;        // per accumulator buffer: power of two >= max(32, bn)
  int n_tiles;               // N tiles per M tile (set by launch_gemm)
  int groups;                // B groups (bounds check of the tile table)
  // TMA-loaded B (ungathered A, BF16): K blocks from b_split on come from
  // tma_b2 (K restarting at 0), e.g. [gate | up] along K from two matrices.
  // 0 = B is tma_b alone.
  CUtensorMap tma_b2;
  int b_split;
  int gather;                // 1: A rows gathered through gather_idx with cp.async (a_base/lda)
  const int* gather_idx;
  const uint8_t* a_base;     // gather: A rows (row stride lda bytes)
  int64_t lda;
  const uint8_t* const* a_rows;  // gather: or one pointer per source row (rows of kd BF16), when not null
  // gather (BF16): a copy of the gathered A rows in tile order, copy_out[p] =
  // A row of tile row p, written by the copier warp from the staged stages
  // (tma_copy: copy_out as [rows, kd] BF16, box {64, 32}, 128B swizzle).
  // null = no copy.
  uint16_t* copy_out;
  int64_t ld_copy;
  CUtensorMap tma_copy;
  // kEpiSwiglu, BF16 lane: the BF16-rounded gate | up pre-activations of
  // every tile row, gu_out[p][chunk * 2c + j] (gate j < c, up j >= c).  null = none.
  uint16_t* gu_out;
  int64_t ld_gu;
  // MXFP8 lane (block-scaled kernel only)
  const uint8_t* sfa;        // A scale bytes [A rows, ld_sfa] row-major (row = gathered source row)
  int64_t ld_sfa;            // bytes per row, multiple of 4
  const uint8_t* sfb;        // B scale atoms [groups][n_tiles][k_blocks][512]
  uint8_t* out_sf;           // kEpiSwiglu: hidden scale bytes [rows, ld_out_sf]
  int64_t ld_out_sf;
  const int4* tiles;         // grouped tiling, or null
  const int* num_tiles;
  int n_valid;               // valid output columns
  int chunk;                 // kEpiSwiglu: gate/up half width
  int h_cols;                // kEpiSwiglu: hidden row length incl. zero padding
  void* out;
  int64_t ldo;
  const uint16_t* bias;      // kEpiStore
  const uint16_t* pos_weight;  // kEpiScatter: routing weight of each sorted position
  CUtensorMap tma_out;       // kEpiScatter: Y [P sorted rows, d] BF16, box {64, 32}, 128B swizzle
  int tma_store;             // kEpiScatter: 1 = tma_out is valid (d % 64 == 0)
  const uint16_t* comb_y;    // kEpiCombine: expert rows Y [P, ldy] in sorted order (weights applied)
  const int* comb_rank;      // kEpiCombine: sorted position of pair t*k+j
  int comb_k;                // kEpiCombine: pairs per token (<= kCombineMaxK)
  const uint16_t* comb_res;  // kEpiCombine: residual stream [rows, ldo] or null; with it
  uint16_t* comb_res_out;    //   comb_res_out = bf16(residual + update) (out may then be null)
  int64_t ldy;
  int max_ctas;              // persistent grid cap (0 = every SM): leaves SMs to concurrent work
  // kEpiScatter to other buffers: the row of sorted position p goes to
  // row_out[row_out_idx[p]] (a row pointer, possibly a peer GPU's) instead of
  // out + p * ldo; plain stores (no TMA store).
  uint16_t* const* row_out;
  const int* row_out_idx;
  // NVFP4 lane (block-scaled kernel with E2M1 operands): the epilogue scales
  // the accumulator by the two per-tensor scales, amax / 2688 each, of A
  // (nv_amax_a[expert], the tile's .w; 0 without a tile table) and B
  // (nv_amax_b[group * nv_b_stride + nv_b_off (+1 for the up half of a SwiGLU
  // tile)]); kEpiSwiglu also raises nv_amax_out[expert] to the largest
  // |hidden| it writes.
  const float* nv_amax_a;
  const float* nv_amax_b;
  int nv_b_stride;
  int nv_b_off;
  float* nv_amax_out;
  int* status;
};

// Host helpers (launch.cu): per-device caches so the hot path issues no
// attribute or device queries after the first call on a device.
int device_sm_count();
// Raise `func`'s dynamic shared memory limit to the device maximum once per device.
int ensure_max_dynamic_smem(const void* func);
// A side stream beside the caller's stream `main` (see launch.cu); false when
// none can be made (e.g. the first call is inside a stream capture).
struct SideStream {
  cudaStream_t side;
  cudaEvent_t fork, join, join2;
};
bool side_stream(cudaStream_t main, SideStream* out);

// Launch with programmatic stream serialisation: the kernel may begin while
// the previous kernel in `stream` runs and must call griddep_wait (sm100.cuh)
// before touching anything that kernel or an earlier one writes.  Used by
// the decode-sized layer's kernel chain, where launch latency and kernel
// prologues are a large part of each step; stream capture keeps the
// programmatic edges.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}
// How many 2-CTA clusters of `func` (with `smem` dynamic bytes) fit on the device at once.
int device_max_pairs(const void* func, size_t smem);

int launch_softplus_table(uint16_t* lut, cudaStream_t stream);
// Per-expert reconstruction error of the low-precision copies (quant_error.cu):
// format 1 = MXFP8, 2 = NVFP4; masters in the reference layouts.
int launch_expert_quant_error(const uint16_t* gate, const uint16_t* up, const uint16_t* down, int E, int d, int inter,
                              int format, float* out, cudaStream_t stream);
int launch_scores_from_logits(uint16_t* values, int64_t n, const uint16_t* lut, cudaStream_t stream);
size_t route_select_smem(int num_experts);
int launch_route(const RouteArgs& a, cudaStream_t stream);
int route_lb_blocks(int64_t tokens);  // rows of the route kernel's load-balance partials
int launch_dispatch(const DispatchArgs& a, cudaStream_t stream);

// Tensor maps with 128-byte rows per box (64 BF16 or 128 bytes of E4M3), 128B swizzle.
// `elem_bytes` 2 = BF16, 1 = bytes; `ld` / `cols` in elements.
int encode_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
              int elem_bytes = 2);
int encode_3d(CUtensorMap* map, const void* base, int64_t groups, int64_t rows, int64_t cols, int box_rows,
              int elem_bytes = 2);
size_t gemm_smem_bytes(int bn, int stages, bool mx, int epi, bool nv = false);
int gemm_pick_stages(int bn, int k_blocks, bool mx, int epi, bool nv = false);
// `mx` selects the block-scaled MXFP8 kernel (bn <= 128, k_blocks of 128 elements).
int launch_gemm(int epi, const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream, bool mx = false,
                bool nv = false);
// CTA-pair (cluster of 2, cta_group::2) GEMM: 256-row tiles of a TMA-loaded A.
size_t gemm_pair_smem_bytes(int bn, int stages);
int gemm_pair_pick_stages(int bn);
int launch_gemm_pair(int epi, const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream);

// Router calibration loss term and NLL attribution (calibration.cu).
size_t calibration_workspace_bytes(int64_t B, int64_t S, int E);
int launch_calibration(const uint16_t* scores, const int64_t* ids, const uint16_t* weights, const float* nll,
                       const uint8_t* valid, int64_t B, int64_t S, int E, int k, float* calibration,
                       float* attributed, float* utilization, void* workspace, cudaStream_t stream);

// MXFP8 quantisers (mxfp8.cu).
int launch_mx_quantize_rows(const uint16_t* src, int64_t rows, int cols, int64_t ld_src, int kp, uint8_t* q,
                            int64_t ld_q, uint8_t* sf, int64_t ld_sf, cudaStream_t stream);
size_t mx_atoms_bytes(int groups, int rows_per_group, int kp, int tile_rows);
int launch_mx_quantize_b(int mode, const uint16_t* a, const uint16_t* b, int groups, int rows_per_group,
                         int rows_real, int k_real, int kp, int tile_rows, int d, int inter, int chunk, int64_t ld,
                         uint8_t* q, uint8_t* atoms, cudaStream_t stream);

// update[t] = bf16(base[t] + sum_j rows_j) with rows_j = Y[rank[t*k + j]], or
// bf16(Y[rank[t*k + j]] * w[t*k + j]) when pair weights are given (base: the
// shared SwiGLU output or null).
// combine with a residual add: update (if not null) = bf16(base + sum_j rows_j),
// residual_out = bf16(residual + update).
int launch_combine_residual(const uint16_t* y, const int* rank, const uint16_t* weights, const uint16_t* base,
                            const uint16_t* residual, int64_t tokens, int d, int k, uint16_t* out,
                            uint16_t* residual_out, cudaStream_t stream);
// Channel RMSNorm of the block (nn/norm.py:28-31): x = bf16(bf16(h * bf16(rsqrt(mean(h^2) + eps))) * w),
// rows of x written with stride ld_out (columns [d, ld_out) zeroed).
int launch_rmsnorm_rows(const uint16_t* h, const uint16_t* w, float eps, int64_t rows, int d, uint16_t* out,
                        int ld_out, cudaStream_t stream);
// One page of a paged expert pass: the tiles of the tables whose expert has
// page_slot[e] >= 0, in order, with the group renamed to that cache slot
// (MXFP8 table optional: tiles_mx null).
struct PageTilesArgs {
  const int4* tiles;
  const int* num_tiles;
  const int4* tiles_mx;
  const int* num_tiles_mx;
  const int* page_slot;  // [num_experts]
  int num_experts;
  int4* out;
  int* out_count;
  int4* out_mx;
  int* out_count_mx;
};
int launch_page_tiles(const PageTilesArgs& a, cudaStream_t stream);

// Rows to (peer) buffers: row i (source row index[i] / index_div, or i) of
// segment g (seg[g] <= i < seg[g+1]) is stored at row dst_row[g] + i - seg[g]
// of dst[g]; seg, dst and dst_row are device arrays.  Fences at system scope.
int launch_rows_to_peers(const uint16_t* src, int64_t ld_src, const int* index, int index_div, int64_t rows, int d,
                         const int64_t* seg, uint16_t* const* dst, const int64_t* dst_row, int64_t ld_dst,
                         int groups, cudaStream_t stream);

// Row pointers of received rows in their senders' buffers (peer.cu).
int launch_peer_row_pointers(const int* const* order, const int64_t* send_at, const int64_t* recv_seg, int groups,
                             int top_k, const uint16_t* const* src_rows, int64_t ld, int64_t rows,
                             const uint16_t** out, cudaStream_t stream);

// ---- NVFP4 (nvfp4.cu).  Quantised rows: E2M1 [rows, kp/2] bytes, UE4M3
// scales [rows, kp/16] bytes (kp a multiple of 256; K beyond `cols` is zero).
// Largest |v| of a row-major matrix, raised into *amax (zeroed by the caller).
int launch_nv_amax(const uint16_t* src, int64_t rows, int cols, int64_t ld, float* amax, cudaStream_t stream);
// Largest |v| of every row into row_amax[rows].
int launch_nv_row_amax(const uint16_t* src, int64_t rows, int cols, int64_t ld, float* row_amax,
                       cudaStream_t stream);
// Per tile of a grouped table: amax[expert] (the tile's .w) raised to the
// largest row_amax of the tile's rows (row p -> source row gather[p]).
int launch_nv_tile_amax(const int4* tiles, const int* num_tiles, int max_tiles, const int* gather,
                        const float* row_amax, float* amax, cudaStream_t stream);
// Dense rows with one per-tensor amax (amax[0]).
int launch_nv_quantize_rows(const uint16_t* src, int64_t rows, int cols, int64_t ld, const float* amax, int kp,
                            uint8_t* q, uint8_t* sf, cudaStream_t stream);
// Rows of a grouped table (sorted positions): source row gather[p] (or p),
// per-tensor amax of the tile's expert (.w).
int launch_nv_quantize_tiles(const int4* tiles, const int* num_tiles, int max_tiles, const uint16_t* src,
                             int64_t ld, int cols, const int* gather, const float* amax, int kp, uint8_t* q,
                             uint8_t* sf, cudaStream_t stream);
// B operands at pack time: E2M1 [groups, rows, kp/2] and the scale atoms
// [groups][row tiles][kp/256][4][ceil(tile rows/128)][512]; per-tensor amax
// amax[g * 4 + proj] (W1 rows: proj 0 gate / 1 up; W2: 2; plain rows: 0).
int launch_nv_quantize_b(int mode, const uint16_t* a, const uint16_t* b, int groups, int rows_per_group,
                         int rows_real, int k_real, int kp, int tile_rows, int d, int inter, int chunk, int64_t ld,
                         const float* amax, uint8_t* q, uint8_t* atoms, cudaStream_t stream);
size_t nv_atoms_bytes(int groups, int rows_per_group, int kp, int tile_rows);
// Per group g: amax[g * stride + off] raised to the largest |v| of the group's
// `per_group` consecutive elements of src.
int launch_nv_group_amax(const uint16_t* src, int groups, int64_t per_group, float* amax, int stride, int off,
                         cudaStream_t stream);
// Whole experts into cache slots: dst[a] + slot * bytes[a] <- src[a] + expert * bytes[a]
// for each (expert, slot) of `pairs` (device int32 [num_pairs][2]); sources may be
// mapped page-locked host memory (read by the GPU over the host link).
constexpr int kStageMaxArrays = 8;
struct StageSlotsArgs {
  const uint8_t* src[kStageMaxArrays];
  uint8_t* dst[kStageMaxArrays];
  int64_t bytes[kStageMaxArrays];
  int arrays;
  const int* pairs;
  int num_pairs;
  int num_experts;
  int slots;
  int ctas;     // persistent grid (CTAs of 512 threads)
  int* status;  // device status word | null
};
int launch_stage_slots(StageSlotsArgs a, cudaStream_t stream);
int launch_combine(const uint16_t* y, const int* rank, const uint16_t* weights, const uint16_t* base, int64_t tokens,
                   int d, int k, uint16_t* out, cudaStream_t stream);
// out[i] = src[index[i] / index_div] (BF16 rows of d elements).
int launch_gather_rows(const uint16_t* src, int64_t ld_src, const int* index, int index_div, int64_t rows, int d,
                       uint16_t* out, int64_t ld_out, cudaStream_t stream);

int launch_pack_chunked_w1(const uint16_t* gate, const uint16_t* up, int experts, int d, int inter, int kd,
                           int chunk, int chunks, int transposed_src, uint16_t* out, cudaStream_t stream);
int launch_pack_w2(const uint16_t* down, int experts, int inter, int d, int kp, int transposed_src, uint16_t* out,
                   cudaStream_t stream);
int launch_pad_rows(const uint16_t* src, int64_t rows, int cols, int ld_out, uint16_t* out, cudaStream_t stream);

// Decode-sized projections as grouped GEMVs (gemv.cu).  An expert pass is
// driven by the dispatch's tile tables, like the tcgen05 GEMMs: a tile
// {group, row0, rows <= 128, expert} covers rows [row0, row0 + rows) of the
// dispatch order with the weights of `group` (an expert, or a cache slot in a
// paged pass); the BF16-lane table and the MXFP8-lane table share one launch.
// A dense pass (tiles == null) is one group of dense_rows rows.
constexpr int64_t kGemvMaxPairs = 1024;  // routed pairs up to which the expert projections use GEMVs
constexpr int64_t kGemvMaxTokens = 128;  // tokens up to which router and shared projections use GEMVs
struct GemvPass {
  const int4* tiles;          // BF16-lane tiles, or null (dense pass)
  const int* num_tiles;
  const int4* tiles_mx;       // MXFP8-lane tiles, or null
  const int* num_tiles_mx;
  int max_tiles;              // capacity of each table
  int tile_grid;              // CTAs per table along grid.x (x2 with tiles_mx): a bound on the tiles a
                              // pass can have (<= max_tiles; each tile holds >= 1 pair); 0 = max_tiles
  int dense_rows;
  const int* src_row;         // A row of each row position (gather), or null (identity)
  int* status;                // device status word
  // SwiGLU pass: A = x [*, kd] (or E4M3 xq [*, kx] + xsf), B = chunked [gate | up] rows
  int d, inter, kd, chunk, nc;
  const uint16_t* x;
  int64_t ldx;
  const uint16_t* w1;         // [groups][nc*2*chunk][kd]
  uint16_t* hid;              // [rows][ldh] BF16 hidden rows
  int ldh;
  const uint8_t* xq;          // MXFP8 lane: [*, kx] E4M3 rows, [*, kx/32] scales
  const uint8_t* xsf;
  int kx, cm, ncm, kh;
  const uint8_t* w1q;         // [groups][ncm*2*cm][kx] + scale atoms
  const uint8_t* w1sf;
  uint8_t* hq;                // [rows][kh] E4M3 hidden rows, [rows][kh/32] scales
  uint8_t* hsf;
  // row pass: out[pos, n] = bf16(bf16(<A[pos], W[g][n]> + bias[n]) * row_w[pos])
  const uint16_t* a2;         // A rows [rows][lda2] (BF16; the MXFP8 lane reads hq / hsf)
  int64_t lda2;
  int k2, k_valid2;           // weight row width (BF16 values) and the K that counts
  const uint16_t* w2;         // [groups][n_out][k2]
  const uint8_t* w2q;         // MXFP8 lane: [groups][n_out][kh] + scale atoms (bn2m-row tiles)
  const uint8_t* w2sf;
  int bn2m;
  int n_out;                  // output columns
  int ksplit;                 // warps sharing one m-tile's K (set at launch)
  int mpw;                    // row pass: 16-column m-tiles per warp (set at launch)
  const uint16_t* bias;       // [n_out] or null
  const uint16_t* row_w;      // [rows] or null (unit)
  uint16_t* out;
  int64_t ldo;
};
bool gemv_swiglu_ok(const GemvPass& a);
bool gemv_rows_ok(const GemvPass& a);
int launch_gemv_swiglu(GemvPass a, cudaStream_t stream);
int launch_gemv_rows(GemvPass a, cudaStream_t stream);

// Routed experts' weight gradients (wgrad.cu): out[e] = A_e^T B_e over each
// expert's rows of A [rows, m_total] and B [rows, n_total] (dispatch order,
// counts[e] rows per expert); output columns [0, n_valid0) of B land in out0
// [E, m_total, ld0], columns [n_start1, n_start1 + n_valid1) in out1.
// One operand of the weight-gradient GEMM, P rows in dispatch order: either
// stored (`rows`, row p at rows + p * ld) or gathered (row p is src[index[p]]).
struct WgradOperand {
  const uint16_t* rows;   // [P, ld] sorted rows, or null when gathered
  const uint16_t* src;    // gathered: [*, ld] source rows
  const int* index;       // gathered: index[p] = source row of sorted row p (< src_rows)
  int64_t src_rows;       // gathered: rows of src
  int64_t ld;
  int total;              // columns
};
struct WgradArgs {
  CUtensorMap tma_a, tma_b;  // 128B swizzle; boxes of 64 rows x 64 columns (stored), 1 x 64 (gathered)
  const int* counts;
  int E, m_total, n_total, bn, m_tiles, n_tiles, stages;
  uint16_t* out0;
  int ld0, n_valid0;
  uint16_t* out1;
  int ld1, n_start1, n_valid1;
  // The gathered operand (at most one): A when g_is_a, else B; g_src null = none.
  const uint16_t* g_src;
  const int* g_index;
  int64_t g_ld;
  int g_is_a;
  int* status;
};
int launch_wgrad(const WgradOperand& a, const WgradOperand& b, int64_t rows, const int* counts, int E,
                 uint16_t* out0, int ld0, int n_valid0, uint16_t* out1, int ld1, int n_start1, int n_valid1,
                 int* status, cudaStream_t stream);

// Backward (backward.cu).
struct BwdRouterArgs {
  const uint16_t* scores;     // [T, E] router scores (BF16)
  const uint16_t* logits;     // [T, E] router logits, or null (identity score transform)
  const int64_t* ids;         // [T, k]
  const uint16_t* weights;    // [T, k] routing weights (BF16)
  const float* dw;            // [T, k] gradient of the routing weights
  const float* fractions;     // [E] expert utilization (pairs / P)
  const uint8_t* resident;    // [E] or null
  const uint16_t* d_aux;      // device BF16 scalar, or null (no load-balance gradient)
  const uint16_t* d_scores;   // [T, E] upstream gradient of router_scores, or null
  uint16_t* d_logits;         // [T, E] out
  int64_t tokens;
  int num_experts;
  int top_k;
};
int launch_bwd_swiglu(const uint16_t* gu, int ld_gu, int c, const uint16_t* dhp, int ld_dhp,
                      const uint16_t* sorted_w, const int* order, int64_t P, int I, int kI, uint16_t* h_sorted,
                      uint16_t* dgu, float* dw_pair, cudaStream_t stream);
int launch_bwd_router(const BwdRouterArgs& a, cudaStream_t stream);

}  // namespace spx
