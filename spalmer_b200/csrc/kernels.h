// Internal kernel interfaces of libspx (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "status.h"

namespace spx {

constexpr int kTileRows = 128;         // M of every tcgen05 tile (cta_group::1)
constexpr int kGemmThreads = 320;      // 10 warps: TMA, MMA, 8 x epilogue (2 per TMEM lane quadrant)
constexpr int kGemmEpilogueWarps = 8;
constexpr int kMaxAccBufs = 4;         // TMEM accumulator buffers per CTA (as many as fit in 512 columns)
constexpr size_t kGemmSmemBudget = 227 * 1024;  // sm_100 opt-in maximum per CTA
constexpr int kSliceCols = 64;                  // epilogue staging slice width
constexpr int kStageBytesPerWarp = 32 * kSliceCols * 2;
constexpr int kRouteRows = 128;        // token rows per route_select CTA
constexpr int kTieWarps = 8;           // rows replayed at once per route_ties CTA (one warp each)
constexpr int kMaxTopK = 20;           // MicroExpertsConfig.max_active_experts default
constexpr int kDispatchChunk = 2048;   // pairs per dispatch CTA
constexpr int kDispatchWarps = 4;
constexpr int kDispatchThreads = 32 * kDispatchWarps;

enum Epi : int { kEpiStore = 0, kEpiSwiglu = 1, kEpiScatter = 2, kEpiCombine = 3 };

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
  int4* tiles;               // [ceil(P/128) + E] {expert, row0, rows, 0}
  int* num_tiles;
  int* order;                // [P] argsort(stable) permutation
  int* src_row;              // [P] token row of each sorted position
  const uint16_t* pair_weights;  // [P] routing weights in pair order, or null
  uint16_t* sorted_weights;  // [P] the same weights in sorted (dispatch) order, or null
  // statistics (any may be null)
  float* utilization;        // [E]
  long long* group_stats;    // [6]
  float* group_ratios;       // [2]
  uint16_t* aux_loss;        // [1] bf16
  const float* lb_partial;   // [lb_blocks, E]
  int lb_blocks;
  int eligible_experts;        // used when resident == null
  const uint8_t* resident;   // [E] resident mask or null
  int execution_loop;        // 1: reference expert_execution == "loop" telemetry
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
  int gather;                // 1: A rows gathered through gather_idx with cp.async (a_base/lda)
  const int* gather_idx;
  const uint16_t* a_base;    // gather: A rows (row stride lda elements)
  int64_t lda;
  const int4* tiles;         // grouped tiling, or null
  const int* num_tiles;
  int n_valid;               // valid output columns
  int chunk;                 // kEpiSwiglu: gate/up half width
  int h_cols;                // kEpiSwiglu: hidden row length incl. zero padding
  void* out;
  int64_t ldo;
  const uint16_t* bias;      // kEpiStore
  const int* pos_to_pair;    // kEpiScatter: pair index of each sorted position
  const uint16_t* pos_weight;  // kEpiScatter: routing weight of each sorted position
  const uint16_t* y_pairs;   // kEpiCombine
  int64_t ld_y;
  int top_k;
  int* status;
};

// Host helpers (launch.cu): per-device caches so the hot path issues no
// attribute or device queries after the first call on a device.
int device_sm_count();
// Raise `func`'s dynamic shared memory limit to the device maximum once per device.
int ensure_max_dynamic_smem(const void* func);

int launch_softplus_table(uint16_t* lut, cudaStream_t stream);
size_t route_select_smem(int num_experts);
int launch_route(const RouteArgs& a, cudaStream_t stream);
int launch_dispatch(const DispatchArgs& a, cudaStream_t stream);

int encode_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows);
int encode_3d(CUtensorMap* map, const void* base, int64_t groups, int64_t rows, int64_t cols, int box_rows);
size_t gemm_smem_bytes(int bn, int stages);
int gemm_pick_stages(int bn, int k_blocks);
int launch_gemm(int epi, const GemmArgs& a, int grid_m, int grid_n, cudaStream_t stream);

int launch_combine(const uint16_t* y, int64_t tokens, int d, int k, uint16_t* out, cudaStream_t stream);

int launch_pack_chunked_w1(const uint16_t* gate, const uint16_t* up, int experts, int d, int inter, int kd,
                           int chunk, int chunks, int transposed_src, uint16_t* out, cudaStream_t stream);
int launch_pack_w2(const uint16_t* down, int experts, int inter, int d, int kp, int transposed_src, uint16_t* out,
                   cudaStream_t stream);
int launch_pad_rows(const uint16_t* src, int64_t rows, int cols, int ld_out, uint16_t* out, cudaStream_t stream);

}  // namespace spx
