// C ABI of libspx (declared in include/spx.h): shapes, workspace layout,
// weight packing and the orchestration of one mixer layer forward.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstring>

#include "kernels.h"
#include "nv.cuh"
#include "sm100.cuh"

namespace spx {
namespace {

constexpr size_t kAlign = 256;

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
int round_up_i(int v, int a) { return (v + a - 1) / a * a; }
int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

uint32_t pow2_at_least(uint32_t v) {
  uint32_t p = 32;
  while (p < v) p <<= 1;
  return p;
}

struct Shape {
  int64_t T, P;
  int d, E, I, S, k;
  int kd;             // d padded to 64 (GEMM1 / router K)
  int c, nc, kp;      // expert GEMM1 chunk, chunks, hidden width padded to 64
  int cs, ncs, ksp;   // shared GEMM1 chunk, chunks, hidden width padded to 64
  bool small;         // decode-sized batch (narrow tiles, single CTAs)
  int bn_router, gn_router;
  int bn_d, gn_d;     // expert down projection N tile
  int bn_sd, gn_sd;   // shared down projection N tile
  int lb_blocks, nchunks, max_tiles;
  // MXFP8 lane
  bool mx;
  int kx;             // GEMM1 K in bytes (d padded to 128)
  int cm, ncm;        // GEMM1 chunk (N tile = 2*cm, up to 256) and chunks
  int kh;             // hidden width in bytes (I padded to 128) = GEMM2 K
  int bn2m, gn2m;     // GEMM2 N tile and tiles
  // NVFP4 lane (dims->mxfp8_lane == 2): the low-precision lane runs the
  // ("nvfp4", "nvfp4") pair; chunking (cm, ncm, bn2m) as the MXFP8 lane.
  bool nv;
  int kxn, khn;       // GEMM1 / GEMM2 K in elements, padded to 256 (128-byte stages of E2M1)
};

int make_shape(const spx_layer_dims* dm, Shape* s) {
  if (dm == nullptr || s == nullptr) return SPX_ERR_INVALID_ARG;
  s->T = dm->tokens;
  s->d = dm->d_model;
  s->E = dm->num_experts;
  s->I = dm->inter_dim;
  s->S = dm->shared_dim;
  s->k = dm->top_k;
  if (s->T < 1 || s->d < 1 || s->E < 1 || s->I < 1 || s->S < 0 || s->k < 1) return SPX_ERR_INVALID_ARG;
  if (s->k > s->E || s->k > kMaxTopK || s->E > 1024 || s->E > 65535) return SPX_ERR_UNSUPPORTED;
  if (s->T * s->k > (int64_t(1) << 31) - 1) return SPX_ERR_UNSUPPORTED;
  s->P = s->T * s->k;
  s->kd = round_up_i(s->d, 64);
  // Decode-sized batches read weights far more than they compute: the router
  // and shared GEMMs (one M tile) take narrow N tiles so each weight matrix
  // spreads over more CTAs.  The packed shared GEMM1 layout follows its chunk
  // width, so it depends on this class.
  const bool small = s->T <= kSmallBatchTokens;
  s->small = small;
  const int wide = small ? 32 : 128;
  s->c = std::min(round_up_i(s->I, 16), 128);
  s->nc = ceil_div(s->I, s->c);
  s->kp = round_up_i(s->nc * s->c, 64);
  if (s->S > 0) {
    s->cs = std::min(round_up_i(s->S, 16), wide);
    s->ncs = ceil_div(s->S, s->cs);
    s->ksp = round_up_i(s->ncs * s->cs, 64);
  } else {
    s->cs = s->ncs = s->ksp = 0;
  }
  s->bn_router = std::min(small ? 32 : 256, round_up_i(s->E, 16));
  s->gn_router = ceil_div(s->E, s->bn_router);
  s->bn_d = std::min(256, round_up_i(s->d, 16));
  s->gn_d = ceil_div(s->d, s->bn_d);
  s->bn_sd = std::min(small ? 64 : 256, round_up_i(s->d, 16));
  s->gn_sd = ceil_div(s->d, s->bn_sd);
  s->lb_blocks = route_lb_blocks(s->T);
  s->nchunks = ceil_div(s->P, kDispatchChunk);
  s->max_tiles = ceil_div(s->P, kTileRows) + s->E;
  if (dm->mxfp8_lane < 0 || dm->mxfp8_lane > 2) return SPX_ERR_INVALID_ARG;
  s->mx = dm->mxfp8_lane != 0;
  s->nv = dm->mxfp8_lane == 2;
  s->kxn = round_up_i(s->d, 256);
  s->khn = round_up_i(s->I, 256);
  if (s->mx) {
    if (s->I % kMxBlock != 0) return SPX_ERR_UNSUPPORTED;
    s->kx = round_up_i(s->d, 128);
    // GEMM1 chunk (N tile = 2 * cm).  The NVFP4 lane takes 64-column chunks:
    // 128-column tiles leave TMEM room for three accumulators below the scale
    // slots, so a tile's epilogue overlaps the next tile's MMAs (measured
    // 1.49 -> 1.46 ms on the 100M shape); the MXFP8 lane is faster with
    // 256-column tiles (1.17 vs 1.22 ms), whose A rows load once per tile.
    s->cm = s->nv ? ((s->I % 64 == 0) ? 64 : 32) : (s->I % 128 == 0) ? 128 : (s->I % 64 == 0) ? 64 : 32;
    s->ncm = s->I / s->cm;
    s->kh = round_up_i(s->I, 128);
    // GEMM2 N tile.  The MXFP8 lane takes 256 columns: with K = I = 128 a tile
    // is one K block, so its fixed costs (scale copies, accumulator hand-off,
    // the A tile's load) weigh more than the lost accumulator overlap
    // (expert GEMM2 stage 207.7 -> 201.9 us on the 100M shape).
    s->bn2m = s->nv ? std::min(kMxDenseBn, round_up_i(s->d, 16)) : std::min(kMxMaxBn, round_up_i(s->d, 16));
    s->gn2m = ceil_div(s->d, s->bn2m);
  } else {
    s->kx = s->cm = s->ncm = s->kh = s->bn2m = s->gn2m = 0;
  }
  return SPX_OK;
}

// Byte sizes of the MXFP8 weight copies.
struct MxPackSizes {
  size_t w1, w1_sf, w2, w2_sf;
};

MxPackSizes mx_pack_sizes(const Shape& s) {
  MxPackSizes z{};
  if (!s.mx) return z;
  const int rows1 = s.ncm * 2 * s.cm;
  if (s.nv) {
    z.w1 = static_cast<size_t>(s.E) * rows1 * (s.kxn / 2);
    z.w1_sf = nv_atoms_bytes(s.E, rows1, s.kxn, 2 * s.cm);
    z.w2 = static_cast<size_t>(s.E) * s.d * (s.khn / 2);
    z.w2_sf = nv_atoms_bytes(s.E, s.d, s.khn, s.bn2m);
    return z;
  }
  z.w1 = static_cast<size_t>(s.E) * rows1 * s.kx;
  z.w1_sf = mx_atoms_bytes(s.E, rows1, s.kx, 2 * s.cm);
  z.w2 = static_cast<size_t>(s.E) * s.d * s.kh;
  z.w2_sf = mx_atoms_bytes(s.E, s.d, s.kh, s.bn2m);
  return z;
}

struct Layout {
  size_t small, tie_rows, lb_partial, lb_sum, chunk_hist, counts, starts, tiles, order, src_row, rank, sorted_w;
  size_t hidden, y, shared_hidden, shared_out, x_pad, x_norm, util, stats, ratios, aux;
  size_t x_q, x_sf, h_q, h_sf, tiles_mx;  // MXFP8 lane (empty otherwise)
  size_t tiles_page, tiles_mx_page;        // one page of a paged expert pass
  size_t nv_row_amax, nv_amax;             // NVFP4 lane: per-token amax [T]; per-expert amax of x, h [2][E]
  size_t total;
};

Layout make_layout(const Shape& s) {
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = round_up(off + bytes, kAlign);
    return at;
  };
  L.small = take(64);
  L.tie_rows = take(sizeof(int) * s.T);
  L.lb_partial = take(sizeof(float) * static_cast<size_t>(s.lb_blocks) * s.E);
  L.lb_sum = take(sizeof(float) * s.E);
  L.chunk_hist = take(sizeof(int) * static_cast<size_t>(s.nchunks) * s.E);
  L.counts = take(sizeof(int) * s.E);
  L.starts = take(sizeof(int) * s.E);
  L.tiles = take(sizeof(int4) * static_cast<size_t>(s.max_tiles));
  L.order = take(sizeof(int) * s.P);
  L.src_row = take(sizeof(int) * s.P);
  L.rank = take(sizeof(int) * s.P);
  L.sorted_w = take(sizeof(uint16_t) * s.P);
  L.hidden = take(2 * static_cast<size_t>(s.P) * s.kp);
  L.y = take(2 * static_cast<size_t>(s.P) * s.d);
  L.shared_hidden = take(s.S > 0 ? 2 * static_cast<size_t>(s.T) * s.ksp : 0);
  L.shared_out = take(s.S > 0 ? 2 * static_cast<size_t>(s.T) * s.d : 0);
  L.x_pad = take(s.kd != s.d ? 2 * static_cast<size_t>(s.T) * s.kd : 0);
  L.x_norm = take(2 * static_cast<size_t>(s.T) * s.kd);
  L.util = take(sizeof(float) * s.E);
  L.stats = take(sizeof(long long) * 6);
  L.ratios = take(sizeof(float) * 2);
  L.aux = take(sizeof(uint16_t) * 2);
  if (s.nv) {  // E2M1 rows per routed pair (each expert's input has its own per-tensor scale)
    L.x_q = take(static_cast<size_t>(s.P) * (s.kxn / 2));
    L.x_sf = take(static_cast<size_t>(s.P) * (s.kxn / kNvBlock));
    L.h_q = take(static_cast<size_t>(s.P) * (s.khn / 2));
    L.h_sf = take(static_cast<size_t>(s.P) * (s.khn / kNvBlock));
  } else {
    L.x_q = take(s.mx ? static_cast<size_t>(s.T) * s.kx : 0);
    L.x_sf = take(s.mx ? static_cast<size_t>(s.T) * (s.kx / kMxBlock) : 0);
    L.h_q = take(s.mx ? static_cast<size_t>(s.P) * s.kh : 0);
    L.h_sf = take(s.mx ? static_cast<size_t>(s.P) * (s.kh / kMxBlock) : 0);
  }
  L.tiles_mx = take(s.mx ? sizeof(int4) * static_cast<size_t>(s.max_tiles) : 0);
  L.tiles_page = take(sizeof(int4) * static_cast<size_t>(s.max_tiles));
  L.tiles_mx_page = take(s.mx ? sizeof(int4) * static_cast<size_t>(s.max_tiles) : 0);
  L.nv_row_amax = take(s.nv ? sizeof(float) * static_cast<size_t>(s.T) : 0);
  L.nv_amax = take(s.nv ? sizeof(float) * 2 * static_cast<size_t>(s.E) : 0);
  L.total = off;
  return L;
}

template <typename T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(ws) + off);
}

int sm_count() { return device_sm_count(); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

GemmArgs base_args(int epi, int bn, int k_blocks, int* status, bool mx = false, bool nv = false) {
  GemmArgs g{};
  g.bn = bn;
  g.k_blocks = k_blocks;
  g.stages = gemm_pick_stages(bn, k_blocks, mx, epi, nv);
  g.tmem_cols = pow2_at_least(static_cast<uint32_t>(bn));
  g.groups = 1;
  g.status = status;
  return g;
}

int run_route(const Shape& s, const uint16_t* logits, const uint16_t* lut, const uint8_t* resident,
              uint16_t* scores, int64_t* ids, uint16_t* weights, void* ws, const Layout& L,
              cudaStream_t st) {
  int* small = at<int>(ws, L.small);
  if (cudaMemsetAsync(small + 1, 0, sizeof(int), st) != cudaSuccess) return SPX_ERR_CUDA;
  RouteArgs r{};
  r.logits = logits;
  r.lut = lut;
  r.resident = resident;
  r.scores = scores;
  r.ids = ids;
  r.weights = weights;
  r.tie_count = small + 1;
  r.tie_rows = at<int>(ws, L.tie_rows);
  r.lb_partial = at<float>(ws, L.lb_partial);
  r.tokens = s.T;
  r.num_experts = s.E;
  r.top_k = s.k;
  r.sm_count = sm_count();
  r.status = small;
  return launch_route(r, st);
}

DispatchArgs dispatch_args(const Shape& s, const int64_t* ids, int* order, int* counts, void* ws,
                           const Layout& L) {
  DispatchArgs a{};
  a.ids = ids;
  a.pairs = s.P;
  a.tokens = s.T;
  a.num_experts = s.E;
  a.top_k = s.k;
  a.chunk_hist = at<int>(ws, L.chunk_hist);
  a.counts = counts != nullptr ? counts : at<int>(ws, L.counts);
  a.starts = at<int>(ws, L.starts);
  a.tiles = at<int4>(ws, L.tiles);
  a.num_tiles = at<int>(ws, L.small) + 2;
  a.order = order != nullptr ? order : at<int>(ws, L.order);
  a.src_row = at<int>(ws, L.src_row);
  a.rank = at<int>(ws, L.rank);
  a.lb_partial = at<float>(ws, L.lb_partial);
  a.lb_sum = at<float>(ws, L.lb_sum);
  a.lb_blocks = s.lb_blocks;
  a.eligible_experts = s.E;
  a.status = at<int>(ws, L.small);
  return a;
}

// One layer's launch context: shape, workspace layout, stream, status word
// and (full layer only) the stage events.
struct Ctx {
  const Shape& s;
  const Layout& L;
  void* ws;
  cudaStream_t st;
  int* status;
  void* const* events;
  void mark(int i) const {
    if (events != nullptr && events[i] != nullptr) cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
  }
};

// A operand source: the hidden states, zero-padded to a multiple of 64 columns if needed.
int stage_pad(const Ctx& c, const uint16_t* hidden, const uint16_t** xa) {
  *xa = hidden;
  if (c.s.kd == c.s.d) return SPX_OK;
  uint16_t* xp = at<uint16_t>(c.ws, c.L.x_pad);
  if (int rc = launch_pad_rows(hidden, c.s.T, c.s.d, c.s.kd, xp, c.st); rc != SPX_OK) return rc;
  *xa = xp;
  return SPX_OK;
}

// Dense GEMV pass for decode-sized batches: rows = the batch's tokens.
GemvPass dense_rows_pass(const Ctx& c, const uint16_t* a, int64_t lda, int k, int k_valid, const uint16_t* w, int n,
                         const uint16_t* bias, uint16_t* out, int64_t ldo) {
  GemvPass g{};
  g.dense_rows = static_cast<int>(c.s.T);
  g.status = c.status;
  g.a2 = a;
  g.lda2 = lda;
  g.k2 = k;
  g.k_valid2 = k_valid;
  g.w2 = w;
  g.n_out = n;
  g.bias = bias;
  g.out = out;
  g.ldo = ldo;
  return g;
}

// K1: router logits (tcgen05 GEMM, bias fused) into `lg`; a GEMV for decode-sized batches.
int stage_router(const Ctx& c, const spx_packed_weights* w, const uint16_t* xa, uint16_t* lg) {
  const Shape& s = c.s;
  if (s.T <= kGemvMaxTokens) {
    const GemvPass g = dense_rows_pass(c, xa, s.kd, s.kd, s.kd, w->router_weight, s.E, w->router_bias, lg, s.E);
    if (gemv_rows_ok(g)) return launch_gemv_rows(g, c.st);
  }
  GemmArgs g = base_args(kEpiStore, s.bn_router, s.kd / 64, c.status);
  if (int rc = encode_2d(&g.tma_a, xa, s.T, s.kd, s.kd, kTileRows); rc != SPX_OK) return rc;
  if (int rc = encode_3d(&g.tma_b, w->router_weight, 1, s.E, s.kd, s.bn_router); rc != SPX_OK) return rc;
  g.m_rows = static_cast<int>(s.T);
  g.n_valid = s.E;
  g.out = lg;
  g.ldo = s.E;
  g.bias = w->router_bias;
  return launch_gemm(kEpiStore, g, ceil_div(s.T, kTileRows), s.gn_router, c.st);
}

// K1 of a layer: router GEMM, then scores / top-k / weights / load-balance
// partials.  Unless the caller injects logits or asks for them, the GEMM
// writes the logits into router_scores and the route maps them to scores in
// place (each route CTA reads its rows before it writes them).
int stage_router_route(const Ctx& c, const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* xa,
                       const spx_layer_outputs* out) {
  const Shape& s = c.s;
  const uint16_t* lut = dims->score_transform == 0 ? w->softplus_table : nullptr;
  int rc = SPX_OK;
  const uint16_t* logits = out->injected_logits;
  if (logits == nullptr) {
    uint16_t* lg = out->router_logits != nullptr ? out->router_logits : out->router_scores;
    if ((rc = stage_router(c, w, xa, lg)) != SPX_OK) return rc;
    logits = lg;
  }
  c.mark(1);
  return run_route(s, logits, lut, w->resident_mask, out->router_scores, out->expert_ids, out->routing_weights,
                   c.ws, c.L, c.st);
}

// K2 arguments for the layer's dispatch: statistics into the caller's outputs
// (or workspace dummies), sorted weights, ranks, the MXFP8 tile table.
DispatchArgs layer_dispatch_args(const Ctx& c, const spx_layer_dims* dims, const spx_packed_weights* w,
                                 const spx_layer_outputs* out) {
  const Shape& s = c.s;
  void* ws = c.ws;
  const Layout& L = c.L;
  DispatchArgs da = dispatch_args(s, out->expert_ids, out->dispatch_order, out->expert_counts, ws, L);
  da.utilization = out->expert_utilization != nullptr ? out->expert_utilization : at<float>(ws, L.util);
  da.group_stats = out->group_stats != nullptr ? reinterpret_cast<long long*>(out->group_stats)
                                               : at<long long>(ws, L.stats);
  da.group_ratios = out->group_ratios != nullptr ? out->group_ratios : at<float>(ws, L.ratios);
  da.aux_loss = out->auxiliary_loss != nullptr ? out->auxiliary_loss : at<uint16_t>(ws, L.aux);
  da.resident = w->resident_mask;
  da.execution_loop = dims->execution_loop;
  da.recon_error = w->expert_quant_error;
  da.quant_error = out->expert_quantization_error;
  da.pair_weights = out->routing_weights;
  da.sorted_weights = at<uint16_t>(ws, L.sorted_w);
  if (out->pair_rank != nullptr) da.rank = out->pair_rank;
  if (s.mx && w->expert_lane_mxfp8 != nullptr) {
    da.lane_mx = w->expert_lane_mxfp8;
    da.tiles_mx = at<int4>(ws, L.tiles_mx);
    da.num_tiles_mx = at<int>(ws, L.small) + 3;
  }
  return da;
}

// Expert weights and tile tables of one expert pass: the whole bank (groups =
// E, the dispatch's tables) or one page of a paged pass (groups = cache
// slots, the page's tables with groups renamed to slots).
struct ExpertPass {
  const uint16_t* w1;
  const uint16_t* w2;
  const uint8_t* w1_mx;
  const uint8_t* w1_mx_sf;
  const uint8_t* w2_mx;
  const uint8_t* w2_mx_sf;
  int groups;
  const int4* tiles;
  const int* num_tiles;
  const int4* tiles_mx;  // null: no low-precision lane in this pass
  const int* num_tiles_mx;
  int max_ctas;  // persistent grid cap of the GEMMs (0 = every SM)
  const float* nv_amax_w;  // NVFP4 lane: weight amax [groups][4] (gate, up, down, unused)
  uint16_t* const* row_out = nullptr;  // GEMM2 rows to row_out[row_out_idx[p]] instead of Y
  const int* row_out_idx = nullptr;
  const uint8_t* const* a_rows = nullptr;  // BF16 GEMM1 rows through one pointer per source row
  uint16_t* saved_x = nullptr;   // training: BF16 GEMM1's gathered rows in dispatch order [P, d]
  uint16_t* saved_gu = nullptr;  // training: BF16 GEMM1's gate | up pre-activations [P, nc * 2c]
};

// NVFP4 lane input: each expert's rows in dispatch order as E2M1 with UE4M3
// block scales under the expert's own per-tensor scale (amax over its rows,
// experts/native.py:240-256 per expert call); zeroes the per-expert hidden
// amax that the NVFP4 GEMM1 epilogue raises.
int stage_quantize_nv_x(const Ctx& c, const uint16_t* hidden, int64_t ld_hidden, const DispatchArgs& da) {
  const Shape& s = c.s;
  const int64_t ld = ld_hidden > 0 ? ld_hidden : s.d;
  float* amax = at<float>(c.ws, c.L.nv_amax);  // [x | h][E]
  float* row_amax = at<float>(c.ws, c.L.nv_row_amax);
  if (cudaMemsetAsync(amax, 0, sizeof(float) * 2 * s.E, c.st) != cudaSuccess) return SPX_ERR_CUDA;
  int rc = launch_nv_row_amax(hidden, s.T, s.d, ld, row_amax, c.st);
  if (rc == SPX_OK)
    rc = launch_nv_tile_amax(da.tiles_mx, da.num_tiles_mx, s.max_tiles, da.src_row, row_amax, amax, c.st);
  if (rc == SPX_OK)
    rc = launch_nv_quantize_tiles(da.tiles_mx, da.num_tiles_mx, s.max_tiles, hidden, ld, s.d, da.src_row, amax,
                                  s.kxn, at<uint8_t>(c.ws, c.L.x_q), at<uint8_t>(c.ws, c.L.x_sf), c.st);
  return rc;
}

// MXFP8 lane input: E4M3 rows of the hidden states with their block scales
// (per token, so every expert's gathered rows share them).
int stage_quantize_x(const Ctx& c, const uint16_t* hidden, int64_t ld_hidden) {
  const Shape& s = c.s;
  return launch_mx_quantize_rows(hidden, s.T, s.d, ld_hidden > 0 ? ld_hidden : s.d, s.kx, at<uint8_t>(c.ws, c.L.x_q),
                                 s.kx, at<uint8_t>(c.ws, c.L.x_sf), s.kx / kMxBlock, c.st);
}

// Decode-sized batches (<= kGemvMaxPairs routed pairs): the expert projections
// of a pass as grouped GEMVs (gemv.cu) over the same tile tables, both lanes in
// one launch per projection; same outputs as the GEMMs below.  Returns 1 when
// the pass does not qualify (NVFP4 lane, peer row pointers, shapes).
int expert_gemvs(const Ctx& c, const uint16_t* xa, const int* src_row, const uint16_t* sorted_w,
                 const ExpertPass& p) {
  const Shape& s = c.s;
  if (s.P > kGemvMaxPairs || s.nv || p.row_out != nullptr || p.a_rows != nullptr || xa == nullptr ||
      p.saved_x != nullptr)
    return 1;
  GemvPass g{};
  g.tiles = p.tiles;
  g.num_tiles = p.num_tiles;
  g.tiles_mx = p.tiles_mx;
  g.num_tiles_mx = p.num_tiles_mx;
  g.max_tiles = s.max_tiles;
  g.tile_grid = static_cast<int>(std::min<int64_t>(s.max_tiles, s.P));  // a tile holds >= 1 pair
  g.src_row = src_row;
  g.status = c.status;
  g.d = s.d;
  g.inter = s.I;
  g.kd = s.kd;
  g.chunk = s.c;
  g.nc = s.nc;
  g.x = xa;
  g.ldx = s.kd;
  g.w1 = p.w1;
  g.hid = at<uint16_t>(c.ws, c.L.hidden);
  g.ldh = s.kp;
  g.a2 = g.hid;
  g.lda2 = s.kp;
  g.k2 = s.kp;
  g.k_valid2 = s.I;
  g.w2 = p.w2;
  g.n_out = s.d;
  g.row_w = sorted_w;
  g.out = at<uint16_t>(c.ws, c.L.y);
  g.ldo = s.d;
  if (p.tiles_mx != nullptr) {
    g.xq = at<uint8_t>(c.ws, c.L.x_q);
    g.xsf = at<uint8_t>(c.ws, c.L.x_sf);
    g.kx = s.kx;
    g.cm = s.cm;
    g.ncm = s.ncm;
    g.kh = s.kh;
    g.bn2m = s.bn2m;
    g.w1q = p.w1_mx;
    g.w1sf = p.w1_mx_sf;
    g.w2q = p.w2_mx;
    g.w2sf = p.w2_mx_sf;
    g.hq = at<uint8_t>(c.ws, c.L.h_q);
    g.hsf = at<uint8_t>(c.ws, c.L.h_sf);
  }
  if (!gemv_swiglu_ok(g) || !gemv_rows_ok(g)) return 1;
  if (int rc = launch_gemv_swiglu(g, c.st); rc != SPX_OK) return rc;
  c.mark(4);
  g.src_row = nullptr;  // the down projection reads the hidden rows in dispatch order
  if (int rc = launch_gemv_rows(g, c.st); rc != SPX_OK) return rc;
  c.mark(5);
  return SPX_OK;
}

// K3 GEMMs: expert GEMM1 (+SwiGLU) and GEMM2 over the tiles of `p`, rows
// gathered from `xa` through src_row; weighted rows land in Y (sorted order).
int stage_expert_gemms(const Ctx& c, const uint16_t* xa, const int* src_row, const uint16_t* sorted_w,
                       const ExpertPass& p) {
  const Shape& s = c.s;
  void* ws = c.ws;
  const Layout& L = c.L;
  int rc = SPX_OK;
  if ((rc = expert_gemvs(c, xa, src_row, sorted_w, p)) != 1) return rc;
  rc = SPX_OK;
  const bool mx = p.tiles_mx != nullptr && !s.nv;
  const bool nv = p.tiles_mx != nullptr && s.nv;
  float* nv_amax_x = at<float>(ws, L.nv_amax);
  float* nv_amax_h = nv_amax_x + s.E;
  uint8_t* xq = at<uint8_t>(ws, L.x_q);
  uint8_t* xsf = at<uint8_t>(ws, L.x_sf);
  uint8_t* hq = at<uint8_t>(ws, L.h_q);
  uint8_t* hsf = at<uint8_t>(ws, L.h_sf);
  uint16_t* hid = at<uint16_t>(ws, L.hidden);
  uint16_t* y = at<uint16_t>(ws, L.y);
  {
    GemmArgs g = base_args(kEpiSwiglu, 2 * s.c, s.kd / 64, c.status);
    if ((rc = encode_3d(&g.tma_b, p.w1, p.groups, static_cast<int64_t>(s.nc) * 2 * s.c, s.kd, 2 * s.c)) != SPX_OK)
      return rc;
    g.groups = p.groups;
    g.max_ctas = p.max_ctas;
    g.gather = 1;
    g.gather_idx = src_row;
    g.a_base = reinterpret_cast<const uint8_t*>(xa);
    g.lda = 2 * static_cast<int64_t>(s.kd);
    g.a_rows = p.a_rows;
    g.tiles = p.tiles;
    g.num_tiles = p.num_tiles;
    g.chunk = s.c;
    g.h_cols = s.kp;
    g.out = hid;
    g.ldo = s.kp;
    if (p.saved_x != nullptr) {  // training: the rows and the pre-activations, for the backward
      g.copy_out = p.saved_x;
      g.ld_copy = s.d;
      if ((rc = encode_2d(&g.tma_copy, p.saved_x, s.P, s.d, s.d, 32)) != SPX_OK) return rc;
      g.gu_out = p.saved_gu;
      g.ld_gu = static_cast<int64_t>(s.nc) * 2 * s.c;
    }
    if ((rc = launch_gemm(kEpiSwiglu, g, s.max_tiles, s.nc, c.st)) != SPX_OK) return rc;
  }
  if (mx) {
    // MXFP8-lane experts: block-scaled GEMM1, hidden written quantised.
    GemmArgs g = base_args(kEpiSwiglu, 2 * s.cm, s.kx / 128, c.status, true);
    if ((rc = encode_3d(&g.tma_b, p.w1_mx, p.groups, static_cast<int64_t>(s.ncm) * 2 * s.cm, s.kx, 2 * s.cm,
                        1)) != SPX_OK)
      return rc;
    g.groups = p.groups;
    g.max_ctas = p.max_ctas;
    g.gather = 1;
    g.gather_idx = src_row;
    g.a_base = xq;
    g.lda = s.kx;
    g.sfa = xsf;
    g.ld_sfa = s.kx / kMxBlock;
    g.sfb = p.w1_mx_sf;
    g.tiles = p.tiles_mx;
    g.num_tiles = p.num_tiles_mx;
    g.chunk = s.cm;
    g.h_cols = s.kh;
    g.out = hq;
    g.ldo = s.kh;
    g.out_sf = hsf;
    g.ld_out_sf = s.kh / kMxBlock;
    if ((rc = launch_gemm(kEpiSwiglu, g, s.max_tiles, s.ncm, c.st, true)) != SPX_OK) return rc;
  }
  if (nv) {
    // NVFP4-lane experts: block-scaled E2M1 GEMM1, BF16 hidden rows (their
    // per-expert amax raised by the epilogue), then the hidden rows quantised
    // under each expert's scale.
    GemmArgs g = base_args(kEpiSwiglu, 2 * s.cm, s.kxn / 256, c.status, true, true);
    if ((rc = encode_3d(&g.tma_b, p.w1_mx, p.groups, static_cast<int64_t>(s.ncm) * 2 * s.cm, s.kxn / 2, 2 * s.cm,
                        1)) != SPX_OK)
      return rc;
    if ((rc = encode_2d(&g.tma_a, xq, s.P, s.kxn / 2, s.kxn / 2, kTileRows, 1)) != SPX_OK) return rc;
    g.groups = p.groups;
    g.max_ctas = p.max_ctas;
    g.sfa = xsf;
    g.ld_sfa = s.kxn / kNvBlock;
    g.sfb = p.w1_mx_sf;
    g.tiles = p.tiles_mx;
    g.num_tiles = p.num_tiles_mx;
    g.chunk = s.cm;
    g.h_cols = s.kp;
    g.out = hid;
    g.ldo = s.kp;
    g.nv_amax_a = nv_amax_x;
    g.nv_amax_b = p.nv_amax_w;
    g.nv_b_stride = 4;
    g.nv_b_off = 0;
    g.nv_amax_out = nv_amax_h;
    if ((rc = launch_gemm(kEpiSwiglu, g, s.max_tiles, s.ncm, c.st, true, true)) != SPX_OK) return rc;
    if ((rc = launch_nv_quantize_tiles(p.tiles_mx, p.num_tiles_mx, s.max_tiles, hid, s.kp, s.I, nullptr, nv_amax_h,
                                       s.khn, hq, hsf, c.st)) != SPX_OK)
      return rc;
  }
  c.mark(4);
  {
    GemmArgs g = base_args(kEpiScatter, s.bn_d, s.kp / 64, c.status);
    if ((rc = encode_2d(&g.tma_a, hid, s.P, s.kp, s.kp, kTileRows)) != SPX_OK) return rc;
    if ((rc = encode_3d(&g.tma_b, p.w2, p.groups, s.d, s.kp, s.bn_d)) != SPX_OK) return rc;
    g.groups = p.groups;
    g.max_ctas = p.max_ctas;
    g.tiles = p.tiles;
    g.num_tiles = p.num_tiles;
    g.n_valid = s.d;
    g.out = y;
    g.ldo = s.d;
    g.tma_store = (s.d % 64) == 0;  // whole 64-column boxes; other widths use plain stores
    if (g.tma_store && (rc = encode_2d(&g.tma_out, y, s.P, s.d, s.d, 32)) != SPX_OK) return rc;
    g.pos_weight = sorted_w;
    g.row_out = p.row_out;
    g.row_out_idx = p.row_out_idx;
    if (p.row_out != nullptr) g.tma_store = 0;
    if ((rc = launch_gemm(kEpiScatter, g, s.max_tiles, s.gn_d, c.st)) != SPX_OK) return rc;
  }
  if (mx) {
    GemmArgs g = base_args(kEpiScatter, s.bn2m, s.kh / 128, c.status, true);
    if ((rc = encode_2d(&g.tma_a, hq, s.P, s.kh, s.kh, kTileRows, 1)) != SPX_OK) return rc;
    if ((rc = encode_3d(&g.tma_b, p.w2_mx, p.groups, s.d, s.kh, s.bn2m, 1)) != SPX_OK) return rc;
    g.groups = p.groups;
    g.max_ctas = p.max_ctas;
    g.tiles = p.tiles_mx;
    g.num_tiles = p.num_tiles_mx;
    g.sfa = hsf;
    g.ld_sfa = s.kh / kMxBlock;
    g.sfb = p.w2_mx_sf;
    g.n_valid = s.d;
    g.out = y;
    g.ldo = s.d;
    g.tma_store = (s.d % 64) == 0;
    if (g.tma_store && (rc = encode_2d(&g.tma_out, y, s.P, s.d, s.d, 32)) != SPX_OK) return rc;
    g.pos_weight = sorted_w;
    g.row_out = p.row_out;
    g.row_out_idx = p.row_out_idx;
    if (p.row_out != nullptr) g.tma_store = 0;
    if ((rc = launch_gemm(kEpiScatter, g, s.max_tiles, s.gn2m, c.st, true)) != SPX_OK) return rc;
  }
  if (nv) {
    GemmArgs g = base_args(kEpiScatter, s.bn2m, s.khn / 256, c.status, true, true);
    if ((rc = encode_2d(&g.tma_a, hq, s.P, s.khn / 2, s.khn / 2, kTileRows, 1)) != SPX_OK) return rc;
    if ((rc = encode_3d(&g.tma_b, p.w2_mx, p.groups, s.d, s.khn / 2, s.bn2m, 1)) != SPX_OK) return rc;
    g.groups = p.groups;
    g.max_ctas = p.max_ctas;
    g.tiles = p.tiles_mx;
    g.num_tiles = p.num_tiles_mx;
    g.sfa = hsf;
    g.ld_sfa = s.khn / kNvBlock;
    g.sfb = p.w2_mx_sf;
    g.n_valid = s.d;
    g.out = y;
    g.ldo = s.d;
    g.tma_store = (s.d % 64) == 0;
    if (g.tma_store && (rc = encode_2d(&g.tma_out, y, s.P, s.d, s.d, 32)) != SPX_OK) return rc;
    g.pos_weight = sorted_w;
    g.row_out = p.row_out;
    g.row_out_idx = p.row_out_idx;
    if (p.row_out != nullptr) g.tma_store = 0;
    g.nv_amax_a = nv_amax_h;
    g.nv_amax_b = p.nv_amax_w;
    g.nv_b_stride = 4;
    g.nv_b_off = 2;
    if ((rc = launch_gemm(kEpiScatter, g, s.max_tiles, s.gn2m, c.st, true, true)) != SPX_OK) return rc;
  }
  c.mark(5);
  return SPX_OK;
}

// K3: expert GEMM1 (+SwiGLU) and GEMM2 over the dispatched rows of `hidden`
// (`xa` = hidden padded), both lanes; weighted rows land in Y (sorted order).
int stage_experts(const Ctx& c, const spx_packed_weights* w, const uint16_t* hidden, const uint16_t* xa,
                  const DispatchArgs& da, int64_t ld_hidden = 0, bool x_quantized = false,
                  uint16_t* saved_x = nullptr, uint16_t* saved_gu = nullptr) {
  const bool mx = da.lane_mx != nullptr;
  if (mx && !x_quantized) {
    const int rc = c.s.nv ? stage_quantize_nv_x(c, hidden, ld_hidden, da) : stage_quantize_x(c, hidden, ld_hidden);
    if (rc != SPX_OK) return rc;
  }
  ExpertPass p{w->expert_w1, w->expert_w2, w->expert_w1_mx, w->expert_w1_mx_scales, w->expert_w2_mx,
               w->expert_w2_mx_scales, c.s.E, da.tiles, da.num_tiles, mx ? da.tiles_mx : nullptr,
               mx ? da.num_tiles_mx : nullptr, 0, w->expert_nvfp4_amax};
  p.saved_x = saved_x;
  p.saved_gu = saved_gu;
  return stage_expert_gemms(c, xa, da.src_row, da.sorted_weights, p);
}

// K4 (shared half), first GEMM: shared gate/up with the SwiGLU into the
// workspace's shared hidden rows.
// gu_out (training): the BF16 gate | up pre-activations too, [T, ncs * 2cs]
// in the chunk layout (tcgen05 path at every batch size).
int stage_shared_gemm1(const Ctx& c, const spx_packed_weights* w, const uint16_t* xa, uint16_t* gu_out = nullptr) {
  const Shape& s = c.s;
  int rc = SPX_OK;
  uint16_t* hs = at<uint16_t>(c.ws, c.L.shared_hidden);
  if (s.T <= kGemvMaxTokens && gu_out == nullptr) {  // decode-sized batch: one dense SwiGLU GEMV
    GemvPass g{};
    g.dense_rows = static_cast<int>(s.T);
    g.status = c.status;
    g.d = s.d;
    g.inter = s.S;
    g.kd = s.kd;
    g.chunk = s.cs;
    g.nc = s.ncs;
    g.x = xa;
    g.ldx = s.kd;
    g.w1 = w->shared_w1;
    g.hid = hs;
    g.ldh = s.ksp;
    if (gemv_swiglu_ok(g)) {
      if ((rc = launch_gemv_swiglu(g, c.st)) != SPX_OK) return rc;
      c.mark(6);
      return SPX_OK;
    }
  }
  // Large batches: CTA pairs (256-row tiles; each CTA loads one of the
  // [gate | up] halves of the B tile).
  const bool pair = !s.small && (2 * s.cs) % 32 == 0;
  GemmArgs g = base_args(kEpiSwiglu, 2 * s.cs, s.kd / 64, c.status);
  if (pair) g.stages = gemm_pair_pick_stages(2 * s.cs);
  if ((rc = encode_2d(&g.tma_a, xa, s.T, s.kd, s.kd, kTileRows)) != SPX_OK) return rc;
  if ((rc = encode_3d(&g.tma_b, w->shared_w1, 1, static_cast<int64_t>(s.ncs) * 2 * s.cs, s.kd,
                      pair ? s.cs : 2 * s.cs)) != SPX_OK)
    return rc;
  g.gu_out = gu_out;
  g.ld_gu = static_cast<int64_t>(s.ncs) * 2 * s.cs;
  g.m_rows = static_cast<int>(s.T);
  g.chunk = s.cs;
  g.h_cols = s.ksp;
  g.out = hs;
  g.ldo = s.ksp;
  rc = pair ? launch_gemm_pair(kEpiSwiglu, g, ceil_div(s.T, 2 * kTileRows), s.ncs, c.st)
            : launch_gemm(kEpiSwiglu, g, ceil_div(s.T, kTileRows), s.ncs, c.st);
  if (rc != SPX_OK) return rc;
  c.mark(6);
  return SPX_OK;
}

// K4 (shared half), down projection.  With `y` given, its epilogue also does
// the combine: out = bf16(shared + the token's k expert rows of y), written
// to `out` (the layer update); otherwise `out` receives the shared output.
int stage_shared_gemm2(const Ctx& c, const spx_packed_weights* w, uint16_t* out, const uint16_t* y = nullptr,
                       const int* rank = nullptr, const uint16_t* residual = nullptr,
                       uint16_t* residual_out = nullptr) {
  const Shape& s = c.s;
  int rc = SPX_OK;
  uint16_t* hs = at<uint16_t>(c.ws, c.L.shared_hidden);
  if (y == nullptr && residual == nullptr && s.T <= kGemvMaxTokens) {  // decode-sized batch: dense GEMV
    const GemvPass g = dense_rows_pass(c, hs, s.ksp, s.ksp, s.S, w->shared_w2, s.d, nullptr, out, s.d);
    if (gemv_rows_ok(g)) return launch_gemv_rows(g, c.st);
  }
  const int epi = y != nullptr ? kEpiCombine : kEpiStore;
  GemmArgs g = base_args(epi, s.bn_sd, s.ksp / 64, c.status);
  if ((rc = encode_2d(&g.tma_a, hs, s.T, s.ksp, s.ksp, kTileRows)) != SPX_OK) return rc;
  if ((rc = encode_3d(&g.tma_b, w->shared_w2, 1, s.d, s.ksp, s.bn_sd)) != SPX_OK) return rc;
  g.m_rows = static_cast<int>(s.T);
  g.n_valid = s.d;
  g.out = out;
  g.ldo = s.d;
  g.comb_y = y;
  g.comb_rank = rank;
  g.comb_k = s.k;
  g.ldy = s.d;
  g.comb_res = residual;
  g.comb_res_out = residual_out;
  return launch_gemm(epi, g, ceil_div(s.T, kTileRows), s.gn_sd, c.st);
}

// K4 (shared half): shared SwiGLU of every token, both GEMMs (see
// stage_shared_gemm2 for `y`).
int stage_shared(const Ctx& c, const spx_packed_weights* w, const uint16_t* xa, uint16_t* out,
                 const uint16_t* y = nullptr, const int* rank = nullptr, const uint16_t* residual = nullptr,
                 uint16_t* residual_out = nullptr) {
  if (int rc = stage_shared_gemm1(c, w, xa); rc != SPX_OK) return rc;
  return stage_shared_gemm2(c, w, out, y, rank, residual, residual_out);
}

// The combine can ride on the shared down projection's epilogue.  Not for
// decode-sized batches: there the few epilogue warps would walk their rows'
// expert rows one latency at a time, where the combine kernel spreads them
// over the whole GPU.
bool fused_combine_ok(const Shape& s) {
  return s.S > 0 && s.T > kSmallBatchTokens && s.k <= kCombineMaxK && (s.d % 64) == 0 && (s.bn_sd % 64) == 0;
}

int check_layer_weights(const Shape& s, const spx_layer_dims* dims, const spx_packed_weights* w, bool router,
                        bool experts, bool shared) {
  if (w == nullptr) return SPX_ERR_INVALID_ARG;
  if (router && w->router_weight == nullptr) return SPX_ERR_INVALID_ARG;
  if (router && dims->score_transform == 0 && w->softplus_table == nullptr) return SPX_ERR_INVALID_ARG;
  if (experts && (w->expert_w1 == nullptr || w->expert_w2 == nullptr)) return SPX_ERR_INVALID_ARG;
  if (shared && s.S > 0 && (w->shared_w1 == nullptr || w->shared_w2 == nullptr)) return SPX_ERR_INVALID_ARG;
  if (experts && w->expert_lane_mxfp8 != nullptr) {
    if (!s.mx) return SPX_ERR_INVALID_ARG;  // the workspace has no low-precision regions
    if (w->expert_w1_mx == nullptr || w->expert_w1_mx_scales == nullptr || w->expert_w2_mx == nullptr ||
        w->expert_w2_mx_scales == nullptr)
      return SPX_ERR_INVALID_ARG;
    if (s.nv && w->expert_nvfp4_amax == nullptr) return SPX_ERR_INVALID_ARG;
  }
  return SPX_OK;
}

}  // namespace
}  // namespace spx

using namespace spx;

extern "C" {

int spx_abi_version(void) { return SPX_ABI_VERSION; }

int spx_layer_saved_gu_cols(const spx_layer_dims* dims, int64_t* cols) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (cols == nullptr) return SPX_ERR_INVALID_ARG;
  *cols = static_cast<int64_t>(s.nc) * 2 * s.c;
  return SPX_OK;
}

int spx_layer_saved_shared_gu(const spx_layer_dims* dims, int64_t* cols, int32_t* chunk) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (cols == nullptr || chunk == nullptr) return SPX_ERR_INVALID_ARG;
  *cols = static_cast<int64_t>(s.ncs) * 2 * s.cs;
  *chunk = s.cs;
  return SPX_OK;
}

const char* spx_status_string(int status) {
  switch (status) {
    case SPX_OK:
      return "ok";
    case SPX_ERR_INVALID_ARG:
      return "invalid argument";
    case SPX_ERR_UNSUPPORTED:
      return "unsupported shape or configuration";
    case SPX_ERR_CUDA:
      return "CUDA runtime error";
    case SPX_ERR_DRIVER:
      return "CUDA driver entry point or tensor map error";
    case SPX_ERR_TIMEOUT:
      return "device wait timed out";
    case SPX_ERR_ALIGNMENT:
      return "pointer or stride not 16-byte aligned";
    case SPX_ERR_WORKSPACE:
      return "workspace missing or too small";
    case SPX_ERR_DEVICE:
      return "a kernel reported an error in the workspace status word";
    case SPX_ERR_SCRATCH_LIMIT:
      return "problem exceeds the fixed scratch of spx_dispatch_static "
             "(tokens * top_k <= 1048576, num_experts <= 1024)";
    default:
      return "unknown status";
  }
}

int spx_layer_sizes(const spx_layer_dims* dims, size_t* workspace_bytes, spx_packed_sizes* packed) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (workspace_bytes != nullptr) *workspace_bytes = make_layout(s).total;
  if (packed != nullptr) {
    const MxPackSizes z = mx_pack_sizes(s);
    packed->expert_w1_mx = z.w1;
    packed->expert_w1_mx_scales = z.w1_sf;
    packed->expert_w2_mx = z.w2;
    packed->expert_w2_mx_scales = z.w2_sf;
    packed->expert_nvfp4_amax = s.nv ? static_cast<size_t>(s.E) * 4 * sizeof(float) : 0;
    packed->router_weight = static_cast<size_t>(s.E) * s.kd;
    packed->expert_w1 = static_cast<size_t>(s.E) * s.nc * 2 * s.c * s.kd;
    packed->expert_w2 = static_cast<size_t>(s.E) * s.d * s.kp;
    packed->shared_w1 = s.S > 0 ? static_cast<size_t>(s.ncs) * 2 * s.cs * s.kd : 0;
    packed->shared_w2 = s.S > 0 ? static_cast<size_t>(s.d) * s.ksp : 0;
  }
  return SPX_OK;
}

int spx_softplus_table(uint16_t* table, void* stream) {
  if (table == nullptr) return SPX_ERR_INVALID_ARG;
  return launch_softplus_table(table, static_cast<cudaStream_t>(stream));
}

int spx_pack_weights(const spx_layer_dims* dims, const spx_reference_weights* src, uint16_t* router_weight,
                     uint16_t* expert_w1, uint16_t* expert_w2, uint16_t* shared_w1, uint16_t* shared_w2,
                     void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (src == nullptr || src->router_weight == nullptr || router_weight == nullptr) return SPX_ERR_INVALID_ARG;
  const bool experts = expert_w1 != nullptr || expert_w2 != nullptr;
  if (experts && (expert_w1 == nullptr || expert_w2 == nullptr || src->gate_proj == nullptr ||
                  src->up_proj == nullptr || src->down_proj == nullptr))
    return SPX_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = launch_pad_rows(src->router_weight, s.E, s.d, s.kd, router_weight, st);
  if (rc == SPX_OK && experts)
    rc = launch_pack_chunked_w1(src->gate_proj, src->up_proj, s.E, s.d, s.I, s.kd, s.c, s.nc, 0, expert_w1, st);
  if (rc == SPX_OK && experts) rc = launch_pack_w2(src->down_proj, s.E, s.I, s.d, s.kp, 0, expert_w2, st);
  if (rc == SPX_OK && s.S > 0) {
    if (src->shared_gate == nullptr || src->shared_up == nullptr || src->shared_down == nullptr ||
        shared_w1 == nullptr || shared_w2 == nullptr)
      return SPX_ERR_INVALID_ARG;
    rc = launch_pack_chunked_w1(src->shared_gate, src->shared_up, 1, s.d, s.S, s.kd, s.cs, s.ncs, 1, shared_w1, st);
    if (rc == SPX_OK) rc = launch_pack_w2(src->shared_down, 1, s.S, s.d, s.ksp, 1, shared_w2, st);
  }
  return rc;
}

int spx_pack_weights_mxfp8(const spx_layer_dims* dims, const spx_reference_weights* src, uint8_t* expert_w1_mx,
                           uint8_t* expert_w1_mx_scales, uint8_t* expert_w2_mx, uint8_t* expert_w2_mx_scales,
                           void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (!s.mx || s.nv) return SPX_ERR_INVALID_ARG;
  if (src == nullptr || src->gate_proj == nullptr || src->up_proj == nullptr || src->down_proj == nullptr ||
      expert_w1_mx == nullptr || expert_w1_mx_scales == nullptr || expert_w2_mx == nullptr ||
      expert_w2_mx_scales == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (!aligned16(expert_w1_mx) || !aligned16(expert_w2_mx) || !aligned16(expert_w1_mx_scales) ||
      !aligned16(expert_w2_mx_scales))
    return SPX_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rows1 = s.ncm * 2 * s.cm;
  int rc = launch_mx_quantize_b(kMxSrcW1, src->gate_proj, src->up_proj, s.E, rows1, rows1, s.d, s.kx, 2 * s.cm, s.d,
                                s.I, s.cm, 0, expert_w1_mx, expert_w1_mx_scales, st);
  if (rc == SPX_OK)
    rc = launch_mx_quantize_b(kMxSrcW2, src->down_proj, nullptr, s.E, s.d, s.d, s.I, s.kh, s.bn2m, s.d, s.I, 0, 0,
                              expert_w2_mx, expert_w2_mx_scales, st);
  return rc;
}

int spx_pack_weights_nvfp4(const spx_layer_dims* dims, const spx_reference_weights* src, uint8_t* expert_w1_nv,
                           uint8_t* expert_w1_nv_scales, uint8_t* expert_w2_nv, uint8_t* expert_w2_nv_scales,
                           float* expert_amax, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (!s.nv) return SPX_ERR_INVALID_ARG;
  if (src == nullptr || src->gate_proj == nullptr || src->up_proj == nullptr || src->down_proj == nullptr ||
      expert_w1_nv == nullptr || expert_w1_nv_scales == nullptr || expert_w2_nv == nullptr ||
      expert_w2_nv_scales == nullptr || expert_amax == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (!aligned16(expert_w1_nv) || !aligned16(expert_w2_nv) || !aligned16(expert_w1_nv_scales) ||
      !aligned16(expert_w2_nv_scales) || !aligned16(expert_amax))
    return SPX_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Per-tensor amax of each expert's gate, up and down matrices ([E][4]).
  if (cudaMemsetAsync(expert_amax, 0, sizeof(float) * 4 * s.E, st) != cudaSuccess) return SPX_ERR_CUDA;
  const int64_t per = static_cast<int64_t>(s.d) * s.I;
  int rc = launch_nv_group_amax(src->gate_proj, s.E, per, expert_amax, 4, 0, st);
  if (rc == SPX_OK) rc = launch_nv_group_amax(src->up_proj, s.E, per, expert_amax, 4, 1, st);
  if (rc == SPX_OK) rc = launch_nv_group_amax(src->down_proj, s.E, per, expert_amax, 4, 2, st);
  const int rows1 = s.ncm * 2 * s.cm;
  if (rc == SPX_OK)
    rc = launch_nv_quantize_b(kMxSrcW1, src->gate_proj, src->up_proj, s.E, rows1, rows1, s.d, s.kxn, 2 * s.cm, s.d,
                              s.I, s.cm, 0, expert_amax, expert_w1_nv, expert_w1_nv_scales, st);
  if (rc == SPX_OK)
    rc = launch_nv_quantize_b(kMxSrcW2, src->down_proj, nullptr, s.E, s.d, s.d, s.I, s.khn, s.bn2m, s.d, s.I, 0, 0,
                              expert_amax, expert_w2_nv, expert_w2_nv_scales, st);
  return rc;
}

int spx_mxfp8_quantize_rows(const uint16_t* src, int64_t rows, int32_t cols, uint8_t* values, uint8_t* scales,
                            void* stream) {
  if (rows < 0 || cols <= 0 || cols % kMxBlock != 0) return SPX_ERR_INVALID_ARG;
  if (rows == 0) return SPX_OK;
  if (src == nullptr || values == nullptr || scales == nullptr) return SPX_ERR_INVALID_ARG;
  return launch_mx_quantize_rows(src, rows, cols, cols, cols, values, cols, scales, cols / kMxBlock,
                                 static_cast<cudaStream_t>(stream));
}

namespace {
struct MmLayout {
  int64_t kp;
  int bn;
  size_t status, lq, lsf, rq, rsf, total;
};

MmLayout mm_layout(int64_t m, int64_t n, int64_t k) {
  MmLayout L{};
  L.kp = static_cast<int64_t>(round_up(static_cast<size_t>(k > 0 ? k : 1), 128));
  L.bn = static_cast<int>(std::min<int64_t>(kMxDenseBn, static_cast<int64_t>(round_up(static_cast<size_t>(n), 16))));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = round_up(off + bytes, kAlign);
    return at;
  };
  L.status = take(64);
  L.lq = take(static_cast<size_t>(m) * L.kp);
  L.lsf = take(static_cast<size_t>(m) * (L.kp / kMxBlock));
  L.rq = take(static_cast<size_t>(n) * L.kp);
  L.rsf = take(mx_atoms_bytes(1, static_cast<int>(n), static_cast<int>(L.kp), L.bn));
  L.total = off;
  return L;
}
}  // namespace

size_t spx_mxfp8_mm_workspace(int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0) return 0;
  return mm_layout(m, n, k).total;
}

int spx_mxfp8_mm_nt(const uint16_t* left, const uint16_t* right_rows, int64_t m, int64_t n, int64_t k,
                    uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 0 || n < 0 || k < 0) return SPX_ERR_INVALID_ARG;
  if (m == 0 || n == 0) return SPX_OK;
  if (out == nullptr) return SPX_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k == 0)  // empty contraction: zeros, as the reference's new_zeros
    return cudaMemsetAsync(out, 0, static_cast<size_t>(m) * n * 2, st) == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
  if (left == nullptr || right_rows == nullptr) return SPX_ERR_INVALID_ARG;
  if (m > (int64_t(1) << 31) - 1 || n > (int64_t(1) << 31) - 1 || k > (int64_t(1) << 30)) return SPX_ERR_UNSUPPORTED;
  const MmLayout L = mm_layout(m, n, k);
  if (workspace == nullptr || workspace_bytes < L.total) return SPX_ERR_WORKSPACE;
  if (!aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  uint8_t* lq = at<uint8_t>(workspace, L.lq);
  uint8_t* lsf = at<uint8_t>(workspace, L.lsf);
  uint8_t* rq = at<uint8_t>(workspace, L.rq);
  uint8_t* rsf = at<uint8_t>(workspace, L.rsf);
  const int kp = static_cast<int>(L.kp);
  int rc = launch_mx_quantize_rows(left, m, static_cast<int>(k), k, kp, lq, kp, lsf, kp / kMxBlock, st);
  if (rc == SPX_OK)
    rc = launch_mx_quantize_b(kMxSrcRows, right_rows, nullptr, 1, static_cast<int>(n), static_cast<int>(n),
                              static_cast<int>(k), kp, L.bn, 0, 0, 0, k, rq, rsf, st);
  if (rc != SPX_OK) return rc;
  GemmArgs g = base_args(kEpiStore, L.bn, kp / 128, at<int>(workspace, L.status), true);
  if ((rc = encode_2d(&g.tma_a, lq, m, kp, kp, kTileRows, 1)) != SPX_OK) return rc;
  if ((rc = encode_3d(&g.tma_b, rq, 1, n, kp, L.bn, 1)) != SPX_OK) return rc;
  g.m_rows = static_cast<int>(m);
  g.n_valid = static_cast<int>(n);
  g.out = out;
  g.ldo = n;
  g.sfa = lsf;
  g.ld_sfa = kp / kMxBlock;
  g.sfb = rsf;
  return launch_gemm(kEpiStore, g, ceil_div(m, kTileRows), ceil_div(n, L.bn), st, true);
}

namespace {
struct NvMmLayout {
  int64_t kp;
  int bn;
  size_t status, amax, lq, lsf, rq, rsf, total;
};

NvMmLayout nv_mm_layout(int64_t m, int64_t n, int64_t k) {
  NvMmLayout L{};
  L.kp = static_cast<int64_t>(round_up(static_cast<size_t>(k > 0 ? k : 1), 256));
  L.bn = static_cast<int>(std::min<int64_t>(kMxDenseBn, static_cast<int64_t>(round_up(static_cast<size_t>(n), 16))));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = round_up(off + bytes, kAlign);
    return at;
  };
  L.status = take(64);
  L.amax = take(16);
  L.lq = take(static_cast<size_t>(m) * (L.kp / 2));
  L.lsf = take(static_cast<size_t>(m) * (L.kp / kNvBlock));
  L.rq = take(static_cast<size_t>(n) * (L.kp / 2));
  L.rsf = take(nv_atoms_bytes(1, static_cast<int>(n), static_cast<int>(L.kp), L.bn));
  L.total = off;
  return L;
}
}  // namespace

size_t spx_nvfp4_mm_workspace(int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0) return 0;
  return nv_mm_layout(m, n, k).total;
}

int spx_nvfp4_quantize_rows(const uint16_t* src, int64_t rows, int32_t cols, uint8_t* values, uint8_t* scales,
                            float* amax, void* stream) {
  if (rows < 0 || cols < 1) return SPX_ERR_INVALID_ARG;
  if (rows == 0) return SPX_OK;
  if (src == nullptr || values == nullptr || scales == nullptr || amax == nullptr) return SPX_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(values) & 7u) != 0) return SPX_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int kp = round_up_i(cols, 256);
  if (cudaMemsetAsync(amax, 0, sizeof(float), st) != cudaSuccess) return SPX_ERR_CUDA;
  int rc = launch_nv_amax(src, rows, cols, cols, amax, st);
  if (rc == SPX_OK) rc = launch_nv_quantize_rows(src, rows, cols, cols, amax, kp, values, scales, st);
  return rc;
}

int spx_nvfp4_mm_nt(const uint16_t* left, const uint16_t* right_rows, int64_t m, int64_t n, int64_t k,
                    uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 0 || n < 0 || k < 0) return SPX_ERR_INVALID_ARG;
  if (m == 0 || n == 0) return SPX_OK;
  if (out == nullptr) return SPX_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k == 0)
    return cudaMemsetAsync(out, 0, static_cast<size_t>(m) * n * 2, st) == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
  if (left == nullptr || right_rows == nullptr) return SPX_ERR_INVALID_ARG;
  if (m > (int64_t(1) << 31) - 1 || n > (int64_t(1) << 31) - 1 || k > (int64_t(1) << 30)) return SPX_ERR_UNSUPPORTED;
  const NvMmLayout L = nv_mm_layout(m, n, k);
  if (workspace == nullptr || workspace_bytes < L.total) return SPX_ERR_WORKSPACE;
  if (!aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  float* amax = at<float>(workspace, L.amax);
  uint8_t* lq = at<uint8_t>(workspace, L.lq);
  uint8_t* lsf = at<uint8_t>(workspace, L.lsf);
  uint8_t* rq = at<uint8_t>(workspace, L.rq);
  uint8_t* rsf = at<uint8_t>(workspace, L.rsf);
  const int kp = static_cast<int>(L.kp);
  if (cudaMemsetAsync(amax, 0, 2 * sizeof(float), st) != cudaSuccess) return SPX_ERR_CUDA;
  int rc = launch_nv_amax(left, m, static_cast<int>(k), k, amax, st);
  if (rc == SPX_OK) rc = launch_nv_amax(right_rows, n, static_cast<int>(k), k, amax + 1, st);
  if (rc == SPX_OK) rc = launch_nv_quantize_rows(left, m, static_cast<int>(k), k, amax, kp, lq, lsf, st);
  if (rc == SPX_OK)
    rc = launch_nv_quantize_b(kMxSrcRows, right_rows, nullptr, 1, static_cast<int>(n), static_cast<int>(n),
                              static_cast<int>(k), kp, L.bn, 0, 0, 0, k, amax + 1, rq, rsf, st);
  if (rc != SPX_OK) return rc;
  GemmArgs g = base_args(kEpiStore, L.bn, kp / 256, at<int>(workspace, L.status), true, true);
  if ((rc = encode_2d(&g.tma_a, lq, m, kp / 2, kp / 2, kTileRows, 1)) != SPX_OK) return rc;
  if ((rc = encode_3d(&g.tma_b, rq, 1, n, kp / 2, L.bn, 1)) != SPX_OK) return rc;
  g.m_rows = static_cast<int>(m);
  g.n_valid = static_cast<int>(n);
  g.out = out;
  g.ldo = n;
  g.sfa = lsf;
  g.ld_sfa = kp / kNvBlock;
  g.sfb = rsf;
  g.nv_amax_a = amax;
  g.nv_amax_b = amax + 1;
  g.nv_b_stride = 4;
  g.nv_b_off = 0;
  return launch_gemm(kEpiStore, g, ceil_div(m, kTileRows), ceil_div(n, L.bn), st, true, true);
}

int spx_route(const spx_layer_dims* dims, const uint16_t* logits, const uint16_t* softplus_table,
              const uint8_t* resident_mask, uint16_t* router_scores, int64_t* expert_ids, uint16_t* routing_weights,
              void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (logits == nullptr || router_scores == nullptr || expert_ids == nullptr || routing_weights == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (dims->score_transform == 0 && softplus_table == nullptr) return SPX_ERR_INVALID_ARG;
  const Layout L = make_layout(s);
  return run_route(s, logits, dims->score_transform == 0 ? softplus_table : nullptr, resident_mask, router_scores,
                   expert_ids, routing_weights, workspace, L, static_cast<cudaStream_t>(stream));
}

int spx_router_sizes(const spx_layer_dims* dims, size_t* workspace_bytes) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (workspace_bytes == nullptr) return SPX_ERR_INVALID_ARG;
  *workspace_bytes = kAlign + (s.kd != s.d ? round_up(2 * static_cast<size_t>(s.T) * s.kd, kAlign) : 0);
  return SPX_OK;
}

int spx_router_forward(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* hidden,
                       uint16_t* router_scores, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (hidden == nullptr || router_scores == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (int rc = check_layer_weights(s, dims, w, true, false, false); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(router_scores) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  // Workspace: the status word, then the K-padded hidden rows when d % 64 != 0.
  Layout L{};
  L.small = 0;
  L.x_pad = kAlign;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Ctx c{s, L, workspace, st, at<int>(workspace, L.small), nullptr};
  const uint16_t* xa = nullptr;
  if (int rc = stage_pad(c, hidden, &xa); rc != SPX_OK) return rc;
  if (int rc = stage_router(c, w, xa, router_scores); rc != SPX_OK) return rc;
  if (dims->score_transform != 0) return SPX_OK;  // identity: the logits are the scores
  return launch_scores_from_logits(router_scores, s.T * s.E, w->softplus_table, st);
}

int spx_dispatch(const spx_layer_dims* dims, const int64_t* expert_ids, int32_t* order, int32_t* counts,
                 void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (expert_ids == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  const Layout L = make_layout(s);
  DispatchArgs a = dispatch_args(s, expert_ids, order, counts, workspace, L);
  a.lb_blocks = 0;  // no routing probabilities here: skip the auxiliary loss
  a.execution_loop = dims->execution_loop;
  return launch_dispatch(a, static_cast<cudaStream_t>(stream));
}

int spx_layer_forward(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* hidden,
                      const spx_layer_outputs* out, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (out == nullptr || hidden == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (out->update == nullptr || out->router_scores == nullptr || out->expert_ids == nullptr ||
      out->routing_weights == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (int rc = check_layer_weights(s, dims, w, true, true, true); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(out->update) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  if ((out->saved_x != nullptr) != (out->saved_gu != nullptr)) return SPX_ERR_INVALID_ARG;
  if (out->saved_x != nullptr) {  // training activations: BF16 experts, d_model % 64 == 0
    if (s.mx || s.kd != s.d) return SPX_ERR_UNSUPPORTED;
    if (!aligned16(out->saved_x) || !aligned16(out->saved_gu)) return SPX_ERR_ALIGNMENT;
  }
  if (out->saved_shared_gu != nullptr && (s.S <= 0 || !aligned16(out->saved_shared_gu))) return SPX_ERR_INVALID_ARG;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), out->stage_events};
  int rc = SPX_OK;
  c.mark(0);
  const uint16_t* xa = nullptr;
  if ((rc = stage_pad(c, hidden, &xa)) != SPX_OK) return rc;
  // ---- side stream: work that needs only the hidden rows runs beside the
  // router, selection and dispatch.  Large batches: the MXFP8 quantisation of
  // the rows (joined before the experts).  Decode-sized batches: the whole
  // shared SwiGLU (two dense GEMVs, joined before the combine) -- route and
  // dispatch occupy a handful of SMs there; forking their 3 us quantisation as
  // well measured no faster.
  const bool fork_mx = s.mx && !s.nv && !s.small && w->expert_lane_mxfp8 != nullptr;
  // (only while the shared projections are dense GEMVs: no tcgen05 kernel,
  // which would want the tensor memory the main stream's kernels hold)
  const bool fork_shared = s.small && s.S > 0 && !fused_combine_ok(s) && s.T <= kGemvMaxTokens &&
                           out->saved_shared_gu == nullptr;
  SideStream ss{};
  const bool forked = (fork_mx || fork_shared) && side_stream(c.st, &ss);
  uint16_t* so = s.S > 0 ? at<uint16_t>(workspace, L.shared_out) : nullptr;
  if (forked) {
    if (cudaEventRecord(ss.fork, c.st) != cudaSuccess || cudaStreamWaitEvent(ss.side, ss.fork, 0) != cudaSuccess)
      return SPX_ERR_CUDA;
    const Ctx cs{s, L, workspace, ss.side, c.status, nullptr};
    if (fork_mx && (rc = stage_quantize_x(cs, hidden, 0)) != SPX_OK) return rc;
    if (cudaEventRecord(ss.join, ss.side) != cudaSuccess) return SPX_ERR_CUDA;  // before the experts
    if (fork_shared) {
      if ((rc = stage_shared_gemm1(cs, w, xa)) != SPX_OK || (rc = stage_shared_gemm2(cs, w, so)) != SPX_OK) return rc;
      if (cudaEventRecord(ss.join2, ss.side) != cudaSuccess) return SPX_ERR_CUDA;  // before the combine
    }
  }
  // ---- K1: router GEMM (unless logits are injected), scores, top-k, weights,
  // load-balance partials
  if ((rc = stage_router_route(c, dims, w, xa, out)) != SPX_OK) return rc;
  c.mark(2);
  // ---- K2: dispatch + statistics
  const DispatchArgs da = layer_dispatch_args(c, dims, w, out);
  if ((rc = launch_dispatch(da, c.st)) != SPX_OK) return rc;
  c.mark(3);
  // ---- K3: grouped experts (both lanes)
  if (fork_mx && forked && cudaStreamWaitEvent(c.st, ss.join, 0) != cudaSuccess) return SPX_ERR_CUDA;
  if ((rc = stage_experts(c, w, hidden, xa, da, 0, fork_mx && forked, out->saved_x, out->saved_gu)) != SPX_OK)
    return rc;
  // ---- K4: shared SwiGLU, then update = shared + the token's k weighted expert rows
  uint16_t* y = at<uint16_t>(workspace, L.y);
  if (fused_combine_ok(s)) {
    if ((rc = stage_shared_gemm1(c, w, xa, out->saved_shared_gu)) != SPX_OK) return rc;
    if ((rc = stage_shared_gemm2(c, w, out->update, y, da.rank)) != SPX_OK) return rc;
  } else {
    if (fork_shared && forked) {
      if (cudaStreamWaitEvent(c.st, ss.join2, 0) != cudaSuccess) return SPX_ERR_CUDA;
      c.mark(6);
    } else if (s.S > 0) {
      if ((rc = stage_shared_gemm1(c, w, xa, out->saved_shared_gu)) != SPX_OK) return rc;
      if ((rc = stage_shared_gemm2(c, w, so)) != SPX_OK) return rc;
    } else {
      c.mark(6);
    }
    if ((rc = launch_combine(y, da.rank, nullptr, so, s.T, s.d, s.k, out->update, c.st)) != SPX_OK) return rc;
  }
  c.mark(7);
  return SPX_OK;
}

int spx_block_channel_forward(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* norm_weight,
                              float eps, const uint16_t* hidden, const spx_layer_outputs* out, uint16_t* hidden_out,
                              void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (out == nullptr || hidden == nullptr || hidden_out == nullptr || norm_weight == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (out->router_scores == nullptr || out->expert_ids == nullptr || out->routing_weights == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (out->injected_logits != nullptr) return SPX_ERR_INVALID_ARG;  // the logits come from the normalised rows
  if (int rc = check_layer_weights(s, dims, w, true, true, true); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(hidden_out) || !aligned16(norm_weight) || !aligned16(workspace) ||
      (out->update != nullptr && !aligned16(out->update)))
    return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), out->stage_events};
  int rc = SPX_OK;
  c.mark(0);
  // ---- channel_norm(h): the normalised rows, K-padded, feed every GEMM and the MXFP8 quantiser
  uint16_t* xn = at<uint16_t>(workspace, L.x_norm);
  if ((rc = launch_rmsnorm_rows(hidden, norm_weight, eps, s.T, s.d, xn, s.kd, c.st)) != SPX_OK) return rc;
  if ((rc = stage_router_route(c, dims, w, xn, out)) != SPX_OK) return rc;
  c.mark(2);
  const DispatchArgs da = layer_dispatch_args(c, dims, w, out);
  if ((rc = launch_dispatch(da, c.st)) != SPX_OK) return rc;
  c.mark(3);
  if ((rc = stage_experts(c, w, xn, xn, da, s.kd)) != SPX_OK) return rc;
  // ---- update and the residual add h + update in the combine
  uint16_t* y = at<uint16_t>(workspace, L.y);
  if (fused_combine_ok(s)) {
    if ((rc = stage_shared(c, w, xn, out->update, y, da.rank, hidden, hidden_out)) != SPX_OK) return rc;
  } else {
    uint16_t* so = nullptr;
    if (s.S > 0) {
      so = at<uint16_t>(workspace, L.shared_out);
      if ((rc = stage_shared(c, w, xn, so)) != SPX_OK) return rc;
    } else {
      c.mark(6);
    }
    if ((rc = launch_combine_residual(y, da.rank, nullptr, so, hidden, s.T, s.d, s.k, out->update, hidden_out,
                                      c.st)) != SPX_OK)
      return rc;
  }
  c.mark(7);
  return SPX_OK;
}

int spx_expert_quant_error(const spx_layer_dims* dims, const spx_reference_weights* src, int32_t weight_format,
                           float* expert_error, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (src == nullptr || src->gate_proj == nullptr || src->up_proj == nullptr || src->down_proj == nullptr ||
      expert_error == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (weight_format != 1 && weight_format != 2) return SPX_ERR_INVALID_ARG;
  return launch_expert_quant_error(src->gate_proj, src->up_proj, src->down_proj, s.E, s.d, s.I, weight_format,
                                   expert_error, static_cast<cudaStream_t>(stream));
}

int spx_rmsnorm_rows(const uint16_t* hidden, const uint16_t* norm_weight, float eps, int64_t rows, int32_t d,
                     uint16_t* out, int32_t ld_out, void* stream) {
  if (rows < 0 || d <= 0) return SPX_ERR_INVALID_ARG;
  if (rows > 0 && (hidden == nullptr || norm_weight == nullptr || out == nullptr)) return SPX_ERR_INVALID_ARG;
  return launch_rmsnorm_rows(hidden, norm_weight, eps, rows, d, out, ld_out, static_cast<cudaStream_t>(stream));
}

int spx_layer_route(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* hidden,
                    const spx_layer_outputs* out, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (out == nullptr || hidden == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (out->router_scores == nullptr || out->expert_ids == nullptr || out->routing_weights == nullptr ||
      out->dispatch_order == nullptr || out->expert_counts == nullptr || out->pair_rank == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (int rc = check_layer_weights(s, dims, w, true, false, false); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), nullptr};
  int rc = SPX_OK;
  const uint16_t* xa = nullptr;
  if ((rc = stage_pad(c, hidden, &xa)) != SPX_OK) return rc;
  if ((rc = stage_router_route(c, dims, w, xa, out)) != SPX_OK) return rc;
  DispatchArgs da = layer_dispatch_args(c, dims, w, out);
  da.lane_mx = nullptr;  // the experts run elsewhere
  return launch_dispatch(da, c.st);
}

// ---------------------------------------------------------------- paged experts
// The layer forward in three calls around a device cache of expert weights
// (experts/bank.py:821-899 with offload.py): begin (router, dispatch, the
// MXFP8 quantisation of the hidden rows, shared GEMM1), one experts call per
// page, finish (shared down projection + combine).

int spx_layer_paged_begin(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* hidden,
                          const spx_layer_outputs* out, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (out == nullptr || hidden == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (out->router_scores == nullptr || out->expert_ids == nullptr || out->routing_weights == nullptr ||
      out->expert_counts == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (int rc = check_layer_weights(s, dims, w, true, false, true); rc != SPX_OK) return rc;
  if (w->expert_lane_mxfp8 != nullptr && !s.mx) return SPX_ERR_INVALID_ARG;
  if (!aligned16(hidden) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), out->stage_events};
  int rc = SPX_OK;
  c.mark(0);
  const uint16_t* xa = nullptr;
  if ((rc = stage_pad(c, hidden, &xa)) != SPX_OK) return rc;
  if ((rc = stage_router_route(c, dims, w, xa, out)) != SPX_OK) return rc;
  c.mark(2);
  const DispatchArgs da = layer_dispatch_args(c, dims, w, out);
  if ((rc = launch_dispatch(da, c.st)) != SPX_OK) return rc;
  c.mark(3);
  if (da.lane_mx != nullptr &&
      (rc = s.nv ? stage_quantize_nv_x(c, hidden, 0, da) : stage_quantize_x(c, hidden, 0)) != SPX_OK)
    return rc;
  if (s.S > 0 && (rc = stage_shared_gemm1(c, w, xa)) != SPX_OK) return rc;
  return SPX_OK;
}

int spx_layer_paged_experts(const spx_layer_dims* dims, const spx_packed_weights* cache, int32_t cache_slots,
                            const int32_t* page_slot, int32_t sm_limit, const uint16_t* hidden, void* workspace,
                            void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (cache == nullptr || page_slot == nullptr || hidden == nullptr || cache_slots < 1 || sm_limit < 0)
    return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (int rc = check_layer_weights(s, dims, cache, false, true, false); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), nullptr};
  const bool mx = s.mx && cache->expert_lane_mxfp8 != nullptr;
  int* small = at<int>(workspace, L.small);
  PageTilesArgs pt{};
  pt.tiles = at<int4>(workspace, L.tiles);
  pt.num_tiles = small + 2;
  pt.tiles_mx = mx ? at<int4>(workspace, L.tiles_mx) : nullptr;
  pt.num_tiles_mx = mx ? small + 3 : nullptr;
  pt.page_slot = page_slot;
  pt.num_experts = s.E;
  pt.out = at<int4>(workspace, L.tiles_page);
  pt.out_count = small + 4;
  pt.out_mx = mx ? at<int4>(workspace, L.tiles_mx_page) : nullptr;
  pt.out_count_mx = mx ? small + 5 : nullptr;
  if (int rc = launch_page_tiles(pt, c.st); rc != SPX_OK) return rc;
  const uint16_t* xa = s.kd != s.d ? at<uint16_t>(workspace, L.x_pad) : hidden;
  const ExpertPass p{cache->expert_w1, cache->expert_w2, cache->expert_w1_mx, cache->expert_w1_mx_scales,
                     cache->expert_w2_mx, cache->expert_w2_mx_scales, cache_slots, pt.out, pt.out_count,
                     pt.out_mx, pt.out_count_mx, sm_limit, cache->expert_nvfp4_amax};
  return stage_expert_gemms(c, xa, at<int>(workspace, L.src_row), at<uint16_t>(workspace, L.sorted_w), p);
}

int spx_layer_paged_finish(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* hidden,
                           const spx_layer_outputs* out, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (out == nullptr || hidden == nullptr || out->update == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (int rc = check_layer_weights(s, dims, w, false, false, true); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(out->update) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), out->stage_events};
  int rc = SPX_OK;
  uint16_t* y = at<uint16_t>(workspace, L.y);
  const int* rank = out->pair_rank != nullptr ? out->pair_rank : at<int>(workspace, L.rank);
  if (fused_combine_ok(s)) {
    if ((rc = stage_shared_gemm2(c, w, out->update, y, rank)) != SPX_OK) return rc;
  } else {
    uint16_t* so = nullptr;
    if (s.S > 0) {
      so = at<uint16_t>(workspace, L.shared_out);
      if ((rc = stage_shared_gemm2(c, w, so)) != SPX_OK) return rc;
    }
    if ((rc = launch_combine(y, rank, nullptr, so, s.T, s.d, s.k, out->update, c.st)) != SPX_OK) return rc;
  }
  c.mark(7);
  return SPX_OK;
}

int spx_stage_expert_slots(const void* const* src, void* const* dst, const int64_t* bytes, int32_t arrays,
                           const int32_t* pairs, int32_t n, int32_t num_experts, int32_t slots, int32_t ctas,
                           void* stream) {
  if (src == nullptr || dst == nullptr || bytes == nullptr || arrays < 1 || arrays > kStageMaxArrays || n < 0)
    return SPX_ERR_INVALID_ARG;
  StageSlotsArgs a{};
  for (int i = 0; i < arrays; ++i) {
    a.src[i] = static_cast<const uint8_t*>(src[i]);
    a.dst[i] = static_cast<uint8_t*>(dst[i]);
    a.bytes[i] = bytes[i];
  }
  a.arrays = arrays;
  a.pairs = pairs;
  a.num_pairs = n;
  a.num_experts = num_experts;
  a.slots = slots;
  a.ctas = ctas;
  return launch_stage_slots(a, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- peer exchange
int spx_ipc_buffer_alloc(size_t bytes, void** device_ptr, uint8_t* handle) {
  if (bytes == 0 || device_ptr == nullptr || handle == nullptr) return SPX_ERR_INVALID_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return SPX_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return SPX_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  *device_ptr = p;
  return SPX_OK;
}

int spx_ipc_buffer_open(const uint8_t* handle, void** peer_ptr) {
  if (handle == nullptr || peer_ptr == nullptr) return SPX_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return SPX_ERR_CUDA;
  }
  *peer_ptr = p;
  return SPX_OK;
}

int spx_ipc_buffer_close(void* peer_ptr) {
  if (peer_ptr == nullptr) return SPX_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(peer_ptr) == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int spx_ipc_buffer_free(void* device_ptr) {
  if (device_ptr == nullptr) return SPX_ERR_INVALID_ARG;
  return cudaFree(device_ptr) == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int spx_rows_to_peers(const uint16_t* src, int64_t ld_src, const int32_t* index, int32_t index_div, int64_t rows,
                      int32_t d, const int64_t* seg_offsets, void* const* dst_ptrs, const int64_t* dst_row_offsets,
                      int64_t ld_dst, int32_t groups, void* stream) {
  if (rows < 0 || d < 1 || index_div < 1 || groups < 1 || ld_src < d || ld_dst < d) return SPX_ERR_INVALID_ARG;
  if (rows == 0) return SPX_OK;
  if (src == nullptr || seg_offsets == nullptr || dst_ptrs == nullptr || dst_row_offsets == nullptr)
    return SPX_ERR_INVALID_ARG;
  return launch_rows_to_peers(src, ld_src, index, index_div, rows, d, seg_offsets,
                              reinterpret_cast<uint16_t* const*>(dst_ptrs), dst_row_offsets, ld_dst, groups,
                              static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- backward
}  // extern "C"

namespace spx {
namespace {

// Backward workspace: the forward's layout (dispatch scratch, sorted weights,
// ranks, tile table; y holds the sorted input-gradient rows) and then:
struct BwdLayout {
  size_t gu;      // [P, nc * 2c] recomputed gate | up pre-activations (chunk layout)
  size_t dhp;     // [P, ldh]     bf16(dY_t @ D_e^T)
  size_t logits;  // [T, E]       recomputed router logits (softplus scores only)
  size_t dw;      // [P] float    routing-weight gradients in pair order
  size_t total;
};

int bwd_ldh(const Shape& s) { return round_up_i(s.I, 16); }
int bwd_ki(const Shape& s) { return round_up_i(s.I, 64); }

BwdLayout make_bwd_layout(const Shape& s, size_t base) {
  BwdLayout B{};
  size_t off = round_up(base, kAlign);
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = round_up(off + bytes, kAlign);
    return at;
  };
  B.gu = take(2 * static_cast<size_t>(s.P) * s.nc * 2 * s.c);
  B.dhp = take(2 * static_cast<size_t>(s.P) * bwd_ldh(s));
  B.logits = take(2 * static_cast<size_t>(s.T) * s.E);
  B.dw = take(sizeof(float) * static_cast<size_t>(s.P));
  B.total = off;
  return B;
}

}  // namespace
}  // namespace spx

extern "C" {

int spx_layer_backward_sizes(const spx_layer_dims* dims, size_t* workspace_bytes) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (workspace_bytes == nullptr) return SPX_ERR_INVALID_ARG;
  *workspace_bytes = make_bwd_layout(s, make_layout(s).total).total;
  return SPX_OK;
}

int spx_layer_backward(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* hidden,
                       const spx_layer_grads* gr, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (gr == nullptr || hidden == nullptr || w == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (s.mx || w->expert_lane_mxfp8 != nullptr) return SPX_ERR_UNSUPPORTED;  // BF16 experts only
  if (s.kd != s.d) return SPX_ERR_UNSUPPORTED;                              // d_model % 64 == 0
  if (gr->expert_ids == nullptr || gr->routing_weights == nullptr || gr->router_scores == nullptr ||
      gr->gate_proj == nullptr || gr->up_proj == nullptr || gr->down_proj == nullptr || gr->d_update == nullptr ||
      gr->d_hidden_experts == nullptr || gr->d_logits == nullptr || gr->h_sorted == nullptr ||
      gr->dgu_sorted == nullptr || gr->expert_counts == nullptr)
    return SPX_ERR_INVALID_ARG;
  const int wgrad_outs = (gr->d_gate_proj != nullptr) + (gr->d_up_proj != nullptr) + (gr->d_down_proj != nullptr);
  if (wgrad_outs != 0 && wgrad_outs != 3) return SPX_ERR_INVALID_ARG;
  const bool wgrad = wgrad_outs == 3;
  // x_sorted / du_sorted: both or neither; neither only with the weight
  // gradients, which then gather their rows themselves.
  const bool sorted_rows = gr->x_sorted != nullptr;
  if (sorted_rows != (gr->du_sorted != nullptr) || (!sorted_rows && !wgrad)) return SPX_ERR_INVALID_ARG;
  if (gr->saved_gu != nullptr && (!sorted_rows || !aligned16(gr->saved_gu))) return SPX_ERR_INVALID_ARG;
  if ((gr->forward_workspace != nullptr) != (gr->expert_utilization != nullptr) ||
      (gr->forward_workspace != nullptr && !aligned16(gr->forward_workspace)))
    return SPX_ERR_INVALID_ARG;
  if (wgrad && s.I % 8 != 0) return SPX_ERR_UNSUPPORTED;
  if (wgrad && (!aligned16(gr->h_sorted) || !aligned16(gr->d_gate_proj) || !aligned16(gr->d_up_proj) ||
                !aligned16(gr->d_down_proj)))
    return SPX_ERR_ALIGNMENT;
  if (int rc = check_layer_weights(s, dims, w, true, true, false); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(gr->d_update) || !aligned16(workspace) || !aligned16(gr->dgu_sorted) ||
      (sorted_rows && (!aligned16(gr->x_sorted) || !aligned16(gr->du_sorted))) || !aligned16(gr->d_hidden_experts) ||
      !aligned16(gr->gate_proj) || !aligned16(gr->up_proj) || !aligned16(gr->down_proj))
    return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const BwdLayout B = make_bwd_layout(s, L.total);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), nullptr};
  const cudaStream_t st = c.st;
  int rc = SPX_OK;
  const int ki = bwd_ki(s), ldh = bwd_ldh(s);
  // [P, nc * 2c] gate | up pre-activations: the forward's (saved_gu) or recomputed here
  const uint16_t* gu = gr->saved_gu != nullptr ? gr->saved_gu : at<uint16_t>(workspace, B.gu);
  uint16_t* dhp = at<uint16_t>(workspace, B.dhp);
  float* dw = at<float>(workspace, B.dw);
  uint16_t* dxs = at<uint16_t>(workspace, L.y);

  // ---- router logits: the forward's (router_logits) or again here
  const bool softplus = dims->score_transform == 0;
  const uint16_t* logits = nullptr;
  if (softplus) {
    if (gr->router_logits != nullptr) {
      logits = gr->router_logits;
    } else {
      uint16_t* lg = at<uint16_t>(workspace, B.logits);
      if ((rc = stage_router(c, w, hidden, lg)) != SPX_OK) return rc;
      logits = lg;
    }
  }

  // ---- the forward's dispatch, read from its workspace (the same layout L),
  // or dispatch again from the forward's expert ids (all experts in the BF16 table)
  DispatchArgs da{};
  if (gr->forward_workspace != nullptr) {
    void* fw = const_cast<void*>(gr->forward_workspace);
    da = dispatch_args(s, gr->expert_ids, nullptr, nullptr, fw, L);
    da.status = c.status;
    da.sorted_weights = at<uint16_t>(fw, L.sorted_w);
    da.utilization = const_cast<float*>(gr->expert_utilization);
    if (cudaMemcpyAsync(gr->expert_counts, da.counts, static_cast<size_t>(s.E) * 4, cudaMemcpyDeviceToDevice, st) !=
        cudaSuccess)
      return SPX_ERR_CUDA;
  } else {
    da = dispatch_args(s, gr->expert_ids, nullptr, gr->expert_counts, workspace, L);
    da.lb_blocks = 0;
    da.pair_weights = gr->routing_weights;
    da.sorted_weights = at<uint16_t>(workspace, L.sorted_w);
    da.utilization = at<float>(workspace, L.util);
    da.resident = w->resident_mask;
    if ((rc = launch_dispatch(da, st)) != SPX_OK) return rc;
  }

  // ---- gate | up pre-activations again: GEMM1 (gathered rows) with a plain
  // epilogue, unless the forward saved them (and the rows: x_sorted)
  if (gr->saved_gu == nullptr) {
    GemmArgs g = base_args(kEpiStore, 2 * s.c, s.kd / 64, c.status);
    if ((rc = encode_3d(&g.tma_b, w->expert_w1, s.E, static_cast<int64_t>(s.nc) * 2 * s.c, s.kd, 2 * s.c)) != SPX_OK)
      return rc;
    g.groups = s.E;
    g.gather = 1;
    g.gather_idx = da.src_row;
    g.a_base = reinterpret_cast<const uint8_t*>(hidden);
    g.lda = 2 * static_cast<int64_t>(s.kd);
    g.tiles = da.tiles;
    g.num_tiles = da.num_tiles;
    g.n_valid = s.nc * 2 * s.c;
    g.out = at<uint16_t>(workspace, B.gu);
    g.ldo = s.nc * 2 * s.c;
    g.copy_out = gr->x_sorted;  // the gathered x rows, kept in dispatch order (or not at all)
    g.ld_copy = s.d;
    if (g.copy_out != nullptr && (rc = encode_2d(&g.tma_copy, g.copy_out, s.P, s.d, s.d, 32)) != SPX_OK) return rc;
    if ((rc = launch_gemm(kEpiStore, g, s.max_tiles, s.nc, st)) != SPX_OK) return rc;
  }
  // ---- dh' = dU_t @ D_e^T (gathered rows of the upstream gradient)
  {
    const int bn = std::min(256, ldh);
    GemmArgs g = base_args(kEpiStore, bn, s.kd / 64, c.status);
    if ((rc = encode_3d(&g.tma_b, gr->down_proj, s.E, s.I, s.d, bn)) != SPX_OK) return rc;
    g.groups = s.E;
    g.gather = 1;
    g.gather_idx = da.src_row;
    g.a_base = reinterpret_cast<const uint8_t*>(gr->d_update);
    g.lda = 2 * static_cast<int64_t>(s.d);
    g.tiles = da.tiles;
    g.num_tiles = da.num_tiles;
    g.n_valid = s.I;
    g.out = dhp;
    g.ldo = ldh;
    g.copy_out = gr->du_sorted;  // the gathered dU rows, kept in dispatch order (or not at all)
    g.ld_copy = s.d;
    if (g.copy_out != nullptr && (rc = encode_2d(&g.tma_copy, g.copy_out, s.P, s.d, s.d, 32)) != SPX_OK) return rc;
    if ((rc = launch_gemm(kEpiStore, g, s.max_tiles, ceil_div(s.I, bn), st)) != SPX_OK) return rc;
  }
  // ---- SwiGLU backward: h, [d gate | d up], routing-weight gradients
  if ((rc = launch_bwd_swiglu(gu, s.nc * 2 * s.c, s.c, dhp, ldh, da.sorted_weights, da.order, s.P, s.I, ki,
                              gr->h_sorted, gr->dgu_sorted, dw, st)) != SPX_OK)
    return rc;
  // ---- input gradient of the experts: dx_p = [d gate | d up] @ [G_e | U_e]^T, then per token.
  // The rows leave through the row epilogue (unweighted: bf16(acc)), which
  // sends whole 32-row boxes by TMA stores as the forward's GEMM2 does.
  {
    GemmArgs g = base_args(kEpiScatter, s.bn_d, 2 * ki / 64, c.status);
    if ((rc = encode_2d(&g.tma_a, gr->dgu_sorted, s.P, 2 * ki, 2 * ki, kTileRows)) != SPX_OK) return rc;
    // B = [G_e | U_e] along K straight from the reference-layout [E, d, I]
    // matrices: K blocks below kI from gate (zero past I), the rest from up
    if ((rc = encode_3d(&g.tma_b, gr->gate_proj, s.E, s.d, s.I, s.bn_d)) != SPX_OK) return rc;
    if ((rc = encode_3d(&g.tma_b2, gr->up_proj, s.E, s.d, s.I, s.bn_d)) != SPX_OK) return rc;
    g.b_split = ki / 64;
    g.groups = s.E;
    g.tiles = da.tiles;
    g.num_tiles = da.num_tiles;
    g.n_valid = s.d;
    g.out = dxs;
    g.ldo = s.d;
    g.tma_store = (s.d % 64) == 0;  // whole 64-column boxes; other widths use plain stores
    if (g.tma_store && (rc = encode_2d(&g.tma_out, dxs, s.P, s.d, s.d, 32)) != SPX_OK) return rc;
    if ((rc = launch_gemm(kEpiScatter, g, s.max_tiles, s.gn_d, st)) != SPX_OK) return rc;
  }
  if ((rc = launch_combine(dxs, da.rank, nullptr, nullptr, s.T, s.d, s.k, gr->d_hidden_experts, st)) != SPX_OK)
    return rc;
  // ---- the experts' weight gradients over the sorted rows (tcgen05, MN-major
  // operands); without sorted copies the x rows and the dU rows are gathered
  // by token inside the kernels
  if (wgrad) {
    WgradOperand xo{}, dguo{}, ho{}, dyo{};
    xo.ld = xo.total = s.d;
    if (sorted_rows) {
      xo.rows = gr->x_sorted;
    } else {
      xo.src = hidden;
      xo.index = da.src_row;
      xo.src_rows = s.T;
    }
    dguo.rows = gr->dgu_sorted;
    dguo.ld = dguo.total = 2 * ki;
    if ((rc = launch_wgrad(xo, dguo, s.P, gr->expert_counts, s.E, gr->d_gate_proj, s.I, s.I, gr->d_up_proj, s.I, ki,
                           s.I, c.status, st)) != SPX_OK)
      return rc;
    ho.rows = gr->h_sorted;
    ho.ld = ho.total = s.I;
    dyo.ld = dyo.total = s.d;
    if (sorted_rows) {
      dyo.rows = gr->du_sorted;
    } else {
      dyo.src = gr->d_update;
      dyo.index = da.src_row;
      dyo.src_rows = s.T;
    }
    if ((rc = launch_wgrad(ho, dyo, s.P, gr->expert_counts, s.E, gr->d_down_proj, s.d, s.d, nullptr, 0, 0, 0,
                           c.status, st)) != SPX_OK)
      return rc;
  }
  // ---- router: selection and load-balance softmaxes, softplus
  BwdRouterArgs ra{};
  ra.scores = gr->router_scores;
  ra.logits = logits;
  ra.ids = gr->expert_ids;
  ra.weights = gr->routing_weights;
  ra.dw = dw;
  ra.fractions = da.utilization;
  ra.resident = w->resident_mask;
  ra.d_aux = gr->d_aux;
  ra.d_scores = gr->d_scores;
  ra.d_logits = gr->d_logits;
  ra.tokens = s.T;
  ra.num_experts = s.E;
  ra.top_k = s.k;
  return launch_bwd_router(ra, st);
}

int spx_experts_forward(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* rows,
                        const int64_t* row_expert, uint16_t* out_rows, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (dims->top_k != 1) return SPX_ERR_INVALID_ARG;  // one expert per row
  if (rows == nullptr || row_expert == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (int rc = check_layer_weights(s, dims, w, false, true, false); rc != SPX_OK) return rc;
  if (!aligned16(rows) || (out_rows != nullptr && !aligned16(out_rows)) || !aligned16(workspace))
    return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), nullptr};
  int rc = SPX_OK;
  const uint16_t* xa = nullptr;
  if ((rc = stage_pad(c, rows, &xa)) != SPX_OK) return rc;
  DispatchArgs da = dispatch_args(s, row_expert, nullptr, nullptr, workspace, L);
  da.lb_blocks = 0;  // no routing probabilities here
  da.utilization = at<float>(workspace, L.util);
  da.group_stats = at<long long>(workspace, L.stats);
  da.group_ratios = at<float>(workspace, L.ratios);
  da.pair_weights = nullptr;  // unit weights: the caller applies the routing weights
  da.sorted_weights = nullptr;
  if (s.mx && w->expert_lane_mxfp8 != nullptr) {
    da.lane_mx = w->expert_lane_mxfp8;
    da.tiles_mx = at<int4>(workspace, L.tiles_mx);
    da.num_tiles_mx = at<int>(workspace, L.small) + 3;
  }
  if ((rc = launch_dispatch(da, c.st)) != SPX_OK) return rc;
  if ((rc = stage_experts(c, w, rows, xa, da)) != SPX_OK) return rc;
  if (out_rows == nullptr) return SPX_OK;  // rows stay in dispatch order (spx_experts_sorted_rows)
  // back to the input row order (one "slot" per row)
  return launch_combine(at<uint16_t>(workspace, L.y), da.rank, nullptr, nullptr, s.T, s.d, 1, out_rows, c.st);
}

int spx_experts_forward_to(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* rows,
                           const int64_t* row_expert, uint16_t* const* row_out, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (dims->top_k != 1) return SPX_ERR_INVALID_ARG;
  if (rows == nullptr || row_expert == nullptr || row_out == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (int rc = check_layer_weights(s, dims, w, false, true, false); rc != SPX_OK) return rc;
  if (!aligned16(rows) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), nullptr};
  int rc = SPX_OK;
  const uint16_t* xa = nullptr;
  if ((rc = stage_pad(c, rows, &xa)) != SPX_OK) return rc;
  DispatchArgs da = dispatch_args(s, row_expert, nullptr, nullptr, workspace, L);
  da.lb_blocks = 0;
  da.utilization = at<float>(workspace, L.util);
  da.group_stats = at<long long>(workspace, L.stats);
  da.group_ratios = at<float>(workspace, L.ratios);
  da.pair_weights = nullptr;
  da.sorted_weights = nullptr;
  if (s.mx && w->expert_lane_mxfp8 != nullptr) {
    da.lane_mx = w->expert_lane_mxfp8;
    da.tiles_mx = at<int4>(workspace, L.tiles_mx);
    da.num_tiles_mx = at<int>(workspace, L.small) + 3;
  }
  if ((rc = launch_dispatch(da, c.st)) != SPX_OK) return rc;
  const bool mx = da.lane_mx != nullptr;
  if (mx) {
    rc = s.nv ? stage_quantize_nv_x(c, rows, 0, da) : stage_quantize_x(c, rows, 0);
    if (rc != SPX_OK) return rc;
  }
  ExpertPass p{w->expert_w1, w->expert_w2, w->expert_w1_mx, w->expert_w1_mx_scales, w->expert_w2_mx,
               w->expert_w2_mx_scales, s.E, da.tiles, da.num_tiles, mx ? da.tiles_mx : nullptr,
               mx ? da.num_tiles_mx : nullptr, 0, w->expert_nvfp4_amax};
  p.row_out = row_out;
  p.row_out_idx = da.src_row;
  return stage_expert_gemms(c, xa, da.src_row, da.sorted_weights, p);
}

int spx_experts_forward_rows(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* const* row_ptrs,
                             const int64_t* row_expert, uint16_t* const* row_out, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (dims->top_k != 1 || s.kd != s.d) return SPX_ERR_UNSUPPORTED;  // rows used as they are: d % 64 == 0
  if (row_ptrs == nullptr || row_expert == nullptr || row_out == nullptr) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (w == nullptr || w->expert_lane_mxfp8 != nullptr) return SPX_ERR_UNSUPPORTED;  // BF16 experts only
  if (int rc = check_layer_weights(s, dims, w, false, true, false); rc != SPX_OK) return rc;
  if (!aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), nullptr};
  DispatchArgs da = dispatch_args(s, row_expert, nullptr, nullptr, workspace, L);
  da.lb_blocks = 0;
  da.utilization = at<float>(workspace, L.util);
  da.group_stats = at<long long>(workspace, L.stats);
  da.group_ratios = at<float>(workspace, L.ratios);
  da.pair_weights = nullptr;
  da.sorted_weights = nullptr;
  if (int rc = launch_dispatch(da, c.st); rc != SPX_OK) return rc;
  ExpertPass p{w->expert_w1, w->expert_w2, nullptr, nullptr, nullptr, nullptr, s.E, da.tiles, da.num_tiles,
               nullptr, nullptr, 0, nullptr};
  p.row_out = row_out;
  p.row_out_idx = da.src_row;
  p.a_rows = reinterpret_cast<const uint8_t* const*>(row_ptrs);
  return stage_expert_gemms(c, nullptr, da.src_row, da.sorted_weights, p);
}

int spx_peer_row_pointers(const int32_t* const* sender_order, const int64_t* send_at, const int64_t* recv_seg,
                          int32_t groups, int32_t top_k, const uint16_t* const* sender_rows, int64_t ld_rows,
                          int64_t rows, const uint16_t** row_ptrs, void* stream) {
  if (groups < 1 || top_k < 1 || rows < 0 || ld_rows < 1) return SPX_ERR_INVALID_ARG;
  if (rows == 0) return SPX_OK;
  if (sender_order == nullptr || send_at == nullptr || recv_seg == nullptr || sender_rows == nullptr ||
      row_ptrs == nullptr)
    return SPX_ERR_INVALID_ARG;
  return launch_peer_row_pointers(sender_order, send_at, recv_seg, groups, top_k, sender_rows, ld_rows, rows,
                                  row_ptrs, static_cast<cudaStream_t>(stream));
}

int spx_experts_sorted_rows(const spx_layer_dims* dims, void* workspace, const uint16_t** sorted_rows,
                            const int32_t** row_rank) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (workspace == nullptr || sorted_rows == nullptr || row_rank == nullptr) return SPX_ERR_INVALID_ARG;
  const Layout L = make_layout(s);
  *sorted_rows = at<uint16_t>(workspace, L.y);
  *row_rank = at<int32_t>(workspace, L.rank);
  return SPX_OK;
}

int spx_shared_forward(const spx_layer_dims* dims, const spx_packed_weights* w, const uint16_t* hidden,
                       uint16_t* shared_out, void* workspace, void* stream) {
  Shape s;
  if (int rc = make_shape(dims, &s); rc != SPX_OK) return rc;
  if (hidden == nullptr || shared_out == nullptr) return SPX_ERR_INVALID_ARG;
  if (s.S == 0) return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr) return SPX_ERR_WORKSPACE;
  if (int rc = check_layer_weights(s, dims, w, false, false, true); rc != SPX_OK) return rc;
  if (!aligned16(hidden) || !aligned16(shared_out) || !aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  const Layout L = make_layout(s);
  const Ctx c{s, L, workspace, static_cast<cudaStream_t>(stream), at<int>(workspace, L.small), nullptr};
  const uint16_t* xa = nullptr;
  if (int rc = stage_pad(c, hidden, &xa); rc != SPX_OK) return rc;
  return stage_shared(c, w, xa, shared_out);
}

int spx_combine(const uint16_t* expert_rows, const int32_t* pair_rank, const uint16_t* pair_weights,
                const uint16_t* shared, int64_t tokens, int32_t d, int32_t top_k, uint16_t* update, void* stream) {
  if (tokens < 0 || d < 1 || top_k < 1 || top_k > kMaxTopK) return SPX_ERR_INVALID_ARG;
  if (tokens == 0) return SPX_OK;
  if (expert_rows == nullptr || pair_rank == nullptr || update == nullptr) return SPX_ERR_INVALID_ARG;
  return launch_combine(expert_rows, pair_rank, pair_weights, shared, tokens, d, top_k, update,
                        static_cast<cudaStream_t>(stream));
}

int spx_gather_rows(const uint16_t* src, int64_t ld_src, const int32_t* index, int32_t index_div, int64_t rows,
                    int32_t d, uint16_t* out, int64_t ld_out, void* stream) {
  if (rows < 0 || d < 1 || index_div < 1 || ld_src < d || ld_out < d) return SPX_ERR_INVALID_ARG;
  if (rows == 0) return SPX_OK;
  if (src == nullptr || index == nullptr || out == nullptr) return SPX_ERR_INVALID_ARG;
  return launch_gather_rows(src, ld_src, index, index_div, rows, d, out, ld_out, static_cast<cudaStream_t>(stream));
}

int spx_swiglu_backward_rows(const uint16_t* gate_up, int64_t ld_gate_up, int32_t chunk, const uint16_t* d_hidden,
                             int64_t ld_d_hidden, const uint16_t* weights, const int32_t* order, int64_t rows,
                             int32_t inter, int32_t inter_pad, uint16_t* hidden, uint16_t* d_gate_up,
                             float* d_weights, void* stream) {
  if (rows < 0 || chunk < 8 || inter < chunk || inter % chunk != 0 || inter_pad < inter || inter_pad % 8 != 0)
    return SPX_ERR_INVALID_ARG;
  if (ld_gate_up < 2 * static_cast<int64_t>(inter) || ld_d_hidden < inter || ld_gate_up > INT32_MAX ||
      ld_d_hidden > INT32_MAX)
    return SPX_ERR_INVALID_ARG;
  if (rows == 0) return SPX_OK;
  if (gate_up == nullptr || d_hidden == nullptr || weights == nullptr || order == nullptr || hidden == nullptr ||
      d_gate_up == nullptr || d_weights == nullptr)
    return SPX_ERR_INVALID_ARG;
  const uintptr_t any = reinterpret_cast<uintptr_t>(gate_up) | reinterpret_cast<uintptr_t>(d_hidden) |
                        reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(d_gate_up);
  if ((any & 15u) != 0) return SPX_ERR_INVALID_ARG;  // 16-byte row loads and stores
  return launch_bwd_swiglu(gate_up, static_cast<int>(ld_gate_up), chunk, d_hidden, static_cast<int>(ld_d_hidden),
                           weights, order, rows, inter, inter_pad, hidden, d_gate_up, d_weights,
                           static_cast<cudaStream_t>(stream));
}

size_t spx_calibration_workspace(int64_t batch, int64_t seq, int32_t num_experts) {
  if (batch < 1 || seq < 2 || num_experts < 1) return 0;
  return calibration_workspace_bytes(batch, seq, num_experts);
}

int spx_surprise_calibration(const uint16_t* router_scores, const int64_t* expert_ids, const uint16_t* routing_weights,
                             const float* token_nll, const uint8_t* valid, int64_t batch, int64_t seq,
                             int32_t num_experts, int32_t top_k, float* calibration, float* attributed_nll,
                             float* utilization, void* workspace, size_t workspace_bytes, void* stream) {
  if (batch < 1 || seq < 2 || num_experts < 1 || num_experts > 4096 || top_k < 1 || top_k > 32)
    return SPX_ERR_INVALID_ARG;
  if (router_scores == nullptr || expert_ids == nullptr || routing_weights == nullptr || token_nll == nullptr ||
      valid == nullptr)
    return SPX_ERR_INVALID_ARG;
  if (workspace == nullptr || workspace_bytes < calibration_workspace_bytes(batch, seq, num_experts))
    return SPX_ERR_WORKSPACE;
  if (!aligned16(workspace)) return SPX_ERR_ALIGNMENT;
  return launch_calibration(router_scores, expert_ids, routing_weights, token_nll, valid, batch, seq, num_experts,
                            top_k, calibration, attributed_nll, utilization, workspace,
                            static_cast<cudaStream_t>(stream));
}

int spx_workspace_status(void* workspace, int* device_status, int clear, void* stream) {
  if (workspace == nullptr || device_status == nullptr) return SPX_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return SPX_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return SPX_ERR_CUDA;
  *device_status = v;
  if (clear && v != 0) {
    if (cudaMemsetAsync(workspace, 0, sizeof(int), st) != cudaSuccess) return SPX_ERR_CUDA;
  }
  return SPX_OK;
}

}  // extern "C"
