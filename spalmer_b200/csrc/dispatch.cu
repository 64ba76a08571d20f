// K2 dispatch: stable counting sort of routed pairs by expert id, the grouped
// GEMM tile table, and the per-layer routing statistics.
//
// Reference: mESmaC/spalmer src/spalmer/experts/bank.py:721-736
// (`_pair_counts`, `cumsum`, `argsort(expert_index, stable=True)`, group ids),
// experts/losses.py:17-33 (utilization), losses.py:58-70 (load-balance loss)
// and experts/mixer.py:244-297 (padding / load telemetry).  The reference
// syncs with the host twice here; this path keeps everything on the device.
//
// Pairs are in the reference's order p = token * k + slot
// (mixer.py:193-197).  The permutation equals argsort(stable=True): pairs of
// one expert keep increasing p.
//   dispatch_count_kernel   per-chunk expert histograms (chunk = 2048 pairs)
//   dispatch_prefix_kernel  per expert: chunk offsets and totals; load-balance sums
//   dispatch_scan_kernel    one CTA: starts, tile tables, utilization, group
//                           statistics, auxiliary loss
//   dispatch_scatter_kernel per-chunk stable placement (warp match_any ranks)
//   dispatch_small_kernel   all of the above in one CTA for <= 4096 pairs
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

__device__ __forceinline__ int64_t min_i64(int64_t a, int64_t b) { return a < b ? a : b; }

__global__ void __launch_bounds__(kDispatchThreads) dispatch_count_kernel(const DispatchArgs a) {
  extern __shared__ int hist[];
  const int E = a.num_experts;
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * kDispatchChunk;
  const int64_t p1 = min_i64(a.pairs, p0 + kDispatchChunk);
  for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const int64_t e = a.ids[p];
    if (e < 0 || e >= E) {
      record_error(a.status, SPX_DEV_BAD_EXPERT);
      continue;
    }
    atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  // Expert-major layout [E][nchunks]: the scan reads each expert's chunks contiguously.
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    a.chunk_hist[static_cast<int64_t>(e) * gridDim.x + blockIdx.x] = hist[e];
}

__device__ __forceinline__ int64_t next_pow2_i64(int64_t n) {
  int64_t c = 1;
  while (c < n) c <<= 1;
  return c;
}

// Parallel prefix work ahead of the single-CTA scan (it was the scan's
// critical path when done by 32 warps serially):
//   blocks [0, E)        one expert each: exclusive scan of its per-chunk counts
//                        in place (chunk offsets within the expert) and its total
//                        into counts[e];
//   blocks [E, E + E/32) the load-balance sums: 32 experts per block, the route
//                        partial rows summed in a fixed order into lb_sum[e].
constexpr int kPrefixWarps = 32;

__global__ void __launch_bounds__(kPrefixWarps * 32) dispatch_prefix_kernel(const DispatchArgs a) {
  const int E = a.num_experts;
  const int nchunks = static_cast<int>((a.pairs + kDispatchChunk - 1) / kDispatchChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (static_cast<int>(blockIdx.x) < E) {
    if (warp != 0) return;
    const int x = blockIdx.x;
    int* row = a.chunk_hist + static_cast<int64_t>(x) * nchunks;
    int carry = 0;
    for (int base = 0; base < nchunks; base += 32 * 16) {
      const int c0 = base + lane * 16;
      int vals[16];
      int sum = 0;
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        vals[q] = (c0 + q < nchunks) ? row[c0 + q] : 0;
        sum += vals[q];
      }
      int incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
        if (lane >= off) incl += v;
      }
      int run = carry + incl - sum;
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        if (c0 + q < nchunks) row[c0 + q] = run;
        run += vals[q];
      }
      carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) a.counts[x] = carry;
    return;
  }
  // load-balance sums: lane -> expert, warp -> every 32nd partial row, then the
  // warps folded in order (deterministic)
  __shared__ float part[kPrefixWarps][32];
  const int x = (blockIdx.x - E) * 32 + lane;
  float acc = 0.0f;
  if (x < E) {
    for (int b0 = warp; b0 < a.lb_blocks; b0 += kPrefixWarps * 8) {
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int b = b0 + q * kPrefixWarps;
        v[q] = b < a.lb_blocks ? a.lb_partial[static_cast<int64_t>(b) * E + x] : 0.0f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) acc += v[q];
    }
  }
  part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && x < E) {
    float t = 0.0f;
    for (int w = 0; w < kPrefixWarps; ++w) t += part[w][lane];
    a.lb_sum[x] = t;
  }
}

// Per-expert inputs of the finishing pass (thread e holds expert e's), loaded
// by the caller ahead of its first barrier so that their latency overlaps the
// counting.
struct ExpertIn {
  int count;     // pairs routed to the expert
  float lb;      // its load-balance sum (used with aux_loss)
  bool mx;       // runs the MXFP8 lane
  bool resident;
  float recon;   // reconstruction error of its low-precision copies (quant_error)
};

__device__ __forceinline__ ExpertIn load_expert_in(const DispatchArgs& a, int e) {
  ExpertIn in{0, 0.0f, false, false, 0.0f};
  if (e < a.num_experts) {
    in.mx = a.lane_mx != nullptr && a.lane_mx[e] != 0;
    in.resident = a.resident != nullptr && a.resident[e] != 0;
    in.recon = a.recon_error != nullptr ? a.recon_error[e] : 0.0f;
  }
  return in;
}

// Shared by the scan kernels: from each expert's inputs, the pair starts,
// both lanes' tile tables, utilization, quantization telemetry, group
// statistics and the auxiliary loss.  One CTA of 1024 threads; E <= 1024.
struct ScanShared {
  int scan[1024];
  unsigned long long scan64[1024];
  float red[32];
  long long stat[32][4];
};

// Inclusive scan over the 1024 threads of the CTA: shuffles within each warp,
// the 32 warp totals scanned by warp 0 (two CTA barriers).  `tot` receives the
// sum of all values.  Integer sums, so the order does not matter.
template <typename T>
__device__ __forceinline__ T block_inclusive_scan(T v, T* warp_tot, T& tot) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const T u = __shfl_up_sync(0xFFFFFFFFu, v, off);
    if (lane >= off) v += u;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T w = warp_tot[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const T u = __shfl_up_sync(0xFFFFFFFFu, w, off);
      if (lane >= off) w += u;
    }
    warp_tot[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  tot = warp_tot[31];
  return v + (warp > 0 ? warp_tot[warp - 1] : T(0));
}

// Returns this thread's expert's first dispatch position.  Barriers: the
// scan (two; four when P >= 2^21 needs separate scans of the pair and tile
// counts) and one for the statistics.
__device__ __forceinline__ int finish_dispatch(const DispatchArgs& a, const ExpertIn& in, ScanShared& sh) {
  const int E = a.num_experts;
  const int e = threadIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool valid = e < E;
  const int count = valid ? in.count : 0;
  const int tiles = (count + kTileRows - 1) / kTileRows;
  // Block-wide exclusive scans of the pair counts and of both lanes' tile
  // counts: one scan of three 21-bit fields while the totals fit.
  int start, tile_start, tiles_bf, tiles_mx;
  if (a.pairs < (int64_t(1) << 21)) {
    const unsigned long long mine =
        static_cast<unsigned long long>(count) |
        (static_cast<unsigned long long>(in.mx ? 0 : tiles) << 21) |
        (static_cast<unsigned long long>(in.mx ? tiles : 0) << 42);
    unsigned long long all = 0ull;
    const unsigned long long excl = block_inclusive_scan<unsigned long long>(mine, sh.scan64, all) - mine;
    constexpr unsigned long long kField = (1ull << 21) - 1ull;
    start = static_cast<int>(excl & kField);
    tile_start = static_cast<int>(in.mx ? (excl >> 42) & kField : (excl >> 21) & kField);
    tiles_bf = static_cast<int>((all >> 21) & kField);
    tiles_mx = static_cast<int>((all >> 42) & kField);
  } else {
    int total_pairs = 0;
    start = block_inclusive_scan<int>(count, sh.scan, total_pairs) - count;
    // BF16-lane tiles in the low 32 bits, MXFP8-lane tiles in the high 32 bits
    const unsigned long long mine =
        in.mx ? (static_cast<unsigned long long>(tiles) << 32) : static_cast<unsigned long long>(tiles);
    unsigned long long all = 0ull;
    const unsigned long long excl = block_inclusive_scan<unsigned long long>(mine, sh.scan64, all) - mine;
    tile_start = in.mx ? static_cast<int>(excl >> 32) : static_cast<int>(excl & 0xFFFFFFFFull);
    tiles_bf = static_cast<int>(all & 0xFFFFFFFFull);
    tiles_mx = static_cast<int>(all >> 32);
  }
  if (threadIdx.x == 1023) {
    *a.num_tiles = tiles_bf;
    if (a.num_tiles_mx != nullptr) *a.num_tiles_mx = tiles_mx;
  }
  // Utilization (losses.py:28-33): count / P in float32.
  const float util = valid ? static_cast<float>(count) / static_cast<float>(a.pairs) : 0.0f;
  if (valid) {
    a.counts[e] = count;
    a.starts[e] = start;
    int4* table = in.mx ? a.tiles_mx : a.tiles;
    for (int t = 0; t < tiles; ++t) {
      const int r0 = t * kTileRows;
      // w repeats the expert: a page of a paged pass renames x to a cache slot
      table[tile_start + t] = make_int4(e, start + r0, min(kTileRows, count - r0), e);
    }
    if (a.utilization != nullptr) a.utilization[e] = util;
    // Quantization telemetry (bank.py:526-566): the error of every selected expert, zero elsewhere.
    if (a.quant_error != nullptr) a.quant_error[e] = count > 0 ? in.recon : 0.0f;
  }

  // Group statistics (mixer.py:257-297) and the load-balance loss
  // (losses.py:58-70) in one reduction round: warp reductions, then thread 0
  // folds the 32 warp results in order.
  const bool act = valid && count > 0;
  long long groups_w = __popc(__ballot_sync(0xFFFFFFFFu, act));
  long long resid_w = __popc(__ballot_sync(0xFFFFFFFFu, valid && in.resident));
  long long max_w = act ? count : 0;
  long long pad_w = act ? (a.execution_loop ? count : next_pow2_i64(count)) : 0;
  // mean_p = bf16(sum_t p / T), frac = bf16(util), prod = bf16(frac*mean_p)
  float prod = 0.0f;
  const bool lb = a.aux_loss != nullptr && a.lb_blocks > 0;
  if (valid && lb) prod = round_bf16(round_bf16(util) * round_bf16(in.lb / static_cast<float>(a.tokens)));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    max_w = max(max_w, __shfl_xor_sync(0xFFFFFFFFu, max_w, off));
    pad_w += __shfl_xor_sync(0xFFFFFFFFu, pad_w, off);
    prod += __shfl_xor_sync(0xFFFFFFFFu, prod, off);
  }
  if (lane == 0) {
    sh.stat[warp][0] = groups_w;
    sh.stat[warp][1] = resid_w;
    sh.stat[warp][2] = max_w;
    sh.stat[warp][3] = pad_w;
    sh.red[warp] = prod;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    long long g = 0, rsd = 0, mx = 0, pad = 0;
    float total = 0.0f;
    for (int w = 0; w < 32; ++w) {
      g += sh.stat[w][0];
      rsd += sh.stat[w][1];
      mx = max(mx, sh.stat[w][2]);
      pad += sh.stat[w][3];
      total += sh.red[w];
    }
    if (a.group_stats != nullptr) {
      const long long real = a.pairs;
      a.group_stats[0] = g;        // expert_group_count
      a.group_stats[1] = mx;       // expert_group_max_load
      a.group_stats[2] = real;     // expert_group_real_pairs
      a.group_stats[3] = pad;      // expert_group_padded_pairs
      a.group_stats[4] = mx * g;   // ..._global_max_counterfactual_padded_pairs
      a.group_stats[5] = g;        // num_active_experts ((utilization > 0).sum())
      a.group_ratios[0] = static_cast<float>(pad) / static_cast<float>(real);
      a.group_ratios[1] = static_cast<float>(mx * g) / static_cast<float>(real);
    }
    if (lb) {
      // total = bf16(sum prod), loss = bf16(bf16(eligible) * total)
      const long long n_eligible = a.resident != nullptr ? rsd : a.eligible_experts;
      const float eligible = round_bf16(static_cast<float>(n_eligible));
      a.aux_loss[0] = f32_to_bf16_rne(eligible * round_bf16(total));
    }
  }
  return start;
}

__global__ void __launch_bounds__(1024) dispatch_scan_kernel(const DispatchArgs a) {
  __shared__ ScanShared sh;
  const int e = threadIdx.x;
  // Chunk offsets, per-expert totals and load-balance sums come from dispatch_prefix_kernel.
  ExpertIn in = load_expert_in(a, e);
  if (e < a.num_experts) {
    in.count = a.counts[e];
    if (a.aux_loss != nullptr && a.lb_blocks > 0) in.lb = a.lb_sum[e];
  }
  finish_dispatch(a, in, sh);
}

// Small batches (pairs <= kDispatchSmallPairs): the whole dispatch in one CTA
// -- counts, the scan work above, then stable placement by warp 0, 32 pairs
// at a time in pair order (match_any ranks within the 32).  Every global read
// is issued before the first barrier.
__global__ void __launch_bounds__(1024) dispatch_small_kernel(const DispatchArgs a) {
  constexpr int kPer = kDispatchSmallPairs / 1024;  // pairs per thread
  __shared__ ScanShared sh;
  __shared__ int s_base[1024];
  __shared__ short s_ids[kDispatchSmallPairs];
  __shared__ uint16_t s_w[kDispatchSmallPairs];  // pair weights, so the placement loop reads no global memory
  const int E = a.num_experts;
  const int e = threadIdx.x;
  const int P = static_cast<int>(a.pairs);
  const bool weights = a.sorted_weights != nullptr;
  griddep_wait();  // the expert ids, weights and load-balance partials come from the route kernel
  griddep_launch_dependents();
  int64_t xid[kPer];
  uint16_t wv[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int p = threadIdx.x + j * 1024;
    xid[j] = p < P ? a.ids[p] : -1;
    wv[j] = (weights && p < P) ? a.pair_weights[p] : static_cast<uint16_t>(0);
  }
  ExpertIn in = load_expert_in(a, e);
  if (e < E && a.aux_loss != nullptr && a.lb_blocks > 0) {
#pragma unroll 8
    for (int b = 0; b < a.lb_blocks; ++b) in.lb += a.lb_partial[static_cast<int64_t>(b) * E + e];
  }
  s_base[e] = 0;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int p = threadIdx.x + j * 1024;
    if (p >= P) continue;
    const int64_t x = xid[j];
    const bool ok = x >= 0 && x < E;
    if (!ok) record_error(a.status, SPX_DEV_BAD_EXPERT);
    s_ids[p] = ok ? static_cast<short>(x) : static_cast<short>(-1);
    s_w[p] = wv[j];
    if (ok) atomicAdd(&s_base[x], 1);
  }
  __syncthreads();
  in.count = e < E ? s_base[e] : 0;
  const int start = finish_dispatch(a, in, sh);
  if (e < E) s_base[e] = start;  // nothing reads s_base between the count above and this store
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int g = 0; g < P; g += 32) {
    const int p = g + lane;
    const int x = p < P ? s_ids[p] : -1;
    const bool ok = x >= 0;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, x);
    int base = 0;
    if (ok) base = s_base[x];
    __syncwarp();
    if (ok) {
      const int pos = base + __popc(peers & lt_mask);
      a.order[pos] = p;
      a.src_row[pos] = p / a.top_k;
      if (a.rank != nullptr) a.rank[p] = pos;
      if (weights) a.sorted_weights[pos] = s_w[p];
      if ((peers & lt_mask) == 0) s_base[x] = base + __popc(peers);
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kDispatchThreads) dispatch_scatter_kernel(const DispatchArgs a) {
  extern __shared__ int warp_base[];  // [kDispatchWarps][E]
  const int E = a.num_experts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kSub = kDispatchChunk / kDispatchWarps;
  for (int i = threadIdx.x; i < kDispatchWarps * E; i += blockDim.x) warp_base[i] = 0;
  __syncthreads();
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * kDispatchChunk + static_cast<int64_t>(warp) * kSub;
  const int64_t p1 = min_i64(a.pairs, p0 + kSub);
  // Pass 1: per-warp counts of this warp's sub-chunk.
  for (int64_t p = p0 + lane; p < p1; p += 32) {
    const int64_t e = a.ids[p];
    if (e >= 0 && e < E) atomicAdd(&warp_base[warp * E + e], 1);
  }
  __syncthreads();
  // Per expert: global base = start + chunk offset, then exclusive over warps.
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int base = a.starts[e] + a.chunk_hist[static_cast<int64_t>(e) * gridDim.x + blockIdx.x];
    for (int w = 0; w < kDispatchWarps; ++w) {
      const int c = warp_base[w * E + e];
      warp_base[w * E + e] = base;
      base += c;
    }
  }
  __syncthreads();
  // Pass 2: stable placement, 32 consecutive pairs at a time.
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t g = p0; g < p1; g += 32) {
    const int64_t p = g + lane;
    const bool valid = p < p1;
    const int e = valid ? static_cast<int>(a.ids[p]) : -1;
    const bool ok = valid && e >= 0 && e < E;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, ok ? e : -1);
    int base = 0;
    if (ok) base = warp_base[warp * E + e];
    __syncwarp();
    if (ok) {
      const int rank = __popc(peers & lt_mask);
      const int pos = base + rank;
      a.order[pos] = static_cast<int>(p);
      a.src_row[pos] = static_cast<int>(p / a.top_k);
      if (a.rank != nullptr) a.rank[p] = pos;
      if (a.sorted_weights != nullptr) a.sorted_weights[pos] = a.pair_weights[p];
      if ((peers & lt_mask) == 0) warp_base[warp * E + e] = base + __popc(peers);
    }
    __syncwarp();
  }
}

int launch_dispatch(const DispatchArgs& a, cudaStream_t stream) {
  if (a.pairs <= 0) return SPX_ERR_INVALID_ARG;
  if (a.num_experts > 1024) return SPX_ERR_UNSUPPORTED;
  if (a.pairs <= kDispatchSmallPairs) {
    return launch_pdl(dispatch_small_kernel, dim3(1), dim3(1024), 0, stream, a);
  }
  const int nchunks = static_cast<int>((a.pairs + kDispatchChunk - 1) / kDispatchChunk);
  dispatch_count_kernel<<<nchunks, kDispatchThreads, a.num_experts * sizeof(int), stream>>>(a);
  if (cudaGetLastError() != cudaSuccess) return SPX_ERR_CUDA;
  const bool lb = a.aux_loss != nullptr && a.lb_blocks > 0;
  if (lb && a.lb_sum == nullptr) return SPX_ERR_INVALID_ARG;
  const int prefix_blocks = a.num_experts + (lb ? (a.num_experts + 31) / 32 : 0);
  dispatch_prefix_kernel<<<prefix_blocks, kPrefixWarps * 32, 0, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess) return SPX_ERR_CUDA;
  dispatch_scan_kernel<<<1, 1024, 0, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess) return SPX_ERR_CUDA;
  dispatch_scatter_kernel<<<nchunks, kDispatchThreads, kDispatchWarps * a.num_experts * sizeof(int), stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
