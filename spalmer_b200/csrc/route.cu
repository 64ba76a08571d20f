// K1 (selection half): surprise scores, least-surprise top-k, routing weights
// and load-balance partial sums, from BF16 router logits.
//
// Reference: mESmaC/spalmer src/spalmer/experts/router.py:52-56 (softplus),
// router.py:80-95 (masked bottom-k, gather, softmax of -scores) and
// experts/losses.py:58-70 (softmax over all experts, mean over tokens).
//
// route_select_kernel: one CTA per 128 token rows, one thread per row.  The
//   CTA stages its rows of logits into shared memory with 16-byte coalesced
//   loads, maps them through the softplus table and writes router_scores.
//   Each thread keeps the k+1 smallest (score, index) keys of its row in
//   registers.  When those k+1 scores are pairwise distinct the CPU tie order
//   cannot matter and the sorted k smallest are final; otherwise the row is
//   appended to a tie list.  The same pass accumulates the per-expert sums of
//   BF16-rounded softmax(-scores) probabilities for the load-balance loss.
// route_ties_kernel: replays PyTorch's CPU top-k (topk_exact.cuh) for every
//   listed row, one warp per row (each partition step data-parallel over the
//   warp), the row staged in shared memory.
// route_rows_kernel: the same results for small batches (<= 4096 rows), one
//   warp per row end to end (tie replay inline), so a handful of rows still
//   spreads over many warps.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"
#include "topk_exact.cuh"

namespace spx {

__device__ __forceinline__ int64_t min_i64(int64_t a, int64_t b) { return a < b ? a : b; }

namespace {

// Total order on BF16 bit patterns that agrees with the CPU comparator:
// -0 == +0, NaN after +inf.
__device__ __forceinline__ uint32_t order_key16(uint16_t b) {
  if ((b & 0x7F80u) == 0x7F80u && (b & 0x007Fu) != 0u) return 0xFFFFu;  // NaN
  if (b == 0x8000u) b = 0;                                               // -0 -> +0
  return (b & 0x8000u) ? (~static_cast<uint32_t>(b) & 0xFFFFu) : (static_cast<uint32_t>(b) | 0x8000u);
}

// Softmax of the negated selected scores, computed in double and rounded to
// BF16 through float (the conversion PyTorch applies).
__device__ __forceinline__ void routing_softmax(const uint16_t* sel, int k, uint16_t* out) {
  double m = -1.0e300;
  for (int j = 0; j < k; ++j) m = fmax(m, -static_cast<double>(bf16_to_f32(sel[j])));
  double sum = 0.0;
  for (int j = 0; j < k; ++j) sum += exp(-static_cast<double>(bf16_to_f32(sel[j])) - m);
  for (int j = 0; j < k; ++j) {
    const double p = exp(-static_cast<double>(bf16_to_f32(sel[j])) - m) / sum;
    out[j] = f32_to_bf16_rne(__double2float_rn(p));
  }
}

}  // namespace

__global__ void softplus_table_kernel(uint16_t* lut) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= 65536) return;
  const uint16_t bits = static_cast<uint16_t>(b);
  const float x = bf16_to_f32(bits);
  uint16_t out;
  if (x != x) {
    out = 0x7FC0u;
  } else if (x > 20.0f) {
    out = bits;  // F.softplus threshold: returns the input unchanged
  } else {
    const double y = log1p(exp(static_cast<double>(x)));
    out = f32_to_bf16_rne(__double2float_rn(y));
  }
  lut[b] = out;
}

template <int K1MAX>
__global__ void __launch_bounds__(kRouteRows) route_select_kernel(const RouteArgs a) {
  extern __shared__ uint32_t route_smem[];
  const int E = a.num_experts;
  const int k = a.top_k;
  const int row_words = (((E + 1) / 2) | 1);  // odd stride -> conflict-free column reads
  uint16_t* tile = reinterpret_cast<uint16_t*>(route_smem);
  uint8_t* resident = reinterpret_cast<uint8_t*>(route_smem + kRouteRows * row_words);
  float* warp_sums = reinterpret_cast<float*>(route_smem + kRouteRows * row_words + (E + 3) / 4);

  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRouteRows;
  const int nrows = static_cast<int>(min_i64(kRouteRows, a.tokens - row0));
  const uint16_t* src = a.logits + row0 * E;
  uint16_t* dst = a.scores + row0 * E;
  const int total = nrows * E;

  for (int c = threadIdx.x; c < E; c += blockDim.x) resident[c] = a.resident ? a.resident[c] : 1;

  // Stage logits -> scores (coalesced), keep a row-strided copy in smem.
  if ((E & 7) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < total / 8; i += blockDim.x) {
      uint4 v = s4[i];
      uint16_t* h = reinterpret_cast<uint16_t*>(&v);
      const int base = i * 8;
      const int r = base / E;
      const int c = base - r * E;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (a.lut != nullptr) h[q] = a.lut[h[q]];
        tile[r * 2 * row_words + c + q] = h[q];
      }
      d4[i] = v;
    }
  } else {
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      uint16_t v = src[i];
      if (a.lut != nullptr) v = a.lut[v];
      const int r = i / E;
      tile[r * 2 * row_words + (i - r * E)] = v;
      dst[i] = v;
    }
  }
  __syncthreads();

  const int r = threadIdx.x;
  const bool live = r < nrows;
  const uint16_t* row = tile + r * 2 * row_words;

  // ---- k+1 smallest keys (packed key16 << 16 | index), ascending.
  uint32_t best[K1MAX];
#pragma unroll
  for (int j = 0; j < K1MAX; ++j) best[j] = 0xFFFFFFFFu;
  if (live) {
    for (int c = 0; c < E; ++c) {
      const uint16_t s = resident[c] ? row[c] : static_cast<uint16_t>(0x7F80u);
      const uint32_t w = (order_key16(s) << 16) | static_cast<uint32_t>(c);
      if (w < best[K1MAX - 1]) {
        best[K1MAX - 1] = w;
#pragma unroll
        for (int j = K1MAX - 1; j > 0; --j) {
          const uint32_t lo = min(best[j - 1], best[j]);
          const uint32_t hi = max(best[j - 1], best[j]);
          best[j - 1] = lo;
          best[j] = hi;
        }
      }
    }
    const int k1 = min(k + 1, E);
    bool tie = false;
#pragma unroll
    for (int j = 0; j + 1 < K1MAX; ++j)
      if (j + 1 < k1 && (best[j] >> 16) == (best[j + 1] >> 16)) tie = true;
    const int64_t grow = row0 + r;
    if (tie) {
      const int slot = atomicAdd(a.tie_count, 1);
      a.tie_rows[slot] = static_cast<int>(grow);
    }
    // The weights depend only on the selected scores in ascending order, which
    // a tie does not change (only which of several equal-score experts is
    // chosen), so they are final for tie rows too.  With a resident mask a
    // selected non-resident expert would carry its unmasked score; the tie
    // replay recomputes the weights in that configuration.
    uint16_t sel[K1MAX];
    uint16_t wts[K1MAX];
#pragma unroll
    for (int j = 0; j < K1MAX; ++j) {
      if (j < k) {
        const int id = static_cast<int>(best[j] & 0xFFFFu);
        if (!tie) a.ids[grow * k + j] = id;
        sel[j] = row[id];
      }
    }
    routing_softmax(sel, k, wts);
#pragma unroll
    for (int j = 0; j < K1MAX; ++j)
      if (j < k) a.weights[grow * k + j] = wts[j];
  }

  // ---- load-balance partials: sum over this CTA's rows of
  // bf16(softmax(-scores)) per expert (non-resident experts get 0).
  float mx = 0.0f, denom = 1.0f;
  if (live) {
    const uint32_t k0 = best[0] >> 16;  // smallest eligible key
    // decode key back to the score value
    const uint16_t b0 = (k0 & 0x8000u) ? static_cast<uint16_t>(k0 & 0x7FFFu) : static_cast<uint16_t>(~k0);
    mx = -bf16_to_f32(b0);
    float s = 0.0f;
    for (int c = 0; c < E; ++c)
      if (resident[c]) s += __expf(-bf16_to_f32(row[c]) - mx);
    denom = 1.0f / s;  // reciprocal: the probabilities below are rounded to BF16
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int g0 = 0; g0 < E; g0 += 32) {
    float v[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const int c = g0 + q;
      float p = 0.0f;
      if (live && c < E && resident[c]) p = round_bf16(__expf(-bf16_to_f32(row[c]) - mx) * denom);
      v[q] = p;
    }
    // Transpose-reduce: after 5 halving steps lane l holds column g0 + l.
#pragma unroll
    for (int width = 16; width >= 1; width >>= 1) {
      const bool upper = (lane & width) != 0;
#pragma unroll
      for (int q = 0; q < width; ++q) {
        const float keep = upper ? v[q + width] : v[q];
        const float send = upper ? v[q] : v[q + width];
        v[q] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, width);
      }
    }
    if (g0 + lane < E) warp_sums[warp * E + g0 + lane] = v[0];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < E; c += blockDim.x) {
    float s = 0.0f;
    for (int w = 0; w < kRouteRows / 32; ++w) s += warp_sums[w * E + c];
    a.lb_partial[static_cast<int64_t>(blockIdx.x) * E + c] = s;
  }
}

// One Hoare partition step of v[lo, hi) by a whole warp: the data-parallel
// form of exact::partition_by_lists (identical result, see topk_exact.cuh).
__device__ int warp_partition(uint32_t* v, int lo, int hi, uint16_t* lpos, uint16_t* rpos, int lane) {
  if (lane == 0) exact::median_to_slot(v, lo, lo + 1, lo + (hi - lo) / 2, hi - 1);
  __syncwarp();
  const uint32_t pivot = v[lo];
  const unsigned lt = (1u << lane) - 1u;
  int nl = 0, nr = 0;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    const bool in = p < hi;
    const uint32_t x = in ? v[p] : 0u;
    const bool is_l = in && p > lo && !exact::before(x, pivot);
    const bool is_r = in && !exact::before(pivot, x);
    const unsigned bl = __ballot_sync(0xFFFFFFFFu, is_l);
    const unsigned br = __ballot_sync(0xFFFFFFFFu, is_r);
    if (is_l) lpos[nl + __popc(bl & lt)] = static_cast<uint16_t>(p);
    if (is_r) rpos[nr + __popc(br & lt)] = static_cast<uint16_t>(p);
    nl += __popc(bl);
    nr += __popc(br);
  }
  __syncwarp();
  // Swaps happen for the leading m with Lo[m] < Ro[m]; the condition is
  // monotone in m, so each ballot is a run of low lanes.
  int m = 0;
  for (int m0 = 0;; m0 += 32) {
    const int q = m0 + lane;
    const bool c = q < nl && q < nr && lpos[q] < rpos[nr - 1 - q];
    const int ones = __popc(__ballot_sync(0xFFFFFFFFu, c));
    m += ones;
    if (ones < 32) break;
  }
  for (int q = lane; q < m; q += 32) {
    const int pl = lpos[q], pr = rpos[nr - 1 - q];
    const uint32_t t = v[pl];
    v[pl] = v[pr];
    v[pr] = t;
  }
  __syncwarp();
  if (m == 0) return lpos[0];
  const int left = m < nl ? lpos[m] : hi;
  const int right_prev = rpos[nr - m];
  return left < right_prev ? left : right_prev;
}

// exact::topk_least_cpu_order with the partition steps spread over a warp;
// the short sequential tails (<= 3 elements, the sort of the first k-1, heap
// fallbacks) run on lane 0.
__device__ void warp_topk_cpu_order(uint32_t* v, int n, int k, uint16_t* lpos, uint16_t* rpos, int lane) {
  if (k * 64 <= n) {
    if (lane == 0) exact::partial_sort_first(v, k, n);
    __syncwarp();
    return;
  }
  const int nth = k - 1;
  int lo = 0, hi = n;
  int depth = 2 * exact::floor_log2(n);
  bool by_heap = false;
  while (hi - lo > 3) {
    if (depth == 0) {
      if (lane == 0) {
        exact::heap_select(v, lo, nth + 1, hi);
        exact::swap_at(v, lo, nth);
      }
      by_heap = true;
      break;
    }
    --depth;
    const int cut = warp_partition(v, lo, hi, lpos, rpos, lane);
    if (cut <= nth)
      lo = cut;
    else
      hi = cut;
  }
  if (lane == 0 && !by_heap) exact::insertion_sort(v, lo, hi);
  __syncwarp();
  const int m = k - 1;
  if (m <= 16) {
    // std::sort of at most 16 elements is a plain insertion sort, i.e. a
    // stable sort: every lane ranks one element (earlier equal ones first).
    uint32_t x = 0;
    int rank = 0;
    if (lane < m) {
      x = v[lane];
      for (int i = 0; i < m; ++i) {
        const uint32_t y = v[i];
        rank += (exact::before(y, x) || (i < lane && !exact::before(x, y))) ? 1 : 0;
      }
    }
    __syncwarp();
    if (lane < m) v[rank] = x;
  } else if (lane == 0) {
    exact::intro_sort(v, m);
  }
  __syncwarp();
}

__device__ __forceinline__ uint16_t key16_to_bits(uint32_t key) {
  return (key & 0x8000u) ? static_cast<uint16_t>(key & 0x7FFFu) : static_cast<uint16_t>(~key & 0xFFFFu);
}

// Column of lane `lane`'s slot q (8 slots per 256-column chunk).
__device__ __forceinline__ int route_col(int q, int lane, bool vec) {
  return vec ? 8 * (32 * (q >> 3) + lane) + (q & 7) : lane + 32 * q;
}

// Small-T route: one warp per token row (rows strided over all warps).  Lane l
// owns 8 consecutive columns per 256-column chunk (one 16-byte load), maps
// them through the softplus table and writes router_scores; the k+1 smallest
// (score, index) keys come out of k+1 rounds of a warp min-reduction
// (redux.sync).  Rows whose k+1 scores are distinct are final; otherwise the
// same warp replays PyTorch's CPU top-k (warp_topk_cpu_order).  Lanes keep
// per-column load-balance sums; a CTA reduces its warps' sums into one
// partial row.  Used when the rows are too few to fill the GPU one thread
// per row (decode-sized batches).
template <int NCH, int K1MAX>
__global__ void __launch_bounds__(kRouteWarps * 32) route_rows_kernel(const RouteArgs a) {
  constexpr int NQ = 8 * NCH;  // columns per lane
  extern __shared__ uint32_t route_smem[];
  const int E = a.num_experts;
  const int k = a.top_k;
  const int k1 = min(k + 1, E);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half_words = (E + 1) / 2;
  float* lb = reinterpret_cast<float*>(route_smem);                               // [warps][E]
  uint8_t* resident = reinterpret_cast<uint8_t*>(lb + kRouteWarps * E);            // [E]
  uint32_t* v = route_smem + kRouteWarps * E + (E + 3) / 4 + warp * (E + 2 * half_words);
  uint16_t* lpos = reinterpret_cast<uint16_t*>(v + E);
  uint16_t* rpos = reinterpret_cast<uint16_t*>(v + E + half_words);
  for (int c = threadIdx.x; c < E; c += blockDim.x) resident[c] = a.resident ? a.resident[c] : 1;
  __syncthreads();

  const bool vec = (E & 7) == 0 && (reinterpret_cast<uintptr_t>(a.logits) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.scores) & 15u) == 0;
  float acc[NQ];
#pragma unroll
  for (int q = 0; q < NQ; ++q) acc[q] = 0.0f;

  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kRouteWarps;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kRouteWarps + warp; row < a.tokens; row += nwarps) {
    const uint16_t* src = a.logits + row * E;
    uint16_t* dst = a.scores + row * E;
    // ---- scores of this lane's columns (raw BF16 bits)
    uint16_t sc[NQ];
    if (vec) {
#pragma unroll
      for (int m = 0; m < NCH; ++m) {
        const int c0 = 8 * (32 * m + lane);
        if (c0 < E) {
          uint4 u = __ldg(reinterpret_cast<const uint4*>(src + c0));
          uint16_t* h = reinterpret_cast<uint16_t*>(&u);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (a.lut != nullptr) h[j] = __ldg(a.lut + h[j]);
            sc[8 * m + j] = h[j];
          }
          *reinterpret_cast<uint4*>(dst + c0) = u;
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) sc[8 * m + j] = 0;
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int c = lane + 32 * q;
        uint16_t b = 0;
        if (c < E) {
          b = src[c];
          if (a.lut != nullptr) b = __ldg(a.lut + b);
          dst[c] = b;
        }
        sc[q] = b;
      }
    }
    // ---- k+1 smallest keys (order_key16 << 16 | column), ascending
    uint32_t key[NQ];
    uint32_t lane_min = 0xFFFFFFFFu;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int c = route_col(q, lane, vec);
      uint32_t w = 0xFFFFFFFFu;
      if (c < E) w = (order_key16(resident[c] ? sc[q] : static_cast<uint16_t>(0x7F80u)) << 16) | static_cast<uint32_t>(c);
      key[q] = w;
      lane_min = min(lane_min, w);
    }
    uint32_t best[K1MAX];
#pragma unroll
    for (int j = 0; j < K1MAX; ++j) {
      best[j] = 0xFFFFFFFFu;
      if (j < k1) {
        const uint32_t m = __reduce_min_sync(0xFFFFFFFFu, lane_min);
        best[j] = m;
        if (lane_min == m) {
          uint32_t nm = 0xFFFFFFFFu;
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            if (key[q] == m) key[q] = 0xFFFFFFFFu;
            nm = min(nm, key[q]);
          }
          lane_min = nm;
        }
      }
    }
    bool tie = false;
#pragma unroll
    for (int j = 0; j + 1 < K1MAX; ++j)
      if (j + 1 < k1 && (best[j] >> 16) == (best[j + 1] >> 16)) tie = true;

    // ---- routing weights: softmax(-selected scores) in double, summed in slot order.
    // They depend only on the selected scores in ascending order, which a tie
    // does not change; with a resident mask a tie row is recomputed below.
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < K1MAX; ++j)
      if (j == lane) mine = best[j];
    const double x0 = -static_cast<double>(bf16_to_f32(key16_to_bits(best[0] >> 16)));
    double e = 0.0;
    if (lane < k) e = exp(-static_cast<double>(bf16_to_f32(key16_to_bits(mine >> 16))) - x0);
    double sum = 0.0;
    for (int j = 0; j < k; ++j) sum += __shfl_sync(0xFFFFFFFFu, e, j);
    if (lane < k) a.weights[row * k + lane] = f32_to_bf16_rne(__double2float_rn(e / sum));

    if (!tie) {
      if (lane < k) a.ids[row * k + lane] = static_cast<int64_t>(mine & 0xFFFFu);
    } else {
      // Exact CPU order: stage (raw bits << 16 | column) and replay nth_element + sort.
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int c = route_col(q, lane, vec);
        if (c < E) {
          const uint16_t b = resident[c] ? sc[q] : static_cast<uint16_t>(0x7F80u);
          v[c] = (static_cast<uint32_t>(b) << 16) | static_cast<uint32_t>(c);
        }
      }
      __syncwarp();
      warp_topk_cpu_order(v, E, k, lpos, rpos, lane);
      if (lane < k) a.ids[row * k + lane] = static_cast<int64_t>(v[lane] & 0xFFFFu);
      if (a.resident != nullptr) {
        // A selected non-resident expert carries its unmasked score (router.py:91).
        __syncwarp();
        if (lane == 0) {
          uint16_t sel[kMaxTopK];
          uint16_t wts[kMaxTopK];
          for (int j = 0; j < k; ++j) sel[j] = dst[v[j] & 0xFFFFu];
          routing_softmax(sel, k, wts);
          for (int j = 0; j < k; ++j) a.weights[row * k + j] = wts[j];
        }
      }
      __syncwarp();
    }

    // ---- load-balance partials: bf16(softmax(-scores)) over eligible experts
    const float mx = -bf16_to_f32(key16_to_bits(best[0] >> 16));  // max of -score
    float ex[NQ];
    float part = 0.0f;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int c = route_col(q, lane, vec);
      ex[q] = 0.0f;
      if (c < E && resident[c]) ex[q] = __expf(-bf16_to_f32(sc[q]) - mx);
      part += ex[q];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xFFFFFFFFu, part, off);
    const float denom = 1.0f / part;  // reciprocal: the probabilities are rounded to BF16
#pragma unroll
    for (int q = 0; q < NQ; ++q) acc[q] += round_bf16(ex[q] * denom);
  }

  // ---- CTA reduction of the per-column sums (fixed order: deterministic)
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int c = route_col(q, lane, vec);
    if (c < E) lb[warp * E + c] = acc[q];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < E; c += blockDim.x) {
    float t = 0.0f;
    for (int w = 0; w < kRouteWarps; ++w) t += lb[w * E + c];
    a.lb_partial[static_cast<int64_t>(blockIdx.x) * E + c] = t;
  }
}

__global__ void __launch_bounds__(kTieWarps * 32) route_ties_kernel(const RouteArgs a) {
  extern __shared__ uint32_t tie_smem[];
  const int E = a.num_experts;
  const int k = a.top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half_words = (E + 1) / 2;
  uint32_t* v = tie_smem + warp * (E + 2 * half_words);
  uint16_t* lpos = reinterpret_cast<uint16_t*>(v + E);
  uint16_t* rpos = reinterpret_cast<uint16_t*>(v + E + half_words);
  const int n_ties = *a.tie_count;
  for (int t = blockIdx.x * kTieWarps + warp; t < n_ties; t += gridDim.x * kTieWarps) {
    const int64_t row = a.tie_rows[t];
    const uint16_t* s = a.scores + row * E;
    for (int c = lane; c < E; c += 32) {
      const bool res = a.resident == nullptr || a.resident[c] != 0;
      const uint16_t b = res ? s[c] : static_cast<uint16_t>(0x7F80u);
      v[c] = (static_cast<uint32_t>(b) << 16) | static_cast<uint32_t>(c);
    }
    __syncwarp();
    warp_topk_cpu_order(v, E, k, lpos, rpos, lane);
    if (lane < k) a.ids[row * k + lane] = static_cast<int64_t>(v[lane] & 0xFFFFu);
    if (lane == 0 && a.resident != nullptr) {  // otherwise route_select's weights are exact
      uint16_t sel[kMaxTopK];
      uint16_t wts[kMaxTopK];
      for (int j = 0; j < k; ++j) sel[j] = s[v[j] & 0xFFFFu];
      routing_softmax(sel, k, wts);
      for (int j = 0; j < k; ++j) a.weights[row * k + j] = wts[j];
    }
    __syncwarp();
  }
}

int launch_softplus_table(uint16_t* lut, cudaStream_t stream) {
  softplus_table_kernel<<<256, 256, 0, stream>>>(lut);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

size_t route_select_smem(int E) {
  const int row_words = (((E + 1) / 2) | 1);
  return static_cast<size_t>(kRouteRows) * row_words * 4 + ((E + 3) / 4) * 4 +
         static_cast<size_t>(kRouteRows / 32) * E * 4;
}

int route_lb_blocks(int64_t tokens) {
  if (tokens <= kRouteRowsMaxTokens) return static_cast<int>((tokens + kRouteWarps - 1) / kRouteWarps);
  return static_cast<int>((tokens + kRouteRows - 1) / kRouteRows);
}

static size_t route_rows_smem(int E) {
  const int half_words = (E + 1) / 2;
  return static_cast<size_t>(kRouteWarps) * E * 4 + ((E + 3) / 4) * 4 +
         static_cast<size_t>(kRouteWarps) * (E + 2 * half_words) * 4;
}

template <int NCH, int K1MAX>
static int launch_route_rows_t(const RouteArgs& a, cudaStream_t stream) {
  const void* fn = reinterpret_cast<const void*>(route_rows_kernel<NCH, K1MAX>);
  if (ensure_max_dynamic_smem(fn) != SPX_OK) return SPX_ERR_CUDA;
  route_rows_kernel<NCH, K1MAX><<<route_lb_blocks(a.tokens), kRouteWarps * 32, route_rows_smem(a.num_experts),
                                  stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

template <int NCH>
static int launch_route_rows_k(const RouteArgs& a, cudaStream_t stream) {
  if (a.top_k + 1 <= 5) return launch_route_rows_t<NCH, 5>(a, stream);
  if (a.top_k + 1 <= 9) return launch_route_rows_t<NCH, 9>(a, stream);
  return launch_route_rows_t<NCH, kMaxTopK + 1>(a, stream);
}

int launch_route(const RouteArgs& a, cudaStream_t stream) {
  if (a.tokens <= 0) return SPX_OK;
  if (a.tokens <= kRouteRowsMaxTokens) {
    const int nch = (a.num_experts + 255) / 256;
    if (nch <= 1) return launch_route_rows_k<1>(a, stream);
    if (nch <= 2) return launch_route_rows_k<2>(a, stream);
    return launch_route_rows_k<4>(a, stream);
  }
  const int blocks = static_cast<int>((a.tokens + kRouteRows - 1) / kRouteRows);
  const size_t smem = route_select_smem(a.num_experts);
  cudaError_t err;
  if (a.top_k + 1 <= 5) {
    if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(route_select_kernel<5>)) != SPX_OK) return SPX_ERR_CUDA;
    route_select_kernel<5><<<blocks, kRouteRows, smem, stream>>>(a);
  } else if (a.top_k + 1 <= 9) {
    if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(route_select_kernel<9>)) != SPX_OK) return SPX_ERR_CUDA;
    route_select_kernel<9><<<blocks, kRouteRows, smem, stream>>>(a);
  } else {
    if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(route_select_kernel<kMaxTopK + 1>)) != SPX_OK) return SPX_ERR_CUDA;
    route_select_kernel<kMaxTopK + 1><<<blocks, kRouteRows, smem, stream>>>(a);
  }
  err = cudaGetLastError();
  if (err != cudaSuccess) return SPX_ERR_CUDA;
  const size_t tsmem = static_cast<size_t>(kTieWarps) * (a.num_experts + 2 * ((a.num_experts + 1) / 2)) * 4;
  if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(route_ties_kernel)) != SPX_OK) return SPX_ERR_CUDA;
  int tie_blocks = static_cast<int>((a.tokens + kTieWarps - 1) / kTieWarps);
  if (tie_blocks > a.sm_count * 8) tie_blocks = a.sm_count * 8;
  route_ties_kernel<<<tie_blocks, kTieWarps * 32, tsmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
