// K1 (selection half): surprise scores, least-surprise top-k, routing weights
// and load-balance partial sums, from BF16 router logits (or from scores
// that the router GEMM's epilogue already mapped through softplus).
//
// Reference: mESmaC/spalmer src/spalmer/experts/router.py:52-56 (softplus),
// router.py:80-95 (masked bottom-k, gather, softmax of -scores) and
// experts/losses.py:58-70 (softmax over all experts, mean over tokens).
//
// route_select_kernel: one CTA per 128 token rows, one thread per row.  The
//   CTA stages its rows into shared memory with 16-byte coalesced loads as
//   16-bit order keys (topk_exact.cuh), applying the softplus table and
//   writing router_scores when asked.  Each thread keeps the k+1 smallest
//   (key, index) words of its row in registers (a branch-free min/max
//   insertion network).  When those k+1 keys are pairwise distinct the CPU
//   tie order cannot matter and the sorted k smallest are final; otherwise
//   the row is appended to a tie list.  The load-balance term then runs
//   column-wise: each thread first records its row's softmax maximum and
//   normaliser, and the CTA sums bf16(softmax(-scores)) per expert over its
//   rows in a fixed order.
// route_ties_kernel: replays PyTorch's CPU top-k (topk_exact.cuh) for every
//   listed row, one warp per row (each partition step data-parallel over the
//   warp), the row staged in shared memory.
// route_rows_kernel: the same results for small batches (<= 4096 rows), one
//   warp per row end to end (tie replay inline), so a handful of rows still
//   spreads over many warps.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.h"
#include "sm100.cuh"
#include "topk_exact.cuh"

namespace spx {

using exact::key16_to_bits;
using exact::order_key16;

__device__ __forceinline__ int64_t min_i64(int64_t a, int64_t b) { return a < b ? a : b; }

namespace {

// Softmax of the negated selected scores x[0..k), computed in double and
// rounded to BF16 through float (the conversion PyTorch applies).
template <int N>
__device__ __forceinline__ void routing_softmax(const float (&x)[N], int k, uint16_t (&out)[N]) {
  double m = -1.0e300;
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (j < k) m = fmax(m, -static_cast<double>(x[j]));
  double e[N];
  double sum = 0.0;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    e[j] = j < k ? exp(-static_cast<double>(x[j]) - m) : 0.0;
    sum += e[j];
  }
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (j < k) out[j] = f32_to_bf16_rne(__double2float_rn(e[j] / sum));
}

// Routing weights of a row whose k selected experts are v[0..k) (low 16 bits),
// read back from the row's scores: routing_softmax with the exponentials
// recomputed instead of held, for the resident-mask case of the tie paths
// (a selected non-resident expert carries its unmasked score), which is rare
// and must not weigh on the replay's registers.
__device__ __forceinline__ void tie_row_weights(const uint32_t* v, const uint16_t* row_scores, int k,
                                                uint16_t* weights) {
  double m = -1.0e300;
#pragma unroll 1
  for (int j = 0; j < k; ++j) m = fmax(m, -static_cast<double>(bf16_to_f32(row_scores[v[j] & 0xFFFFu])));
  double sum = 0.0;
#pragma unroll 1
  for (int j = 0; j < k; ++j) sum += exp(-static_cast<double>(bf16_to_f32(row_scores[v[j] & 0xFFFFu])) - m);
#pragma unroll 1
  for (int j = 0; j < k; ++j) {
    const double e = exp(-static_cast<double>(bf16_to_f32(row_scores[v[j] & 0xFFFFu])) - m);
    weights[j] = f32_to_bf16_rne(__double2float_rn(e / sum));
  }
}

// bf16 round trip with the hardware conversion (round to nearest even).
__device__ __forceinline__ float bf16_round_hw(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

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

// Shared memory of route_select_kernel: the key tile [kRouteRows][2*row_words]
// (odd word stride: a column read across the CTA's rows is conflict-free) and
// the resident flags, then a region used first for the hot part of the
// softplus table (while staging) and then for per-row softmax statistics and
// per-quarter column sums of the load-balance term.  Sized so that four CTAs
// fit on an SM at E = 200.
constexpr int kLbQuarters = 4;
constexpr uint32_t kRouteLutLo = 121u << 7;  // magnitude bits of 2^-6
constexpr uint32_t kRouteLutN = 10u * 128u;  // binades [2^-6, 16) per sign

__host__ __device__ __forceinline__ int route_row_words(int E) { return ((E + 1) / 2) | 1; }

__host__ __device__ __forceinline__ size_t route_select_aux_bytes(int E) {
  const size_t lb = 2 * static_cast<size_t>(kRouteRows) * 4 + static_cast<size_t>(kLbQuarters) * E * 4;
  const size_t lut = 2 * kRouteLutN * 2;
  return lb > lut ? lb : lut;
}

// NONNEG: the staged values are softplus scores (>= +0, NaN only as 0x7FC0),
// whose BF16 bit patterns already sort like the CPU comparator, so the keys
// are the bits themselves.
template <int K1MAX, bool MASK, bool NONNEG>
__global__ void __launch_bounds__(2 * kRouteRows) route_select_kernel(const RouteArgs a) {
  extern __shared__ uint32_t route_smem[];
  const int E = a.num_experts;
  const int k = a.top_k;
  const int row_words = route_row_words(E);
  uint16_t* tile = reinterpret_cast<uint16_t*>(route_smem);
  uint8_t* resident = reinterpret_cast<uint8_t*>(route_smem + kRouteRows * row_words);
  uint32_t* aux = route_smem + kRouteRows * row_words + (E + 3) / 4;
  uint16_t* lut_hot = reinterpret_cast<uint16_t*>(aux);   // while staging
  float* row_mx = reinterpret_cast<float*>(aux);           // afterwards
  float* row_inv = row_mx + kRouteRows;
  float* quarter_sum = row_inv + kRouteRows;               // [kLbQuarters][E]

  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRouteRows;
  const int nrows = static_cast<int>(min_i64(kRouteRows, a.tokens - row0));
  const uint16_t* src = a.logits + row0 * E;
  uint16_t* dst = a.scores != nullptr ? a.scores + row0 * E : nullptr;  // may equal src (in place)
  const int total = nrows * E;

  if constexpr (MASK) {
    for (int c = threadIdx.x; c < E; c += blockDim.x) resident[c] = a.resident[c];
  }
  const uint16_t* lut = a.lut;
  if (lut != nullptr) {
    for (uint32_t i = threadIdx.x; i < 2 * kRouteLutN; i += blockDim.x) {
      const uint32_t neg = i >= kRouteLutN ? 1u : 0u;
      lut_hot[i] = __ldg(lut + ((neg << 15) | (kRouteLutLo + i - neg * kRouteLutN)));
    }
    __syncthreads();
  }
  auto map = [&](uint16_t b) -> uint16_t {
    if (lut == nullptr) return b;
    const uint32_t idx = (b & 0x7FFFu) - kRouteLutLo;
    return idx < kRouteLutN ? lut_hot[(b >> 15) * kRouteLutN + idx] : __ldg(lut + b);
  };
  auto key_of = [](uint16_t b) -> uint16_t { return NONNEG ? b : static_cast<uint16_t>(order_key16(b)); };

  // ---- stage keys (coalesced 16-byte loads, kStageBatch in flight per
  // thread; scores written back when asked, possibly in place)
  if ((E & 7) == 0) {
    constexpr int kStageBatch = 4;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    const int n16 = total / 8;
    for (int i0 = threadIdx.x; i0 < n16; i0 += kStageBatch * blockDim.x) {
      uint4 v[kStageBatch];
#pragma unroll
      for (int u = 0; u < kStageBatch; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < n16) v[u] = s4[i];
      }
#pragma unroll
      for (int u = 0; u < kStageBatch; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < n16) {
          uint16_t* h = reinterpret_cast<uint16_t*>(&v[u]);
          const int base = i * 8;
          const int r = base / E;
          const int c = base - r * E;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            h[q] = map(h[q]);
            tile[r * 2 * row_words + c + q] = key_of(h[q]);
          }
          if (dst != nullptr) d4[i] = v[u];
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const uint16_t v = map(src[i]);
      const int r = i / E;
      tile[r * 2 * row_words + (i - r * E)] = key_of(v);
      if (dst != nullptr) dst[i] = v;
    }
  }
  __syncthreads();  // the table region is reused below

  // Two threads per row: lanes 2r' and 2r'+1 of a warp share a row, each
  // taking the columns of its parity (the two reads of a column pair hit the
  // same shared-memory word).
  const int r = threadIdx.x >> 1;
  const int h = threadIdx.x & 1;
  const bool live = r < nrows;
  uint16_t* row = tile + r * 2 * row_words;
  auto value_of = [](uint32_t key) -> float {
    return bf16_to_f32(NONNEG ? static_cast<uint16_t>(key) : key16_to_bits(key));
  };
  // key of +inf (a masked expert)
  constexpr uint32_t kInfKey = NONNEG ? 0x7F80u : 0xFF80u;
  auto insert = [](uint32_t (&b)[K1MAX], uint32_t x) {
#pragma unroll
    for (int j = 0; j < K1MAX; ++j) {
      const uint32_t lo = min(b[j], x);
      x = max(b[j], x);
      b[j] = lo;
    }
  };

  // ---- k+1 smallest (key << 16 | index) words, ascending.  Each thread runs
  // two independent insertion networks over its columns (two dependency
  // chains in flight); the four partial lists of a row are merged at the end.
  uint32_t best[K1MAX];
#pragma unroll
  for (int j = 0; j < K1MAX; ++j) best[j] = 0xFFFFFFFFu;
  if (live) {
    uint32_t alt[K1MAX];
#pragma unroll
    for (int j = 0; j < K1MAX; ++j) alt[j] = 0xFFFFFFFFu;
    auto word = [&](int c) -> uint32_t {
      uint32_t key = row[c];
      if constexpr (MASK) key = resident[c] ? key : kInfKey;
      return (key << 16) | static_cast<uint32_t>(c);
    };
    int c = h;
#pragma unroll 2
    for (; c + 2 < E; c += 4) {
      insert(best, word(c));
      insert(alt, word(c + 2));
    }
    if (c < E) insert(best, word(c));
#pragma unroll
    for (int j = 0; j < K1MAX; ++j) insert(best, alt[j]);
  }
  // Merge the pair's lists (both threads end with the same list).
  uint32_t other[K1MAX];
#pragma unroll
  for (int j = 0; j < K1MAX; ++j) other[j] = __shfl_xor_sync(0xFFFFFFFFu, best[j], 1);
#pragma unroll
  for (int j = 0; j < K1MAX; ++j) insert(best, other[j]);
  if (live && h == 0) {
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
    // chosen), so they are final for tie rows too.  A selected non-resident
    // expert carries its unmasked score (router.py:91); with a resident mask
    // the tie replay recomputes the weights of its rows.
    float sel[K1MAX];
    uint16_t wts[K1MAX];
#pragma unroll
    for (int j = 0; j < K1MAX; ++j) {
      sel[j] = 0.0f;
      if (j < k) {
        const int id = static_cast<int>(best[j] & 0xFFFFu);
        if (!tie) a.ids[grow * k + j] = id;
        sel[j] = value_of(row[id]);
      }
    }
    routing_softmax<K1MAX>(sel, k, wts);
#pragma unroll
    for (int j = 0; j < K1MAX; ++j)
      if (j < k) a.weights[grow * k + j] = wts[j];
  }
  __syncthreads();  // keys -> exponentials below; the selection is done with the tile

  // ---- load balance, row half: e_c = exp(-score_c - max) over the eligible
  // experts (BF16, in place of the keys) and the row's normaliser.
  float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // independent add chains
  if (live) {
    const float mx = -value_of(best[0] >> 16);  // max of -score = -(smallest eligible score)
    int c = h;
    for (; c + 6 < E; c += 8) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int cc = c + 2 * q;
        float e = 0.0f;
        if (!MASK || resident[cc]) e = __expf(-value_of(row[cc]) - mx);
        part[q] += e;
        row[cc] = __bfloat16_as_ushort(__float2bfloat16_rn(e));
      }
    }
    for (; c < E; c += 2) {
      float e = 0.0f;
      if (!MASK || resident[c]) e = __expf(-value_of(row[c]) - mx);
      part[0] += e;
      row[c] = __bfloat16_as_ushort(__float2bfloat16_rn(e));
    }
    if (h == 0) row_mx[r] = mx;
  }
  float sum = (part[0] + part[1]) + (part[2] + part[3]);
  sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
  if (live && h == 0) row_inv[r] = 1.0f / sum;  // the probabilities are rounded to BF16
  __syncthreads();

  // ---- load balance, column half: per expert, the sum over this CTA's rows
  // of bf16(softmax(-scores)) = bf16(e * (1/sum)), rows in quarters.
  const int rq = (nrows + kLbQuarters - 1) / kLbQuarters;
  for (int item = threadIdx.x; item < kLbQuarters * E; item += blockDim.x) {
    const int q = item / E;
    const int c = item - q * E;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int r1 = min(nrows, (q + 1) * rq);
    int rr = q * rq;
    for (; rr + 3 < r1; rr += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        acc[u] += bf16_round_hw(bf16_to_f32(tile[(rr + u) * 2 * row_words + c]) * row_inv[rr + u]);
    }
    for (; rr < r1; ++rr) acc[0] += bf16_round_hw(bf16_to_f32(tile[rr * 2 * row_words + c]) * row_inv[rr]);
    quarter_sum[item] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < E; c += blockDim.x) {
    float t = 0.0f;
#pragma unroll
    for (int q = 0; q < kLbQuarters; ++q) t += quarter_sum[q * E + c];
    a.lb_partial[static_cast<int64_t>(blockIdx.x) * E + c] = t;
  }
}

// One Hoare partition step of v[lo, hi) by a whole warp: the data-parallel
// form of exact::partition_by_lists (identical result, see topk_exact.cuh).
__device__ int warp_partition(uint32_t* v, int lo, int hi, uint16_t* lpos, uint16_t* rpos, int lane) {
  if (lane == 0) exact::median_to_slot(v, lo, lo + 1, lo + (hi - lo) / 2, hi - 1);
  __syncwarp();
  const uint32_t pivot = v[lo];
  // !before(x, pivot) <=> x >= pivot_lo;  !before(pivot, x) <=> x <= pivot_hi
  const uint32_t pivot_lo = pivot & 0xFFFF0000u, pivot_hi = pivot | 0xFFFFu;
  const unsigned lt = (1u << lane) - 1u;
  int nl = 0, nr = 0;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    const bool in = p < hi;
    const uint32_t x = in ? v[p] : 0u;
    const bool is_l = in && p > lo && x >= pivot_lo;
    const bool is_r = in && x <= pivot_hi;
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
  griddep_wait();  // the logits (and the mask) come from earlier kernels
  griddep_launch_dependents();
  for (int c = threadIdx.x; c < E; c += blockDim.x) resident[c] = a.resident ? a.resident[c] : 1;
  __syncthreads();

  const bool vec = (E & 7) == 0 && (reinterpret_cast<uintptr_t>(a.logits) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.scores) & 15u) == 0;
  // Scores are re-read by the tie path below: from the output, or from the
  // input when it already holds scores (no table, no output).
  const uint16_t* score_src = a.scores != nullptr ? a.scores : a.logits;
  float acc[NQ];
#pragma unroll
  for (int q = 0; q < NQ; ++q) acc[q] = 0.0f;

  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kRouteWarps;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kRouteWarps + warp; row < a.tokens; row += nwarps) {
    const uint16_t* src = a.logits + row * E;
    uint16_t* dst = a.scores != nullptr ? a.scores + row * E : nullptr;
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
          if (dst != nullptr) *reinterpret_cast<uint4*>(dst + c0) = u;
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
          if (dst != nullptr) dst[c] = b;
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
      // Exact CPU order: stage (order key << 16 | column) and replay nth_element + sort.
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int c = route_col(q, lane, vec);
        if (c < E) v[c] = exact::make_elem(resident[c] ? sc[q] : static_cast<uint16_t>(0x7F80u), c);
      }
      __syncwarp();
      warp_topk_cpu_order(v, E, k, lpos, rpos, lane);
      if (lane < k) a.ids[row * k + lane] = static_cast<int64_t>(v[lane] & 0xFFFFu);
      if (a.resident != nullptr) {
        // A selected non-resident expert carries its unmasked score (router.py:91).
        __syncwarp();
        if (lane == 0) tie_row_weights(v, score_src + row * E, k, a.weights + row * k);
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

// NONNEG as in route_select_kernel: the staged words carry the score bits
// themselves as keys.
template <bool NONNEG>
__global__ void __launch_bounds__(kTieWarps * 32) route_ties_kernel(const RouteArgs a) {
  extern __shared__ uint32_t tie_smem[];
  const int E = a.num_experts;
  const int k = a.top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half_words = (E + 1) / 2;
  uint32_t* v = tie_smem + warp * (E + 2 * half_words);
  uint16_t* lpos = reinterpret_cast<uint16_t*>(v + E);
  uint16_t* rpos = reinterpret_cast<uint16_t*>(v + E + half_words);
  // Scores as route_select left them: its output, or its input when that
  // already held scores.
  const uint16_t* scores = a.scores != nullptr ? a.scores : a.logits;
  const int n_ties = *a.tie_count;
  for (int t = blockIdx.x * kTieWarps + warp; t < n_ties; t += gridDim.x * kTieWarps) {
    const int64_t row = a.tie_rows[t];
    const uint16_t* s = scores + row * E;
    for (int c0 = 0; c0 < E; c0 += 8 * 32) {  // up to 8 loads in flight per lane
      uint16_t b[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        b[u] = c < E ? s[c] : static_cast<uint16_t>(0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < E) {
          const bool res = a.resident == nullptr || a.resident[c] != 0;
          const uint16_t bb = res ? b[u] : static_cast<uint16_t>(0x7F80u);
          v[c] = NONNEG ? (static_cast<uint32_t>(bb) << 16) | static_cast<uint32_t>(c) : exact::make_elem(bb, c);
        }
      }
    }
    __syncwarp();
    warp_topk_cpu_order(v, E, k, lpos, rpos, lane);
    if (lane < k) a.ids[row * k + lane] = static_cast<int64_t>(v[lane] & 0xFFFFu);
    if (lane == 0 && a.resident != nullptr)  // otherwise route_select's weights are exact
      tie_row_weights(v, s, k, a.weights + row * k);
    __syncwarp();
  }
}

int launch_softplus_table(uint16_t* lut, cudaStream_t stream) {
  softplus_table_kernel<<<256, 256, 0, stream>>>(lut);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

// Router scores from logits in place: v = lut[v] for every BF16 value
// (F.softplus on BF16, experts/router.py:56), eight values per 16-byte load.
__global__ void scores_from_logits_kernel(uint16_t* __restrict__ v, int64_t n, const uint16_t* __restrict__ lut) {
  const int64_t n8 = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  uint4* v8 = reinterpret_cast<uint4*>(v);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    uint4 q = v8[i];
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = static_cast<uint32_t>(__ldg(lut + (w[j] & 0xFFFFu))) |
             (static_cast<uint32_t>(__ldg(lut + (w[j] >> 16))) << 16);
    v8[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (int64_t i = n8 * 8 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    v[i] = __ldg(lut + v[i]);
}

int launch_scores_from_logits(uint16_t* values, int64_t n, const uint16_t* lut, cudaStream_t stream) {
  if (n <= 0) return SPX_OK;
  if ((reinterpret_cast<uintptr_t>(values) & 15u) != 0) return SPX_ERR_ALIGNMENT;
  int64_t blocks = (n / 8 + 255) / 256;
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(device_sm_count()) * 8));
  scores_from_logits_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(values, n, lut);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

size_t route_select_smem(int E) {
  return static_cast<size_t>(kRouteRows) * route_row_words(E) * 4 + ((E + 3) / 4) * 4 + route_select_aux_bytes(E);
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
  return launch_pdl(route_rows_kernel<NCH, K1MAX>, dim3(route_lb_blocks(a.tokens)), dim3(kRouteWarps * 32),
                    route_rows_smem(a.num_experts), stream, a);
}

template <int NCH>
static int launch_route_rows_k(const RouteArgs& a, cudaStream_t stream) {
  if (a.top_k + 1 <= 5) return launch_route_rows_t<NCH, 5>(a, stream);
  if (a.top_k + 1 <= 9) return launch_route_rows_t<NCH, 9>(a, stream);
  return launch_route_rows_t<NCH, kMaxTopK + 1>(a, stream);
}

template <int K1MAX, bool MASK, bool NONNEG>
static int launch_route_select_t(const RouteArgs& a, int blocks, cudaStream_t stream) {
  const void* fn = reinterpret_cast<const void*>(route_select_kernel<K1MAX, MASK, NONNEG>);
  if (ensure_max_dynamic_smem(fn) != SPX_OK) return SPX_ERR_CUDA;
  route_select_kernel<K1MAX, MASK, NONNEG><<<blocks, 2 * kRouteRows, route_select_smem(a.num_experts), stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

template <bool MASK, bool NONNEG>
static int launch_route_select_k(const RouteArgs& a, int blocks, cudaStream_t stream) {
  if (a.top_k + 1 <= 5) return launch_route_select_t<5, MASK, NONNEG>(a, blocks, stream);
  if (a.top_k + 1 <= 9) return launch_route_select_t<9, MASK, NONNEG>(a, blocks, stream);
  return launch_route_select_t<kMaxTopK + 1, MASK, NONNEG>(a, blocks, stream);
}

int launch_route(const RouteArgs& a, cudaStream_t stream) {
  if (a.tokens <= 0) return SPX_OK;
  if (a.scores == nullptr && a.lut != nullptr) return SPX_ERR_INVALID_ARG;  // mapped scores must go somewhere
  if (a.tokens <= kRouteRowsMaxTokens) {
    const int nch = (a.num_experts + 255) / 256;
    if (nch <= 1) return launch_route_rows_k<1>(a, stream);
    if (nch <= 2) return launch_route_rows_k<2>(a, stream);
    return launch_route_rows_k<4>(a, stream);
  }
  const int blocks = static_cast<int>((a.tokens + kRouteRows - 1) / kRouteRows);
  // The softplus table only yields non-negative scores (and its one NaN).
  const bool nonneg = a.lut != nullptr;
  int rc;
  if (a.resident != nullptr)
    rc = nonneg ? launch_route_select_k<true, true>(a, blocks, stream) : launch_route_select_k<true, false>(a, blocks, stream);
  else
    rc = nonneg ? launch_route_select_k<false, true>(a, blocks, stream)
                : launch_route_select_k<false, false>(a, blocks, stream);
  if (rc != SPX_OK) return rc;
  const size_t tsmem = static_cast<size_t>(kTieWarps) * (a.num_experts + 2 * ((a.num_experts + 1) / 2)) * 4;
  const void* tfn = nonneg ? reinterpret_cast<const void*>(route_ties_kernel<true>)
                           : reinterpret_cast<const void*>(route_ties_kernel<false>);
  if (ensure_max_dynamic_smem(tfn) != SPX_OK) return SPX_ERR_CUDA;
  int tie_blocks = static_cast<int>((a.tokens + kTieWarps - 1) / kTieWarps);
  if (tie_blocks > a.sm_count * 8) tie_blocks = a.sm_count * 8;
  if (nonneg)
    route_ties_kernel<true><<<tie_blocks, kTieWarps * 32, tsmem, stream>>>(a);
  else
    route_ties_kernel<false><<<tie_blocks, kTieWarps * 32, tsmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
