// Exact restatement of the CPU top-k tie order, usable on host and device.
//
// The reference routes with `scores.topk(k, largest=False)`
// (mESmaC/spalmer src/spalmer/experts/router.py:92).  On CPU PyTorch
// (ATen/native/TopKImpl.h:44-89) sorts (float value, index) pairs with the
// comparator "NaN last, otherwise value <": `partial_sort` of the first k when
// k*64 <= n, otherwise `nth_element` at k-1 followed by `sort` of the first k-1.
// Equal values therefore come out in the order the GNU libstdc++ algorithms
// leave them.  Rows whose k+1 smallest values are all distinct have a unique
// answer and never reach this file; rows with ties are replayed here step by
// step so the indices match bit for bit.
//
// The algorithms are written from their published descriptions:
//   * introselect (Musser 1997): quickselect with a depth limit of
//     2*floor(log2 n) partitions, falling back to heap selection; ranges of
//     at most 3 elements finish with straight insertion sort;
//   * the partition step: median of {second, middle, last} moved to the
//     front as the pivot, then Hoare's two-pointer partition of the rest,
//     both scanners stopping on elements equal to the pivot;
//   * introsort (Musser 1997): the same partition while a range exceeds 16
//     elements (heapsort past the depth limit), then insertion sort;
//   * binary max-heaps with Floyd's sift (move the hole to a leaf along the
//     larger child, then sift the saved value back up).
// tests/test_topk_exact_host.py compiles this header with g++ and checks it
// against std::nth_element / std::partial_sort / std::sort on millions of
// tie-heavy rows.
//
// Elements are 32-bit words: bits [31:16] hold the BF16 score as an order
// key (order_key16), bits [15:0] the expert index.  Only the key takes part in
// comparisons, as one unsigned compare: the key maps the comparator "NaN
// last, otherwise value <" onto integer order (-0 and +0 share a key, every
// NaN gets the largest key, so NaNs compare equal to each other, as they do
// under that comparator).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define SPX_HD __host__ __device__ __forceinline__
#else
#define SPX_HD inline
#endif

namespace spx {
namespace exact {

SPX_HD uint32_t order_key16(uint16_t b) {
  if ((b & 0x7F80u) == 0x7F80u && (b & 0x007Fu) != 0u) return 0xFFFFu;  // NaN
  if (b == 0x8000u) b = 0;                                               // -0 -> +0
  return (b & 0x8000u) ? (~static_cast<uint32_t>(b) & 0xFFFFu) : (static_cast<uint32_t>(b) | 0x8000u);
}

// BF16 bits back from an order key (+0 for the zero key, a NaN for the NaN key).
SPX_HD uint16_t key16_to_bits(uint32_t key) {
  return (key & 0x8000u) ? static_cast<uint16_t>(key & 0x7FFFu) : static_cast<uint16_t>(~key & 0xFFFFu);
}

// The element of score bits `b` at index `idx`.
SPX_HD uint32_t make_elem(uint16_t b, uint32_t idx) { return (order_key16(b) << 16) | idx; }

// "a before b": a's score comes strictly first.
SPX_HD bool before(uint32_t a, uint32_t b) { return (a >> 16) < (b >> 16); }

SPX_HD void swap_at(uint32_t* v, int i, int j) {
  const uint32_t t = v[i];
  v[i] = v[j];
  v[j] = t;
}

SPX_HD int floor_log2(int n) {
  int r = 0;
  while (n > 1) {
    n >>= 1;
    ++r;
  }
  return r;
}

// Shift v[pos] left past every element it precedes.  Needs a sentinel: some
// element to the left must not come after v[pos].
SPX_HD void linear_insert_unguarded(uint32_t* v, int pos) {
  const uint32_t x = v[pos];
  int j = pos;
  while (before(x, v[j - 1])) {
    v[j] = v[j - 1];
    --j;
  }
  v[j] = x;
}

// Straight insertion sort of v[lo, hi): an element that precedes the current
// front is moved there directly, others are inserted without a bound check.
SPX_HD void insertion_sort(uint32_t* v, int lo, int hi) {
  if (lo == hi) return;
  for (int i = lo + 1; i < hi; ++i) {
    if (before(v[i], v[lo])) {
      const uint32_t x = v[i];
      for (int j = i; j > lo; --j) v[j] = v[j - 1];
      v[lo] = x;
    } else {
      linear_insert_unguarded(v, i);
    }
  }
}

// Move the median of v[a], v[b], v[c] into slot r.
SPX_HD void median_to_slot(uint32_t* v, int r, int a, int b, int c) {
  if (before(v[a], v[b])) {
    if (before(v[b], v[c]))
      swap_at(v, r, b);
    else if (before(v[a], v[c]))
      swap_at(v, r, c);
    else
      swap_at(v, r, a);
  } else if (before(v[a], v[c])) {
    swap_at(v, r, a);
  } else if (before(v[b], v[c])) {
    swap_at(v, r, c);
  } else {
    swap_at(v, r, b);
  }
}

// Hoare partition of v[lo+1, hi) around the pivot held at v[lo]; returns the
// first index of the upper part.  The pivot slot bounds the right scanner and
// the median-of-three guarantees an element that stops the left scanner.
SPX_HD int partition_around_front(uint32_t* v, int lo, int hi) {
  const int mid = lo + (hi - lo) / 2;
  median_to_slot(v, lo, lo + 1, mid, hi - 1);
  const uint32_t pivot = v[lo];
  int left = lo + 1;
  int right = hi;
  while (true) {
    while (before(v[left], pivot)) ++left;
    --right;
    while (before(pivot, v[right])) --right;
    if (!(left < right)) return left;
    swap_at(v, left, right);
    ++left;
  }
}

// The same partition computed from two position lists instead of two moving
// scanners, which makes it data-parallel (route.cu runs it with one warp per
// row).  With the pivot at v[lo]:
//   Lo = positions in (lo, hi) holding an element not before the pivot, ascending
//   Ro = positions in [lo, hi) holding an element the pivot is not before, descending
// Before any swap the scanners see original values only, and a swap at step m
// exchanges v[Lo[m]] and v[Ro[m]] while Lo[m] < Ro[m].  The first m with
// Lo[m] >= Ro[m] (Lo past its end counts as +inf, Ro past its end as -inf)
// ends the loop, and the left scanner then rests at Lo[m], or at the swapped
// slot Ro[m-1] if that comes first.  `lpos`/`rpos` are caller scratch of n
// entries; Ro[m] is stored as rpos[nR-1-m] (ascending).
SPX_HD int partition_by_lists(uint32_t* v, int lo, int hi, uint16_t* lpos, uint16_t* rpos) {
  const int mid = lo + (hi - lo) / 2;
  median_to_slot(v, lo, lo + 1, mid, hi - 1);
  const uint32_t pivot = v[lo];
  int nl = 0, nr = 0;
  for (int p = lo; p < hi; ++p) {
    if (p > lo && !before(v[p], pivot)) lpos[nl++] = static_cast<uint16_t>(p);
    if (!before(pivot, v[p])) rpos[nr++] = static_cast<uint16_t>(p);
  }
  int m = 0;
  while (m < nl && m < nr && lpos[m] < rpos[nr - 1 - m]) ++m;
  for (int q = 0; q < m; ++q) swap_at(v, lpos[q], rpos[nr - 1 - q]);
  if (m == 0) return lpos[0];
  const int left = m < nl ? lpos[m] : hi;
  const int right_prev = rpos[nr - m];
  return left < right_prev ? left : right_prev;
}

// ---- binary max-heap on base[0, len) ordered by `before`.
SPX_HD void heap_sift_up(uint32_t* base, int hole, int top, uint32_t x) {
  int parent = (hole - 1) / 2;
  while (hole > top && before(base[parent], x)) {
    base[hole] = base[parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  base[hole] = x;
}

// Floyd's sift: drive the hole at `hole` down to a leaf along the larger
// child, then place x by sifting it back up (never above `hole`).
SPX_HD void heap_fill_hole(uint32_t* base, int hole, int len, uint32_t x) {
  const int top = hole;
  int child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (before(base[child], base[child - 1])) --child;
    base[hole] = base[child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    base[hole] = base[child - 1];
    hole = child - 1;
  }
  heap_sift_up(base, hole, top, x);
}

SPX_HD void heap_build(uint32_t* base, int len) {
  if (len < 2) return;
  for (int parent = (len - 2) / 2;; --parent) {
    heap_fill_hole(base, parent, len, base[parent]);
    if (parent == 0) return;
  }
}

// Replace the heap top (base[0, len)) by the value at `slot`, which receives the old top.
SPX_HD void heap_pop_into(uint32_t* base, int len, uint32_t* slot) {
  const uint32_t x = *slot;
  *slot = base[0];
  heap_fill_hole(base, 0, len, x);
}

// Keep in v[lo, mid) the (mid-lo) elements that come first; v[lo] ends up
// holding the last of them (heap top).
SPX_HD void heap_select(uint32_t* v, int lo, int mid, int hi) {
  heap_build(v + lo, mid - lo);
  for (int i = mid; i < hi; ++i)
    if (before(v[i], v[lo])) heap_pop_into(v + lo, mid - lo, v + i);
}

SPX_HD void heap_sort_range(uint32_t* v, int lo, int hi) {
  while (hi - lo > 1) {
    --hi;
    heap_pop_into(v + lo, hi - lo, v + hi);
  }
}

// partial_sort(first, first + mid, first + n)
SPX_HD void partial_sort_first(uint32_t* v, int mid, int n) {
  heap_select(v, 0, mid, n);
  heap_sort_range(v, 0, mid);
}

// nth_element(first, first + nth, first + n): introselect.
SPX_HD void select_nth(uint32_t* v, int nth, int n) {
  if (n == 0 || nth == n) return;
  int lo = 0, hi = n;
  int depth = 2 * floor_log2(n);
  while (hi - lo > 3) {
    if (depth == 0) {
      heap_select(v, lo, nth + 1, hi);
      swap_at(v, lo, nth);
      return;
    }
    --depth;
    const int cut = partition_around_front(v, lo, hi);
    if (cut <= nth)
      lo = cut;
    else
      hi = cut;
  }
  insertion_sort(v, lo, hi);
}

// sort(first, first + n): introsort, ranges > 16 partitioned (upper part
// first, iterating on the lower part), heapsort past the depth limit, then a
// final insertion sort (unguarded beyond the first 16 elements).
SPX_HD void intro_sort(uint32_t* v, int n) {
  if (n < 2) return;
  constexpr int kThreshold = 16;
  // Explicit stack of pending (lo, hi, depth) ranges; depth <= 2*log2(n).
  int st_lo[64], st_hi[64], st_depth[64];
  int sp = 0;
  st_lo[sp] = 0;
  st_hi[sp] = n;
  st_depth[sp] = 2 * floor_log2(n);
  ++sp;
  while (sp > 0) {
    --sp;
    int lo = st_lo[sp], hi = st_hi[sp], depth = st_depth[sp];
    while (hi - lo > kThreshold) {
      if (depth == 0) {
        heap_select(v, lo, hi, hi);
        heap_sort_range(v, lo, hi);
        break;
      }
      --depth;
      const int cut = partition_around_front(v, lo, hi);
      // Both halves inherit the decremented depth.  They are disjoint, so the
      // order in which they are finished does not change the result; the
      // lower half waits on the stack while the loop continues on the upper.
      st_lo[sp] = lo;
      st_hi[sp] = cut;
      st_depth[sp] = depth;
      ++sp;
      lo = cut;
    }
  }
  if (n > kThreshold) {
    insertion_sort(v, 0, kThreshold);
    for (int i = kThreshold; i < n; ++i) linear_insert_unguarded(v, i);
  } else {
    insertion_sort(v, 0, n);
  }
}

// The full CPU top-k ordering: v[0, n) holds the row, the first k entries
// receive the selection in PyTorch's order.
SPX_HD void topk_least_cpu_order(uint32_t* v, int n, int k) {
  if (k * 64 <= n) {
    partial_sort_first(v, k, n);
  } else {
    select_nth(v, k - 1, n);
    intro_sort(v, k - 1);
  }
}

}  // namespace exact
}  // namespace spx
