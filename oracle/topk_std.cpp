// CPU oracle for the reference's least-surprise top-k (TEST INFRASTRUCTURE ONLY).
//
// The reference selects experts with `eligible.topk(k, dim=-1, largest=False)`
// (mESmaC/spalmer src/spalmer/experts/router.py:92).  On CPU PyTorch runs
// ATen/native/TopKImpl.h:44-89 (torch 2.11.0): every row becomes a vector of
// (float value, int64 index) pairs; when k*64 <= n it calls std::partial_sort
// over the first k, otherwise std::nth_element at k-1 followed by std::sort of
// the first k-1 entries.  The comparator orders NaN last and is otherwise
// `a < b` on the float value (indices never take part), so the order of equal
// values is whatever those standard algorithms leave behind.  This file simply
// calls the same standard-library algorithms with the same comparator; it is
// the definition of the tie order that the GPU kernels must reproduce.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <utility>
#include <vector>

namespace {

using Elem = std::pair<float, int64_t>;

inline bool least_first(const Elem& x, const Elem& y) {
  return (!std::isnan(x.first) && std::isnan(y.first)) || (x.first < y.first);
}

void select_row(const float* row, int64_t n, int64_t k, std::vector<Elem>& q,
                int64_t* out) {
  for (int64_t j = 0; j < n; ++j) q[j] = Elem(row[j], j);
  if (k * 64 <= n) {
    std::partial_sort(q.begin(), q.begin() + k, q.end(), least_first);
  } else {
    std::nth_element(q.begin(), q.begin() + k - 1, q.end(), least_first);
    std::sort(q.begin(), q.begin() + k - 1, least_first);
  }
  for (int64_t j = 0; j < k; ++j) out[j] = q[j].second;
}

}  // namespace

extern "C" int oracle_topk_least(const float* scores, int64_t rows, int64_t n,
                                 int64_t k, int64_t* out_idx) {
  if (rows < 0 || n < 1 || k < 1 || k > n) return -1;
#pragma omp parallel
  {
    std::vector<Elem> q(n);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) select_row(scores + r * n, n, k, q, out_idx + r * k);
  }
  return 0;
}
