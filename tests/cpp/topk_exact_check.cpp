// Host check of spalmer_b200/csrc/topk_exact.cuh against the GNU standard
// library algorithms PyTorch's CPU top-k runs (std::nth_element /
// std::partial_sort / std::sort with the "NaN last, value <" comparator).
//
// usage: topk_exact_check <rows_per_shape> <seed>
// Prints "OK <rows checked>" or the first mismatch and exits non-zero.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <utility>
#include <vector>

#include "../../spalmer_b200/csrc/topk_exact.cuh"

namespace {

using Elem = std::pair<float, int64_t>;

bool least_first(const Elem& x, const Elem& y) {
  return (!std::isnan(x.first) && std::isnan(y.first)) || (x.first < y.first);
}

uint16_t bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return static_cast<uint16_t>(u >> 16);  // inputs below are exact BF16 values
}

float from_bits(uint16_t b) {
  uint32_t u = static_cast<uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

}  // namespace

int main(int argc, char** argv) {
  const long rows = argc > 1 ? std::atol(argv[1]) : 20000;
  const unsigned seed = argc > 2 ? static_cast<unsigned>(std::atol(argv[2])) : 1u;
  std::mt19937_64 rng(seed);
  const int ns[] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 15, 16, 17, 18, 31, 33, 64, 100, 199, 200, 201, 256};
  long checked = 0;
  std::vector<Elem> q;
  std::vector<uint32_t> v;
  for (int n : ns) {
    for (int k = 1; k <= std::min(n, 20); ++k) {
      for (long r = 0; r < rows; ++r) {
        // Mix of value distributions: few levels (heavy ties), many levels,
        // negative values, occasional +inf (masked experts), NaN and signed
        // zeros.  Elements carry the order key of their BF16 bits.
        const int mode = static_cast<int>(rng() % 6);
        const int levels = mode == 0 ? 1 : mode == 1 ? 2 : mode == 2 ? 4 : mode == 3 ? 16 : 128;
        q.resize(n);
        v.resize(n);
        for (int j = 0; j < n; ++j) {
          float x = 0.25f * static_cast<float>(rng() % levels);
          if (mode == 4) x -= 16.0f;  // negative scores too (identity score transform)
          const unsigned sp = static_cast<unsigned>(rng() % 97);
          if (mode == 5 && sp == 0) x = NAN;
          if (mode == 5 && sp == 1) x = INFINITY;
          if (mode == 5 && sp == 2) x = -0.0f;
          const uint16_t b = std::isnan(x) ? uint16_t(0x7FC0) : bf16_bits(x);
          q[j] = Elem(from_bits(b), j);
          v[j] = spx::exact::make_elem(b, static_cast<uint32_t>(j));
        }
        if (k * 64 <= n) {
          std::partial_sort(q.begin(), q.begin() + k, q.end(), least_first);
        } else {
          std::nth_element(q.begin(), q.begin() + k - 1, q.end(), least_first);
          std::sort(q.begin(), q.begin() + k - 1, least_first);
        }
        spx::exact::topk_least_cpu_order(v.data(), n, k);
        for (int j = 0; j < k; ++j) {
          if (static_cast<int64_t>(v[j] & 0xFFFFu) != q[j].second) {
            std::printf("MISMATCH n=%d k=%d row=%ld slot=%d got=%u want=%lld\n", n, k, r, j,
                        v[j] & 0xFFFFu, static_cast<long long>(q[j].second));
            return 1;
          }
        }
        ++checked;
      }
    }
  }
  // The list form of the partition (parallelised on the device) must leave the
  // array and the cut exactly as the two-scanner form does.
  std::vector<uint32_t> a, b;
  std::vector<uint16_t> lpos, rpos;
  long parts = 0;
  for (int n : ns) {
    if (n < 4) continue;
    for (long r = 0; r < rows * 4; ++r) {
      const int levels = 1 + static_cast<int>(rng() % 8) * static_cast<int>(rng() % 20);
      a.resize(n);
      lpos.resize(n);
      rpos.resize(n);
      for (int j = 0; j < n; ++j) {
        float x = 0.25f * static_cast<float>(rng() % static_cast<unsigned>(levels));
        if (rng() % 211 == 0) x = NAN;
        const uint16_t bits = std::isnan(x) ? uint16_t(0x7FC0) : bf16_bits(x);
        a[j] = spx::exact::make_elem(bits, static_cast<uint32_t>(j));
      }
      const int lo = static_cast<int>(rng() % static_cast<unsigned>(n - 3));
      const int hi = lo + 4 + static_cast<int>(rng() % static_cast<unsigned>(n - lo - 3));
      b = a;
      const int c1 = spx::exact::partition_around_front(a.data(), lo, hi);
      const int c2 = spx::exact::partition_by_lists(b.data(), lo, hi, lpos.data(), rpos.data());
      if (c1 != c2 || a != b) {
        std::printf("PARTITION MISMATCH n=%d lo=%d hi=%d cut %d vs %d\n", n, lo, hi, c1, c2);
        return 1;
      }
      ++parts;
    }
  }
  std::printf("OK %ld rows, %ld partitions\n", checked, parts);
  return 0;
}
