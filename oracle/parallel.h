// parallel.h — splits an index range across std::threads (test infrastructure only).
//
// The oracle's multi-core CPU baseline runs the same per-index code as the
// single-threaded restatement; each thread takes one contiguous chunk.
#pragma once

#include <algorithm>
#include <cstdint>
#include <thread>
#include <vector>

namespace oracle_detail {

template <typename Fn>
void parallel_for(std::int64_t begin, std::int64_t end, int threads, Fn&& fn) {
  const std::int64_t total = end - begin;
  if (total <= 0) return;
  int t = threads > 0 ? threads : 1;
  if (t > total) t = static_cast<int>(total);
  if (t == 1) {
    for (std::int64_t i = begin; i < end; ++i) fn(i);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(static_cast<std::size_t>(t));
  const std::int64_t chunk = (total + t - 1) / t;
  for (int w = 0; w < t; ++w) {
    const std::int64_t lo = begin + w * chunk;
    const std::int64_t hi = std::min(end, lo + chunk);
    if (lo >= hi) break;
    pool.emplace_back([lo, hi, &fn] {
      for (std::int64_t i = lo; i < hi; ++i) fn(i);
    });
  }
  for (auto& th : pool) th.join();
}

}  // namespace oracle_detail
