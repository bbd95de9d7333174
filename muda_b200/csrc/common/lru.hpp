// lru.hpp — bounded least-recently-used cache shared by plans.
//
// The reference keeps per-configuration GEMM and FFT resources in bounded LRU
// caches (libraries/common/include/muda/libraries/plan_cache.hpp:31-87: 256
// GEMM entries, 128 FFT entries).  Here the cached values are device resources
// (twiddle tables, TMA descriptors) held by shared_ptr, so an evicted entry stays
// alive until the last plan that uses it is destroyed.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <list>
#include <map>
#include <memory>
#include <mutex>
#include <utility>

namespace mb200 {

template <typename Key, typename Value>
class LruCache {
 public:
  explicit LruCache(std::size_t capacity) : capacity_(capacity ? capacity : 1) {}

  std::shared_ptr<Value> find(const Key& k) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = index_.find(k);
    if (it == index_.end()) return nullptr;
    order_.splice(order_.begin(), order_, it->second);
    return it->second->second;
  }

  void put(const Key& k, std::shared_ptr<Value> v) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = index_.find(k);
    if (it != index_.end()) {
      it->second->second = std::move(v);
      order_.splice(order_.begin(), order_, it->second);
      return;
    }
    order_.emplace_front(k, std::move(v));
    index_[k] = order_.begin();
    while (order_.size() > capacity_) {
      index_.erase(order_.back().first);
      order_.pop_back();
    }
  }

  std::size_t size() const {
    std::lock_guard<std::mutex> g(mu_);
    return order_.size();
  }

 private:
  using Item = std::pair<Key, std::shared_ptr<Value>>;
  std::size_t capacity_;
  mutable std::mutex mu_;
  std::list<Item> order_;
  std::map<Key, typename std::list<Item>::iterator> index_;
};

// Device allocation owned by a shared_ptr; freed on the device it came from.
struct DeviceBuffer {
  void* ptr = nullptr;
  std::size_t bytes = 0;
  int device = -1;
  DeviceBuffer() = default;
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  ~DeviceBuffer() {
    if (ptr == nullptr) return;
    int prev = -1;
    (void)cudaGetDevice(&prev);
    if (device >= 0 && device != prev) (void)cudaSetDevice(device);
    (void)cudaFree(ptr);
    if (device >= 0 && device != prev && prev >= 0) (void)cudaSetDevice(prev);
  }

  // Allocates `bytes` on the current device; null on failure.
  static std::shared_ptr<DeviceBuffer> make(std::size_t bytes) {
    auto b = std::make_shared<DeviceBuffer>();
    if (cudaGetDevice(&b->device) != cudaSuccess) return nullptr;
    if (cudaMalloc(&b->ptr, bytes ? bytes : 1) != cudaSuccess) {
      (void)cudaGetLastError();
      b->ptr = nullptr;
      return nullptr;
    }
    b->bytes = bytes;
    return b;
  }
};

}  // namespace mb200
