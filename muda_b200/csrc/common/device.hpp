// device.hpp — small host-side helpers shared by the five libraries.
//
// The reference resolves every user pointer to (buffer, offset) and rejects a
// span that does not fit its allocation before it dispatches
// (libraries/common/src/metal_executor.mm:56-80).  On CUDA the equivalent check
// is cuMemGetAddressRange: a span that leaves its allocation, or a pointer the
// GPU cannot reach, is turned into an error status here instead of an illegal
// address on the device.
#pragma once

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <array>
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>

namespace mb200 {

inline int current_device() noexcept {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

// Streaming multiprocessor count of `dev`, cached (148 on a B200).
inline int sm_count(int dev) noexcept {
  static std::array<std::atomic<int>, 64> cache{};
  if (dev < 0 || dev >= 64) return 0;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

inline int max_smem_optin(int dev) noexcept {
  static std::array<std::atomic<int>, 64> cache{};
  if (dev < 0 || dev >= 64) return 0;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
      return 0;
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

inline AddressRangeFn address_range_fn() noexcept {
  static AddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<AddressRangeFn>(nullptr);
    return reinterpret_cast<AddressRangeFn>(p);
  }();
  return fn;
}

// True when [p, p + bytes) is memory the current device can address: one device
// or managed allocation that contains the whole span, or pinned host memory
// mapped into the device address space.  bytes == 0 always passes.
inline bool device_span_ok(const void* p, std::size_t bytes) noexcept {
  if (bytes == 0) return true;
  if (p == nullptr) return false;
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  if (attr.type == cudaMemoryTypeHost) return attr.devicePointer != nullptr;
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) return false;
  AddressRangeFn fn = address_range_fn();
  if (fn == nullptr) return true;  // no driver entry point: pointer kind already checked
  CUdeviceptr base = 0;
  size_t size = 0;
  const auto addr = static_cast<CUdeviceptr>(reinterpret_cast<std::uintptr_t>(p));
  if (fn(&base, &size, addr) != CUDA_SUCCESS) return false;
  return addr >= base && bytes <= size && addr - base <= size - bytes;
}

inline bool aligned_to(const void* p, std::size_t a) noexcept {
  return (reinterpret_cast<std::uintptr_t>(p) % a) == 0;
}

}  // namespace mb200
