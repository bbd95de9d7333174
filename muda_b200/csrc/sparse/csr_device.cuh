// csr_device.cuh — device helpers shared by the CSR kernels: clamped row
// offsets and fp16 <-> fp32 conversion of values.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mb200::sparse {
namespace {

__device__ __forceinline__ int clamp_off(std::int32_t v, int base, std::int64_t nnz) {
  const std::int64_t t = static_cast<std::int64_t>(v) - base;
  return static_cast<int>(t < 0 ? 0 : (t > nnz ? nnz : t));
}

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(__half v) { return __half2float(v); }
template <class T>
__device__ __forceinline__ T narrow(float v);
template <>
__device__ __forceinline__ float narrow<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half narrow<__half>(float v) {
  return __float2half_rn(v);
}

}  // namespace
}  // namespace mb200::sparse
