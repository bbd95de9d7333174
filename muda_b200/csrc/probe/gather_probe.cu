// gather_probe.cu — the gather ceiling of a CSR SpMV, measured (benchmark tool).
//
// Not part of the drop-in API.  mb200ProbeGather streams an index array the way an
// SpMV streams its column indices (coalesced, evict-first) and gathers x[idx] the
// way it gathers the dense vector (L2-only loads), summing the gathered values so
// that nothing is optimised away, and nothing else: no values, no row structure,
// no output vector.  Run on a matrix's own column indices it gives the rate at
// which this GPU can serve that matrix's random x gathers, the ceiling against
// which an SpMV kernel's gather rate is judged.  mb200ProbeScatter does the same for
// the transposed product: it streams the indices and adds to y[idx] by reductions that
// return nothing, the scatter of A^T x without its loads of values and x; and
// mb200ProbeRowGather gathers whole 256-byte rows of a 64-column B per index, the
// gathers of an SpMM without its products.
//
// Layout: grid-stride over the indices; kPerLane consecutive indices per lane per
// step (one 16-byte load of four indices when kPerLane is 4), all gathers of a step
// issued before any is used.
#include <cuda_runtime.h>

#include <cstdint>

#pragma GCC visibility push(default)
#include "mb200_probe.h"
#pragma GCC visibility pop

namespace {

constexpr int kThreads = 256;

template <int kPerLane>
__global__ void __launch_bounds__(kThreads)
    gather_kernel(const float* __restrict__ x, const int* __restrict__ idx, long long n,
                  float* __restrict__ out) {
  const long long stride = static_cast<long long>(gridDim.x) * kThreads;
  long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x;
  float s = 0.0f;
  if constexpr (kPerLane == 4) {
    const int4* idx4 = reinterpret_cast<const int4*>(idx);
    const long long n4 = n / 4;
    for (; t < n4; t += stride) {
      const int4 c = __ldcs(idx4 + t);
      const float a = __ldcg(x + c.x), b = __ldcg(x + c.y), d = __ldcg(x + c.z),
                  e = __ldcg(x + c.w);
      s += (a + b) + (d + e);
    }
  } else {
    for (; t < n; t += stride) s += __ldcg(x + __ldcs(idx + t));
  }
  out[static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x] = s;
}

// The scatter of a transposed SpMV without its products: y[idx[i]] += 1 by a
// reduction that returns nothing (red.global.add.f32, resolved in L2).
template <int kPerLane>
__global__ void __launch_bounds__(kThreads)
    scatter_kernel(float* y, const int* __restrict__ idx, long long n) {
  const long long stride = static_cast<long long>(gridDim.x) * kThreads;
  long long t = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x;
  if constexpr (kPerLane == 4) {
    const int4* idx4 = reinterpret_cast<const int4*>(idx);
    const long long n4 = n / 4;
    for (; t < n4; t += stride) {
      const int4 c = __ldcs(idx4 + t);
      atomicAdd(y + c.x, 1.0f);
      atomicAdd(y + c.y, 1.0f);
      atomicAdd(y + c.z, 1.0f);
      atomicAdd(y + c.w, 1.0f);
    }
  } else {
    for (; t < n; t += stride) atomicAdd(y + __ldcs(idx + t), 1.0f);
  }
}

// The row gathers of an SpMM with a row-major B of 64 columns without its products:
// for each index, the 16 lanes of a group load the 16 float4 slices of row idx[i]
// (L2-only loads), four entries per group in flight, and sum them.
__global__ void __launch_bounds__(kThreads)
    row_gather_kernel(const float4* __restrict__ b, const int* __restrict__ idx, long long n,
                      float* __restrict__ out) {
  constexpr int G = 16, U = 4;
  const long long groups = static_cast<long long>(gridDim.x) * (kThreads / G);
  const long long grp = static_cast<long long>(blockIdx.x) * (kThreads / G) + threadIdx.x / G;
  const int lane = threadIdx.x % G;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (long long e = grp; e < n; e += U * groups) {
    int c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long t = e + u * groups;
      c[u] = t < n ? __ldcs(idx + t) : -1;
    }
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      v[u] = c[u] >= 0 ? __ldcg(b + static_cast<long long>(c[u]) * G + lane)
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      acc.x += v[u].x;
      acc.y += v[u].y;
      acc.z += v[u].z;
      acc.w += v[u].w;
    }
  }
  out[static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x] =
      (acc.x + acc.y) + (acc.z + acc.w);
}

}  // namespace

extern "C" int mb200ProbeRowGather(const float* b, const int* idx, long long n, float* out,
                                   unsigned grid, cudaStream_t stream) {
  if (b == nullptr || idx == nullptr || out == nullptr || n < 0 || grid == 0) return 1;
  if ((reinterpret_cast<std::uintptr_t>(b) & 15u) != 0) return 1;
  row_gather_kernel<<<grid, kThreads, 0, stream>>>(reinterpret_cast<const float4*>(b), idx, n,
                                                   out);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

extern "C" int mb200ProbeScatter(float* y, const int* idx, long long n, int per_lane,
                                 unsigned grid, cudaStream_t stream) {
  if (y == nullptr || idx == nullptr || n < 0 || grid == 0) return 1;
  if (per_lane == 4) {
    if ((reinterpret_cast<std::uintptr_t>(idx) & 15u) != 0) return 1;
    scatter_kernel<4><<<grid, kThreads, 0, stream>>>(y, idx, n);
  } else {
    scatter_kernel<1><<<grid, kThreads, 0, stream>>>(y, idx, n);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

extern "C" int mb200ProbeGather(const float* x, const int* idx, long long n, int per_lane,
                                float* out, unsigned grid, cudaStream_t stream) {
  if (x == nullptr || idx == nullptr || out == nullptr || n < 0 || grid == 0) return 1;
  if (per_lane == 4) {
    if ((reinterpret_cast<std::uintptr_t>(idx) & 15u) != 0) return 1;
    gather_kernel<4><<<grid, kThreads, 0, stream>>>(x, idx, n, out);
  } else {
    gather_kernel<1><<<grid, kThreads, 0, stream>>>(x, idx, n, out);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}
