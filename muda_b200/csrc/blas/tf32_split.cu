// tf32_split.cu — fp32 -> (hi, lo) tf32 plane kernels (HBM-bound, one pass).
#include "blas/tf32_split.hpp"

#include <cuda_runtime.h>

#include <cstdint>

#include "common/device.hpp"

namespace mb200::tc {
namespace {

__device__ __forceinline__ void split(float x, float& hi, float& lo) {
  tf32_split_value(x, hi, lo);
}

constexpr int kTile = 32;
constexpr int kRowsPerPass = 8;

// One 32 x 32 tile (32 k by 32 rows) of job j, staged in shared memory so both
// the contiguous read (along k or along rows) and the k-contiguous write coalesce.
__device__ __forceinline__ void split_tile(const SplitJob& j, long long z, long long r0,
                                           long long k0, float (*tile)[kTile + 1]) {
  const int tx = threadIdx.x, ty = threadIdx.y;
  const bool kcontig = j.ks == 1;
  const float* sz = j.src + z * j.zs;
#pragma unroll
  for (int i = 0; i < kTile / kRowsPerPass; ++i) {
    const int a = ty + i * kRowsPerPass;  // the non-contiguous index of the tile
    const long long r = kcontig ? r0 + a : r0 + tx;
    const long long k = kcontig ? k0 + tx : k0 + a;
    float v = 0.0f;
    if (r < j.rows && k < j.cols) v = sz[r * j.rs + k * j.ks];
    if (kcontig)
      tile[a][tx] = v;
    else
      tile[tx][a] = v;
  }
  __syncthreads();
  const long long plane = static_cast<long long>(j.batch) * j.rows * j.ldk;
  float* dz = j.dst + z * j.rows * j.ldk;
#pragma unroll
  for (int i = 0; i < kTile / kRowsPerPass; ++i) {
    const int a = ty + i * kRowsPerPass;
    const long long r = r0 + a, k = k0 + tx;
    if (r < j.rows && k < j.cols) {
      float hi, lo;
      split(tile[a][tx], hi, lo);
      dz[r * j.ldk + k] = hi;
      dz[plane + r * j.ldk + k] = lo;
    }
  }
  __syncthreads();
}

// A job whose k is contiguous and whose rows, planes and pointers keep 16-byte
// alignment needs no transpose: each thread splits four consecutive k of a row
// (one 16-byte load, two 16-byte stores).
__host__ __device__ inline bool streaming(const SplitJob& j) {
  return j.ks == 1 && j.cols % 4 == 0 && j.rs % 4 == 0 && j.zs % 4 == 0 && j.ldk % 4 == 0 &&
         reinterpret_cast<std::uintptr_t>(j.src) % 16 == 0 &&
         reinterpret_cast<std::uintptr_t>(j.dst) % 16 == 0;
}

__device__ void split_stream(const SplitJob& j) {
  const long long k4 = j.cols / 4;
  const long long per_z = j.rows * k4;
  const long long total = per_z * j.batch;
  const long long plane = static_cast<long long>(j.batch) * j.rows * j.ldk;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * blockDim.y;
  for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x * blockDim.y +
                     threadIdx.y * blockDim.x + threadIdx.x;
       t < total; t += stride) {
    const long long z = t / per_z, rem = t - z * per_z;
    const long long r = rem / k4, k = (rem - r * k4) * 4;
    const float4 v = __ldg(reinterpret_cast<const float4*>(j.src + z * j.zs + r * j.rs + k));
    float4 hi, lo;
    split(v.x, hi.x, lo.x);
    split(v.y, hi.y, lo.y);
    split(v.z, hi.z, lo.z);
    split(v.w, hi.w, lo.w);
    float* d = j.dst + (z * j.rows + r) * j.ldk + k;
    *reinterpret_cast<float4*>(d) = hi;
    *reinterpret_cast<float4*>(d + plane) = lo;
  }
}

// Blocks stride over the tiles of job blockIdx.y (0 or 1; one job when y == 1).
__global__ void __launch_bounds__(kTile* kRowsPerPass)
    split_jobs(const SplitJob j0, const SplitJob j1) {
  __shared__ float tile[kTile][kTile + 1];  // [row][k]
  const SplitJob& j = blockIdx.y == 0 ? j0 : j1;
  if (streaming(j)) {
    split_stream(j);
    return;
  }
  const long long tiles_k = (j.cols + kTile - 1) / kTile;
  const long long tiles_r = (j.rows + kTile - 1) / kTile;
  const long long per = tiles_k * tiles_r;
  const long long total = per * j.batch;
  for (long long t = blockIdx.x; t < total; t += gridDim.x) {
    const long long z = t / per, rt = t % per;
    split_tile(j, z, (rt / tiles_k) * kTile, (rt % tiles_k) * kTile, tile);
  }
}

__global__ void split_filter(const float* __restrict__ w, int K, int C, int R, int S, int krsc,
                             float* __restrict__ dst) {
  const long long rsc = static_cast<long long>(R) * S * C;
  const long long total = rsc * K;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long k = i / rsc;
    const int j = static_cast<int>(i % rsc);  // (r*S + s)*C + c
    const int c = j % C;
    const int rs = j / C;
    const long long from = krsc ? i : (k * C + c) * R * S + rs;
    float hi, lo;
    split(w[from], hi, lo);
    dst[i] = hi;
    dst[total + i] = lo;
  }
}

}  // namespace

namespace {

unsigned split_grid(const SplitJob& a, const SplitJob* b) {
  auto tiles = [](const SplitJob& j) {
    if (streaming(j))  // CTAs of kTile * kRowsPerPass threads, one 4-float group each
      return (j.rows * (j.cols / 4) * j.batch + kTile * kRowsPerPass - 1) / (kTile * kRowsPerPass);
    return ((j.cols + kTile - 1) / kTile) * ((j.rows + kTile - 1) / kTile) * j.batch;
  };
  long long t = tiles(a);
  if (b != nullptr && tiles(*b) > t) t = tiles(*b);
  const int sms = sm_count(current_device());
  const long long cap = static_cast<long long>(sms > 0 ? sms : 148) * 8;
  return static_cast<unsigned>(t < 1 ? 1 : (t < cap ? t : cap));
}

}  // namespace

cudaError_t launch_tf32_split(const float* src, long long rows, long long cols, int batch,
                              long long rs, long long ks, long long zs, float* dst,
                              long long ldk, cudaStream_t stream) noexcept {
  if (rows <= 0 || cols <= 0 || batch <= 0) return cudaSuccess;
  const SplitJob j{src, rows, cols, batch, rs, ks, zs, dst, ldk};
  split_jobs<<<dim3(split_grid(j, nullptr), 1), dim3(kTile, kRowsPerPass), 0, stream>>>(j, j);
  return cudaGetLastError();
}

cudaError_t launch_tf32_split_pair(const SplitJob& a, const SplitJob& b,
                                   cudaStream_t stream) noexcept {
  if (a.rows <= 0 || a.cols <= 0 || a.batch <= 0 || b.rows <= 0 || b.cols <= 0 || b.batch <= 0)
    return cudaErrorInvalidValue;
  split_jobs<<<dim3(split_grid(a, &b), 2), dim3(kTile, kRowsPerPass), 0, stream>>>(a, b);
  return cudaGetLastError();
}

cudaError_t launch_tf32_split_filter(const float* w, int K, int C, int R, int S, bool krsc,
                                     float* dst, cudaStream_t stream) noexcept {
  const long long total = static_cast<long long>(K) * C * R * S;
  if (total <= 0) return cudaSuccess;
  const long long want = (total + 255) / 256;
  split_filter<<<static_cast<unsigned>(want < 4096 ? want : 4096), 256, 0, stream>>>(
      w, K, C, R, S, krsc ? 1 : 0, dst);
  return cudaGetLastError();
}

}  // namespace mb200::tc
