// tf32_split.cu — fp32 -> (hi, lo) tf32 plane kernels (HBM-bound, one pass).
#include "blas/tf32_split.hpp"

#include <cuda_runtime.h>

namespace mb200::tc {
namespace {

__device__ __forceinline__ void split(float x, float& hi, float& lo) {
  const unsigned b = __float_as_uint(x);
  if ((b & 0x7F800000u) == 0x7F800000u) {  // inf / nan: both planes carry x
    hi = x;
    lo = x;
    return;
  }
  hi = __uint_as_float(b & 0xFFFFE000u);  // toward zero: lo keeps the sign of x
  float r = __fsub_rn(x, hi);              // exact
  if (r == 0.0f) r = __fmul_rn(x, 0x1p-40f);
  unsigned t;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(r));
  lo = __uint_as_float(t);
}

constexpr int kTile = 32;
constexpr int kRowsPerPass = 8;

// One 32 x 32 tile (32 k by 32 rows) per block of 32 x 8 threads, staged in
// shared memory so both the contiguous read and the k-contiguous write coalesce.
template <bool KContig>
__global__ void __launch_bounds__(kTile* kRowsPerPass)
    split_tiles(const float* __restrict__ src, long long rows, long long cols, int batch,
                long long rs, long long ks, long long zs, float* __restrict__ dst, long long ldk) {
  __shared__ float tile[kTile][kTile + 1];  // [row][k]
  const long long tiles_k = (cols + kTile - 1) / kTile;
  const long long tiles_r = (rows + kTile - 1) / kTile;
  const long long plane = static_cast<long long>(batch) * rows * ldk;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (long long z = blockIdx.z; z < batch; z += gridDim.z) {
    const float* sz = src + z * zs;
    float* dz = dst + z * rows * ldk;
    for (long long tr = blockIdx.y; tr < tiles_r; tr += gridDim.y) {
      for (long long tk = blockIdx.x; tk < tiles_k; tk += gridDim.x) {
        const long long r0 = tr * kTile, k0 = tk * kTile;
#pragma unroll
        for (int i = 0; i < kTile / kRowsPerPass; ++i) {
          const int a = ty + i * kRowsPerPass;  // the non-contiguous index of the tile
          const long long r = KContig ? r0 + a : r0 + tx;
          const long long k = KContig ? k0 + tx : k0 + a;
          float v = 0.0f;
          if (r < rows && k < cols) v = sz[r * rs + k * ks];
          if (KContig)
            tile[a][tx] = v;
          else
            tile[tx][a] = v;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kTile / kRowsPerPass; ++i) {
          const int a = ty + i * kRowsPerPass;
          const long long r = r0 + a, k = k0 + tx;
          if (r < rows && k < cols) {
            float hi, lo;
            split(tile[a][tx], hi, lo);
            dz[r * ldk + k] = hi;
            dz[plane + r * ldk + k] = lo;
          }
        }
        __syncthreads();
      }
    }
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

cudaError_t launch_tf32_split(const float* src, long long rows, long long cols, int batch,
                              long long rs, long long ks, long long zs, float* dst,
                              long long ldk, cudaStream_t stream) noexcept {
  if (rows <= 0 || cols <= 0 || batch <= 0) return cudaSuccess;
  const long long tiles_k = (cols + kTile - 1) / kTile;
  const long long tiles_r = (rows + kTile - 1) / kTile;
  const dim3 grid(static_cast<unsigned>(tiles_k < 1024 ? tiles_k : 1024),
                  static_cast<unsigned>(tiles_r < 65535 ? tiles_r : 65535),
                  static_cast<unsigned>(batch < 65535 ? batch : 65535));
  const dim3 block(kTile, kRowsPerPass);
  if (ks == 1)
    split_tiles<true><<<grid, block, 0, stream>>>(src, rows, cols, batch, rs, ks, zs, dst, ldk);
  else
    split_tiles<false><<<grid, block, 0, stream>>>(src, rows, cols, batch, rs, ks, zs, dst, ldk);
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
