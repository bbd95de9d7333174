// softmax_kernels.cu — softmax forward for sm_100a.
//
// Semantics follow the reference kernels (libraries/dnn/shaders/cudnn_kernels.metal):
//   ACCURATE: m = max(x);  FAST: m = 0;  LOG: m = max(x)
//   s = sum exp(x - m)
//   val = LOG ? (x - m) - log(s) : exp(x - m) * (1/s)
//   y = fma(alpha, val, beta == 0 ? 0 : beta * y)
// (warp kernel cudnn_kernels.metal:529-568, generic kernel :447-527).
//
// The reference's contiguous path reads each row three times (max, sum, write).
// Here a row is read from HBM once into registers, reduced twice on chip, and
// written once: 8 bytes of HBM traffic per element (12 with beta != 0).
//   rows of <= 1024 floats: one warp per row, 8 rows per CTA;
//   rows of <= 8192 floats: one 256-thread CTA per row, 16-byte loads when aligned;
//   longer rows: one CTA per row with an online (max, sum) pass and a write pass.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "common/device.hpp"
#include "dnn/dnn.hpp"

namespace mb200::dnn {
namespace {

constexpr int kBlock = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reduction through shared memory; every thread receives the result.
template <bool IsMax>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  v = IsMax ? warp_max(v) : warp_sum(v);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (kBlock / 32) ? red[lane] : (IsMax ? -FLT_MAX : 0.0f);
    t = IsMax ? warp_max(t) : warp_sum(t);
    if (lane == 0) red[kBlock / 32] = t;
  }
  __syncthreads();
  const float r = red[kBlock / 32];
  __syncthreads();  // red[] is reused by the next reduction
  return r;
}

__device__ __forceinline__ float finish(float xv, float m, float inv_or_logsum, SoftmaxAlgo a,
                                        float alpha, float beta, const float* yp) {
  const float sh = xv - m;
  const float val = (a == SoftmaxAlgo::kLog) ? (sh - inv_or_logsum) : (expf(sh) * inv_or_logsum);
  const float prev = (beta == 0.0f) ? 0.0f : beta * *yp;
  return fmaf(alpha, val, prev);
}

// ---- one warp per row, ITEMS elements per lane (lane-strided, coalesced)
template <int ITEMS>
__global__ void __launch_bounds__(kBlock) softmax_warp_rows(const float* __restrict__ x,
                                                            float* __restrict__ y,
                                                            std::int64_t rows, int len,
                                                            SoftmaxAlgo algo, float alpha,
                                                            float beta) {
  const int lane = threadIdx.x & 31;
  const std::int64_t warps = static_cast<std::int64_t>(gridDim.x) * (kBlock / 32);
  for (std::int64_t row = static_cast<std::int64_t>(blockIdx.x) * (kBlock / 32) + (threadIdx.x >> 5);
       row < rows; row += warps) {
    const float* xr = x + row * len;
    float* yr = y + row * len;
    float v[ITEMS];
    float m = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int idx = i * 32 + lane;
      v[i] = idx < len ? xr[idx] : -FLT_MAX;
      m = fmaxf(m, v[i]);
    }
    m = (algo == SoftmaxAlgo::kFast) ? 0.0f : warp_max(m);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int idx = i * 32 + lane;
      if (idx < len) s += expf(v[i] - m);
    }
    s = warp_sum(s);
    const float k = (algo == SoftmaxAlgo::kLog) ? logf(s) : 1.0f / s;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int idx = i * 32 + lane;
      if (idx < len) yr[idx] = finish(v[i], m, k, algo, alpha, beta, yr + idx);
    }
  }
}

// ---- one CTA per row held in registers; VEC = 4 uses 16-byte accesses
template <int VEC, int ITEMS>
__global__ void __launch_bounds__(kBlock) softmax_block_rows(const float* __restrict__ x,
                                                             float* __restrict__ y,
                                                             std::int64_t rows, int len,
                                                             SoftmaxAlgo algo, float alpha,
                                                             float beta) {
  __shared__ float red[kBlock / 32 + 1];
  const int nvec = len / VEC;
  for (std::int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * len;
    float* yr = y + row * len;
    float v[ITEMS][VEC];
    float m = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int idx = i * kBlock + threadIdx.x;
      if constexpr (VEC == 4) {
        float4 t = idx < nvec ? reinterpret_cast<const float4*>(xr)[idx]
                              : make_float4(-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX);
        v[i][0] = t.x;
        v[i][1] = t.y;
        v[i][2] = t.z;
        v[i][3] = t.w;
      } else {
        v[i][0] = idx < nvec ? xr[idx] : -FLT_MAX;
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) m = fmaxf(m, v[i][j]);
    }
    m = (algo == SoftmaxAlgo::kFast) ? 0.0f : block_reduce<true>(m, red);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int idx = i * kBlock + threadIdx.x;
      if (idx < nvec) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) s += expf(v[i][j] - m);
      }
    }
    s = block_reduce<false>(s, red);
    const float k = (algo == SoftmaxAlgo::kLog) ? logf(s) : 1.0f / s;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int idx = i * kBlock + threadIdx.x;
      if (idx < nvec) {
        if constexpr (VEC == 4) {
          float4 o;
          o.x = finish(v[i][0], m, k, algo, alpha, beta, yr + 4 * idx + 0);
          o.y = finish(v[i][1], m, k, algo, alpha, beta, yr + 4 * idx + 1);
          o.z = finish(v[i][2], m, k, algo, alpha, beta, yr + 4 * idx + 2);
          o.w = finish(v[i][3], m, k, algo, alpha, beta, yr + 4 * idx + 3);
          reinterpret_cast<float4*>(yr)[idx] = o;
        } else {
          yr[idx] = finish(v[i][0], m, k, algo, alpha, beta, yr + idx);
        }
      }
    }
  }
}

// ---- rows too long for registers: online (max, sum) pass, then a write pass
__global__ void __launch_bounds__(kBlock) softmax_long_rows(const float* __restrict__ x,
                                                            float* __restrict__ y,
                                                            std::int64_t rows, std::int64_t len,
                                                            SoftmaxAlgo algo, float alpha,
                                                            float beta) {
  __shared__ float red[kBlock / 32 + 1];
  for (std::int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* xr = x + row * len;
    float* yr = y + row * len;
    float m = (algo == SoftmaxAlgo::kFast) ? 0.0f : -FLT_MAX;
    float s = 0.0f;
    for (std::int64_t i = threadIdx.x; i < len; i += kBlock) {
      const float v = xr[i];
      if (algo != SoftmaxAlgo::kFast && v > m) {
        s = s * expf(m - v);
        m = v;
      }
      s += expf(v - m);
    }
    float gm = m;
    if (algo != SoftmaxAlgo::kFast) gm = block_reduce<true>(m, red);
    s = (s == 0.0f) ? 0.0f : s * expf(m - gm);
    s = block_reduce<false>(s, red);
    const float k = (algo == SoftmaxAlgo::kLog) ? logf(s) : 1.0f / s;
    for (std::int64_t i = threadIdx.x; i < len; i += kBlock)
      yr[i] = finish(xr[i], gm, k, algo, alpha, beta, yr + i);
  }
}

// ---- arbitrary strides: one thread per reduction group, three passes like the
// reference's generic kernel (cudnn_kernels.metal:447-527).
__global__ void softmax_strided(const float* __restrict__ x, View4 xv, float* __restrict__ y,
                                View4 yv, bool instance, SoftmaxAlgo algo, float alpha,
                                float beta) {
  const std::int64_t groups =
      instance ? xv.n : static_cast<std::int64_t>(xv.n) * xv.h * xv.w;
  for (std::int64_t g = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       g < groups; g += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    int b, h0 = 0, w0 = 0, hn = xv.h, wn = xv.w;
    if (instance) {
      b = static_cast<int>(g);
    } else {
      w0 = static_cast<int>(g % xv.w);
      h0 = static_cast<int>((g / xv.w) % xv.h);
      b = static_cast<int>(g / (static_cast<std::int64_t>(xv.w) * xv.h));
      hn = h0 + 1;
      wn = w0 + 1;
    }
    auto xo = [&](int c, int h, int w) { return b * xv.ns + c * xv.cs + h * xv.hs + w * xv.ws; };
    auto yo = [&](int c, int h, int w) { return b * yv.ns + c * yv.cs + h * yv.hs + w * yv.ws; };
    float m = 0.0f;
    if (algo != SoftmaxAlgo::kFast) {
      m = -FLT_MAX;
      for (int c = 0; c < xv.c; ++c)
        for (int h = h0; h < hn; ++h)
          for (int w = w0; w < wn; ++w) m = fmaxf(m, x[xo(c, h, w)]);
    }
    float s = 0.0f;
    for (int c = 0; c < xv.c; ++c)
      for (int h = h0; h < hn; ++h)
        for (int w = w0; w < wn; ++w) s += expf(x[xo(c, h, w)] - m);
    const float k = (algo == SoftmaxAlgo::kLog) ? logf(s) : 1.0f / s;
    for (int c = 0; c < xv.c; ++c)
      for (int h = h0; h < hn; ++h)
        for (int w = w0; w < wn; ++w)
          y[yo(c, h, w)] = finish(x[xo(c, h, w)], m, k, algo, alpha, beta, y + yo(c, h, w));
  }
}

unsigned grid_for(std::int64_t work_ctas, int ctas_per_sm) {
  const int sms = sm_count(current_device());
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * ctas_per_sm * 16;
  return static_cast<unsigned>(work_ctas < cap ? (work_ctas > 0 ? work_ctas : 1) : cap);
}

template <int ITEMS>
void warp_launch(const float* x, float* y, std::int64_t rows, int len, SoftmaxAlgo a, float al,
                 float be, cudaStream_t st) {
  softmax_warp_rows<ITEMS><<<grid_for((rows + 7) / 8, 8), kBlock, 0, st>>>(x, y, rows, len, a,
                                                                           al, be);
}

template <int VEC, int ITEMS>
void block_launch(const float* x, float* y, std::int64_t rows, int len, SoftmaxAlgo a, float al,
                  float be, cudaStream_t st) {
  softmax_block_rows<VEC, ITEMS><<<grid_for(rows, 8), kBlock, 0, st>>>(x, y, rows, len, a, al,
                                                                       be);
}

}  // namespace

cudaError_t launch_softmax_rows(const float* x, float* y, std::int64_t rows, std::int64_t len,
                                SoftmaxAlgo algo, float alpha, float beta,
                                cudaStream_t stream) noexcept {
  if (rows <= 0 || len <= 0) return cudaSuccess;
  const int L = static_cast<int>(len);
  if (len <= 1024) {
    if (L <= 32) warp_launch<1>(x, y, rows, L, algo, alpha, beta, stream);
    else if (L <= 64) warp_launch<2>(x, y, rows, L, algo, alpha, beta, stream);
    else if (L <= 128) warp_launch<4>(x, y, rows, L, algo, alpha, beta, stream);
    else if (L <= 256) warp_launch<8>(x, y, rows, L, algo, alpha, beta, stream);
    else if (L <= 512) warp_launch<16>(x, y, rows, L, algo, alpha, beta, stream);
    else warp_launch<32>(x, y, rows, L, algo, alpha, beta, stream);
    return cudaGetLastError();
  }
  const bool vec4 = (len % 4 == 0) && aligned_to(x, 16) && aligned_to(y, 16);
  if (len <= 8192) {
    if (vec4) {
      const int n4 = L / 4;
      if (n4 <= kBlock) block_launch<4, 1>(x, y, rows, L, algo, alpha, beta, stream);
      else if (n4 <= 2 * kBlock) block_launch<4, 2>(x, y, rows, L, algo, alpha, beta, stream);
      else if (n4 <= 4 * kBlock) block_launch<4, 4>(x, y, rows, L, algo, alpha, beta, stream);
      else block_launch<4, 8>(x, y, rows, L, algo, alpha, beta, stream);
    } else {
      if (L <= 8 * kBlock) block_launch<1, 8>(x, y, rows, L, algo, alpha, beta, stream);
      else if (L <= 16 * kBlock) block_launch<1, 16>(x, y, rows, L, algo, alpha, beta, stream);
      else block_launch<1, 32>(x, y, rows, L, algo, alpha, beta, stream);
    }
    return cudaGetLastError();
  }
  softmax_long_rows<<<grid_for(rows, 8), kBlock, 0, stream>>>(x, y, rows, len, algo, alpha, beta);
  return cudaGetLastError();
}

cudaError_t launch_softmax_strided(const float* x, const View4& xv, float* y, const View4& yv,
                                   bool instance, SoftmaxAlgo algo, float alpha, float beta,
                                   cudaStream_t stream) noexcept {
  const std::int64_t groups = instance ? xv.n : static_cast<std::int64_t>(xv.n) * xv.h * xv.w;
  if (groups <= 0) return cudaSuccess;
  const unsigned grid = grid_for((groups + 127) / 128, 8);
  softmax_strided<<<grid, 128, 0, stream>>>(x, xv, y, yv, instance, algo, alpha, beta);
  return cudaGetLastError();
}

}  // namespace mb200::dnn
