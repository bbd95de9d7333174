// dft_kernels.cu — direct DFT for lengths that are not powers of two.
//
// The reference evaluates such axes with an O(n^2) DFT, one thread per output,
// computing each twiddle with sincos (libraries/fft/shaders/cufft_kernels.metal:298-325).
// Same complexity here, but one CTA stages its whole transform in shared memory
// (so in-place calls are safe) and twiddles come from the exact-rounded table,
// indexed by (t*k) mod n with integer arithmetic so no angle loses precision.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <utility>
#include <vector>

#include "common/device.hpp"
#include "fft/fft.hpp"

namespace mb200::fft {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}

template <int S>
__global__ void __launch_bounds__(kThreads) direct_dft_kernel(const Batch1D bt, int n) {
  extern __shared__ float2 xs[];
  for (std::int64_t tr = blockIdx.x; tr < bt.batch; tr += gridDim.x) {
    const std::int64_t outer = tr / bt.inner_count;
    const std::int64_t inner = tr % bt.inner_count;
    const float2* in = bt.in + outer * bt.in_outer + inner * bt.in_inner;
    float2* out = bt.out + outer * bt.out_outer + inner * bt.out_inner;
    __syncthreads();  // previous transform's readers are done with xs
    for (int t = threadIdx.x; t < n; t += kThreads) xs[t] = in[t * bt.in_stride];
    __syncthreads();
    for (int k = threadIdx.x; k < n; k += kThreads) {
      float2 acc = make_float2(0.0f, 0.0f);
      int m = 0;  // (t * k) mod n
      for (int t = 0; t < n; ++t) {
        float2 w = __ldg(bt.tw + m);
        if (S > 0) w.y = -w.y;
        const float2 p = cmul(xs[t], w);
        acc.x += p.x;
        acc.y += p.y;
        m += k;
        if (m >= n) m -= n;
      }
      if (bt.post_tw != nullptr) {
        float2 w = __ldg(bt.post_tw + (inner * k) % bt.post_n);
        if (S > 0) w.y = -w.y;
        acc = cmul(acc, w);
      }
      out[k * bt.out_stride] = acc;
    }
  }
}

}  // namespace

cudaError_t launch_direct_dft(std::int64_t n, int sign, const Batch1D& b,
                              cudaStream_t stream) noexcept {
  if (b.batch <= 0) return cudaSuccess;
  if (n < 1 || n * static_cast<std::int64_t>(sizeof(float2)) > 200 * 1024)
    return cudaErrorInvalidValue;
  const int smem = static_cast<int>(n * sizeof(float2));
  const int sms = sm_count(current_device());
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 16;
  const unsigned grid = static_cast<unsigned>(b.batch < cap ? b.batch : cap);
  if (sign < 0) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(direct_dft_kernel<-1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return cudaErrorInvalidValue;
    direct_dft_kernel<-1><<<grid, kThreads, smem, stream>>>(b, static_cast<int>(n));
  } else {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(direct_dft_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return cudaErrorInvalidValue;
    direct_dft_kernel<1><<<grid, kThreads, smem, stream>>>(b, static_cast<int>(n));
  }
  return cudaGetLastError();
}

void host_twiddles(std::int64_t n, float2* tw) noexcept {
  const double two_pi = 6.283185307179586476925286766559;
  for (std::int64_t m = 0; m < n; ++m) {
    const double a = two_pi * static_cast<double>(m) / static_cast<double>(n);
    tw[m].x = static_cast<float>(std::cos(a));
    tw[m].y = static_cast<float>(-std::sin(a));
  }
}

// chirp[m] = exp(-pi*i*q/n) with q = m^2 mod 2n taken in integers, so the angle
// is exact before the one rounding; bhat = FFT(b) / mb by an in-place iterative
// radix-2 transform in double precision (host), rounded once.
void host_bluestein_tables(std::int64_t n, std::int64_t mb, float2* chirp, float2* bhat) noexcept {
  const double pi = 3.141592653589793238462643383279;
  std::vector<double> re(static_cast<std::size_t>(mb), 0.0), im(static_cast<std::size_t>(mb), 0.0);
  for (std::int64_t m = 0; m < n; ++m) {
    const std::int64_t q = static_cast<std::int64_t>(
        (static_cast<unsigned long long>(m) * static_cast<unsigned long long>(m)) %
        static_cast<unsigned long long>(2 * n));
    const double a = pi * static_cast<double>(q) / static_cast<double>(n);
    const double c = std::cos(a), sn = std::sin(a);
    chirp[m].x = static_cast<float>(c);
    chirp[m].y = static_cast<float>(-sn);
    // b[m] = conj(chirp[m]) = exp(+pi*i*q/n), mirrored to mb - m
    re[static_cast<std::size_t>(m)] = c;
    im[static_cast<std::size_t>(m)] = sn;
    if (m > 0) {
      re[static_cast<std::size_t>(mb - m)] = c;
      im[static_cast<std::size_t>(mb - m)] = sn;
    }
  }
  // bit-reversal permutation, then log2(mb) butterfly stages with exp(-2*pi*i*k/len)
  for (std::int64_t i = 1, j = 0; i < mb; ++i) {
    std::int64_t bit = mb >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) {
      std::swap(re[static_cast<std::size_t>(i)], re[static_cast<std::size_t>(j)]);
      std::swap(im[static_cast<std::size_t>(i)], im[static_cast<std::size_t>(j)]);
    }
  }
  for (std::int64_t len = 2; len <= mb; len <<= 1) {
    const std::int64_t half = len / 2;
    std::vector<double> wr(static_cast<std::size_t>(half)), wi(static_cast<std::size_t>(half));
    for (std::int64_t k = 0; k < half; ++k) {
      const double a = 2.0 * pi * static_cast<double>(k) / static_cast<double>(len);
      wr[static_cast<std::size_t>(k)] = std::cos(a);
      wi[static_cast<std::size_t>(k)] = -std::sin(a);
    }
    for (std::int64_t s0 = 0; s0 < mb; s0 += len) {
      for (std::int64_t k = 0; k < half; ++k) {
        const std::size_t u = static_cast<std::size_t>(s0 + k);
        const std::size_t v = static_cast<std::size_t>(s0 + k + half);
        const double xr = re[v] * wr[static_cast<std::size_t>(k)] - im[v] * wi[static_cast<std::size_t>(k)];
        const double xi = re[v] * wi[static_cast<std::size_t>(k)] + im[v] * wr[static_cast<std::size_t>(k)];
        re[v] = re[u] - xr;
        im[v] = im[u] - xi;
        re[u] += xr;
        im[u] += xi;
      }
    }
  }
  const double inv = 1.0 / static_cast<double>(mb);
  for (std::int64_t k = 0; k < mb; ++k) {
    bhat[k].x = static_cast<float>(re[static_cast<std::size_t>(k)] * inv);
    bhat[k].y = static_cast<float>(im[static_cast<std::size_t>(k)] * inv);
  }
}

}  // namespace mb200::fft
