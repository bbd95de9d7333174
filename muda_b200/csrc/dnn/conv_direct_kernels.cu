// conv_direct_kernels.cu — direct convolution forward, any geometry.
//
// One thread per output element with an fp32 accumulator, looping over the
// input channels of its group and the filter taps.  Index arithmetic follows the
// reference's direct kernel (libraries/dnn/shaders/cudnn_kernels.metal:20-62):
// tap (r, s) reads x at (oy*stride_h - pad_h + r*dil_h, ox*stride_w - pad_w + s*dil_w);
// CUDNN_CONVOLUTION flips the filter (kh-1-r, kw-1-s); the filter offset is
// ((k*C + c)*R + r)*S + s for KCRS and ((k*R + r)*S + s)*C + c for KRSC
// (cudnn_kernels.metal:13-18); y = fma(alpha, acc, beta == 0 ? 0 : beta*y).
//
// This kernel covers grouped, dilated, strided, flipped and arbitrarily strided
// tensors.  The dense NHWC/KRSC shapes are served by the tensor-core implicit
// GEMM instead.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common/device.hpp"
#include "dnn/dnn.hpp"

namespace mb200::dnn {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  if constexpr (sizeof(T) == 2) {
    return __bfloat162float(*p);
  } else {
    return *p;
  }
}

template <typename T>
__device__ __forceinline__ void st(T* p, float v) {
  if constexpr (sizeof(T) == 2) {
    *p = __float2bfloat16_rn(v);
  } else {
    *p = v;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) conv_direct(const T* __restrict__ x, const T* __restrict__ w,
                                                   T* __restrict__ y, ConvShape s, float alpha,
                                                   float beta) {
  const std::int64_t total = static_cast<std::int64_t>(s.y.n) * s.y.c * s.y.h * s.y.w;
  const int cin_g = s.x.c / s.groups;
  const int cout_g = s.y.c / s.groups;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    // Output index order (n, k, oy, ox) with ox fastest, as in the reference.
    const int ox = static_cast<int>(t % s.y.w);
    std::int64_t rem = t / s.y.w;
    const int oy = static_cast<int>(rem % s.y.h);
    rem /= s.y.h;
    const int oc = static_cast<int>(rem % s.y.c);
    const int b = static_cast<int>(rem / s.y.c);
    const int g = oc / cout_g;
    float acc = 0.0f;
    for (int cg = 0; cg < cin_g; ++cg) {
      const int ic = g * cin_g + cg;
      for (int r = 0; r < s.kh; ++r) {
        const int fr = s.convolution ? (s.kh - 1 - r) : r;
        const int iy = oy * s.stride_h - s.pad_h + r * s.dil_h;
        if (iy < 0 || iy >= s.x.h) continue;
        for (int q = 0; q < s.kw; ++q) {
          const int fs = s.convolution ? (s.kw - 1 - q) : q;
          const int ix = ox * s.stride_w - s.pad_w + q * s.dil_w;
          if (ix < 0 || ix >= s.x.w) continue;
          const std::int64_t xi = b * s.x.ns + ic * s.x.cs + iy * s.x.hs + ix * s.x.ws;
          const std::int64_t wi =
              s.filter_krsc
                  ? ((static_cast<std::int64_t>(oc) * s.kh + fr) * s.kw + fs) * cin_g + cg
                  : ((static_cast<std::int64_t>(oc) * cin_g + cg) * s.kh + fr) * s.kw + fs;
          acc = fmaf(ld(x + xi), ld(w + wi), acc);
        }
      }
    }
    const std::int64_t yi = b * s.y.ns + oc * s.y.cs + oy * s.y.hs + ox * s.y.ws;
    const float prev = (beta == 0.0f) ? 0.0f : beta * ld(y + yi);
    st(y + yi, fmaf(alpha, acc, prev));
  }
}

}  // namespace

cudaError_t launch_conv_direct(const void* x, const void* w, void* y, const ConvShape& s,
                               ConvDtype dt, float alpha, float beta, cudaStream_t stream) noexcept {
  const std::int64_t total = static_cast<std::int64_t>(s.y.n) * s.y.c * s.y.h * s.y.w;
  if (total <= 0) return cudaSuccess;
  const int sms = sm_count(current_device());
  const std::int64_t want = (total + 255) / 256;
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 64;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  if (dt == ConvDtype::kBF16) {
    conv_direct<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
        static_cast<__nv_bfloat16*>(y), s, alpha, beta);
  } else {
    conv_direct<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(x),
                                                 static_cast<const float*>(w),
                                                 static_cast<float*>(y), s, alpha, beta);
  }
  return cudaGetLastError();
}

}  // namespace mb200::dnn
