// real_kernels.cu — real <-> complex passes of the R2C / C2R transforms.
//
// Semantics are those of the reference (libraries/fft/src/cufft_exec.mm:213-438):
// R2C is the forward complex transform of (x, 0) over all axes, keeping entries
// 0 .. L/2 of the last axis; C2R inverts the leading axes on the half spectrum,
// expands each last-axis row by conjugate symmetry (cufft_kernels.metal:94-117)
// and keeps the real part of the inverse (:119-132); no scaling.
//
// B200 path for even L: the reals of a row are read as L/2 complex pairs, one
// length-L/2 complex FFT runs on them, and the post-pass below turns its output
// into the L/2 + 1 half-spectrum entries (C2R: the pre-pass, then a length-L/2
// inverse written straight into the real output).  That halves the FFT work and
// skips the reference's gather and scatter passes over full-length complex rows.
// The gather/scatter/expand kernels serve the general path (odd L, strided reals).
#include <cuda_runtime.h>

#include <cstdint>

#include "common/device.hpp"
#include "fft/fft.hpp"

namespace mb200::fft {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

unsigned grid_for(std::int64_t work) {
  const int sms = sm_count(current_device());
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 8;
  const std::int64_t want = (work + kThreads - 1) / kThreads;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

__global__ void __launch_bounds__(kThreads)
    r2c_post(RealRows g, const float2* __restrict__ Z, float2* __restrict__ out,
             std::int64_t odist, std::int64_t ostride) {
  const std::int64_t H = g.M + 1;
  const std::int64_t total = g.rows * H;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       t < total; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = t / H, k = t % H;
    const float2* z = Z + r * g.M;
    const float2 a = z[k == g.M ? 0 : k];
    const float2 c = z[k == 0 ? 0 : g.M - k];
    const float2 b = make_float2(c.x, -c.y);  // conj(Z[M - k])
    const float2 e = make_float2(0.5f * (a.x + b.x), 0.5f * (a.y + b.y));
    const float2 d = make_float2(0.5f * (a.x - b.x), 0.5f * (a.y - b.y));
    const float2 o = make_float2(d.y, -d.x);  // -i d
    const float2 w = cmul(g.tw[k], o);
    const std::int64_t b_i = r / g.prefix, p = r % g.prefix;
    out[b_i * odist + (p * H + k) * ostride] = make_float2(e.x + w.x, e.y + w.y);
  }
}

__global__ void __launch_bounds__(kThreads)
    c2r_pre(RealRows g, const float2* __restrict__ X, std::int64_t idist, std::int64_t istride,
            float2* __restrict__ Z) {
  const std::int64_t H = g.M + 1;
  const std::int64_t total = g.rows * g.M;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       t < total; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = t / g.M, k = t % g.M;
    const std::int64_t b_i = r / g.prefix, p = r % g.prefix;
    const float2* x = X + b_i * idist + p * H * istride;
    float2 xk = x[k * istride];
    float2 xc;
    if (k == 0) {
      xk.y = 0.0f;
      xc = make_float2(x[g.M * istride].x, 0.0f);
    } else {
      const float2 v = x[(g.M - k) * istride];
      xc = make_float2(v.x, -v.y);
    }
    const float2 e = make_float2(xk.x + xc.x, xk.y + xc.y);
    const float2 w = g.tw[k];
    const float2 o = cmul(make_float2(xk.x - xc.x, xk.y - xc.y), make_float2(w.x, -w.y));
    Z[r * g.M + k] = make_float2(e.x - o.y, e.y + o.x);  // e + i o
  }
}

__global__ void __launch_bounds__(kThreads)
    gather_real(std::int64_t rows, std::int64_t prefix, std::int64_t L, const float* __restrict__ in,
                std::int64_t idist, std::int64_t istride, float2* __restrict__ out) {
  const std::int64_t total = rows * L;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       t < total; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = t / L, i = t % L;
    const std::int64_t b = r / prefix, p = r % prefix;
    out[t] = make_float2(in[b * idist + (p * L + i) * istride], 0.0f);
  }
}

__global__ void __launch_bounds__(kThreads)
    scatter_half(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                 const float2* __restrict__ in, float2* __restrict__ out, std::int64_t odist,
                 std::int64_t ostride) {
  const std::int64_t H = L / 2 + 1;
  const std::int64_t total = rows * H;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       t < total; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = t / H, k = t % H;
    const std::int64_t b = r / prefix, p = r % prefix;
    out[b * odist + (p * H + k) * ostride] = in[r * L + k];
  }
}

__global__ void __launch_bounds__(kThreads)
    gather_half(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                const float2* __restrict__ in, std::int64_t idist, std::int64_t istride,
                float2* __restrict__ out) {
  const std::int64_t H = L / 2 + 1;
  const std::int64_t total = rows * H;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       t < total; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = t / H, k = t % H;
    const std::int64_t b = r / prefix, p = r % prefix;
    out[t] = in[b * idist + (p * H + k) * istride];
  }
}

__global__ void __launch_bounds__(kThreads)
    expand_half(std::int64_t rows, std::int64_t L, const float2* __restrict__ in,
                float2* __restrict__ out) {
  const std::int64_t H = L / 2 + 1;
  const std::int64_t total = rows * L;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       t < total; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = t / L, k = t % L;
    if (k < H) {
      out[t] = in[r * H + k];
    } else {
      const float2 v = in[r * H + (L - k)];
      out[t] = make_float2(v.x, -v.y);
    }
  }
}

__global__ void __launch_bounds__(kThreads)
    scatter_real(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                 const float2* __restrict__ in, float* __restrict__ out, std::int64_t odist,
                 std::int64_t ostride) {
  const std::int64_t total = rows * L;
  for (std::int64_t t = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       t < total; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = t / L, i = t % L;
    const std::int64_t b = r / prefix, p = r % prefix;
    out[b * odist + (p * L + i) * ostride] = in[t].x;
  }
}

}  // namespace

cudaError_t launch_r2c_post(const RealRows& g, const float2* Z, float2* out, std::int64_t odist,
                            std::int64_t ostride, cudaStream_t stream) noexcept {
  r2c_post<<<grid_for(g.rows * (g.M + 1)), kThreads, 0, stream>>>(g, Z, out, odist, ostride);
  return cudaGetLastError();
}

cudaError_t launch_c2r_pre(const RealRows& g, const float2* X, std::int64_t idist,
                           std::int64_t istride, float2* Z, cudaStream_t stream) noexcept {
  c2r_pre<<<grid_for(g.rows * g.M), kThreads, 0, stream>>>(g, X, idist, istride, Z);
  return cudaGetLastError();
}

cudaError_t launch_gather_real(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                               const float* in, std::int64_t idist, std::int64_t istride,
                               float2* out, cudaStream_t stream) noexcept {
  gather_real<<<grid_for(rows * L), kThreads, 0, stream>>>(rows, prefix, L, in, idist, istride,
                                                           out);
  return cudaGetLastError();
}

cudaError_t launch_scatter_half(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                                const float2* in, float2* out, std::int64_t odist,
                                std::int64_t ostride, cudaStream_t stream) noexcept {
  scatter_half<<<grid_for(rows * (L / 2 + 1)), kThreads, 0, stream>>>(rows, prefix, L, in, out,
                                                                      odist, ostride);
  return cudaGetLastError();
}

cudaError_t launch_gather_half(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                               const float2* in, std::int64_t idist, std::int64_t istride,
                               float2* out, cudaStream_t stream) noexcept {
  gather_half<<<grid_for(rows * (L / 2 + 1)), kThreads, 0, stream>>>(rows, prefix, L, in, idist,
                                                                     istride, out);
  return cudaGetLastError();
}

cudaError_t launch_expand_half(std::int64_t rows, std::int64_t L, const float2* in, float2* out,
                               cudaStream_t stream) noexcept {
  expand_half<<<grid_for(rows * L), kThreads, 0, stream>>>(rows, L, in, out);
  return cudaGetLastError();
}

cudaError_t launch_scatter_real(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                                const float2* in, float* out, std::int64_t odist,
                                std::int64_t ostride, cudaStream_t stream) noexcept {
  scatter_real<<<grid_for(rows * L), kThreads, 0, stream>>>(rows, prefix, L, in, out, odist,
                                                            ostride);
  return cudaGetLastError();
}

}  // namespace mb200::fft
