// fft.hpp — launch interface of the complex-to-complex FFT kernels.
#pragma once

#include <cuda_runtime_api.h>

#include <cstdint>

namespace mb200::fft {

// One batched 1-D transform of length n.  Transform b reads element t at
//   in + (b / inner_count) * in_outer + (b % inner_count) * in_inner + t * in_stride
// and writes output k at the same form with the out_* strides (element units of
// float2).  inner_count > 1 expresses the axis passes of 2-D/3-D transforms and
// the column pass of the large-n split.  If post_tw is set, output k of transform
// b is multiplied by post_tw[((b % inner_count) * k) % post_n] (conjugated for
// sign > 0) before it is stored.
struct Batch1D {
  const float2* in;
  float2* out;
  std::int64_t in_stride, in_outer, in_inner;
  std::int64_t out_stride, out_outer, out_inner;
  std::int64_t batch;
  std::int64_t inner_count;
  const float2* tw;        // exp(-2*pi*i*m/n), m in [0, n)
  const float2* post_tw;   // exp(-2*pi*i*m/post_n), or null
  std::int64_t post_n;
};

// True when the shared-memory Stockham kernel handles length n in one pass.
bool single_pass_supported(std::int64_t n) noexcept;

// Largest length of a single-pass transform.
constexpr std::int64_t kMaxSinglePass = 16384;

// sign = -1 forward, +1 inverse (unnormalised).  n must be a power of two in
// [2, kMaxSinglePass].  In-place (in == out with equal strides) is allowed.
cudaError_t launch_stockham(std::int64_t n, int sign, const Batch1D& b,
                            cudaStream_t stream) noexcept;

// Direct O(n^2) DFT for lengths that are not powers of two, n in [1, kMaxDirect],
// reading twiddles from tw (n entries).  Each transform is staged in shared
// memory before any output is written, so in-place calls are allowed.
constexpr std::int64_t kMaxDirect = 25600;
cudaError_t launch_direct_dft(std::int64_t n, int sign, const Batch1D& b,
                              cudaStream_t stream) noexcept;

// Fills tw[0 .. n) with exp(-2*pi*i*m/n) rounded from double precision.
void host_twiddles(std::int64_t n, float2* tw) noexcept;

}  // namespace mb200::fft
