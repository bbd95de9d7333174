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

// Mixed-radix transforms (radices 16, 8, 4, 2, 3, 5, 7) of lengths that are not powers
// of two and have no prime factor above 7, n <= kMaxMixed: one kernel, the whole
// transform in shared memory; b.tw = exp(-2*pi*i*m/n).  In-place calls are allowed.
constexpr std::int64_t kMaxMixed = 12288;
bool mixed_radix_supported(std::int64_t n) noexcept;
cudaError_t launch_mixed_radix(std::int64_t n, int sign, const Batch1D& b,
                               cudaStream_t stream) noexcept;

// Fills tw[0 .. n) with exp(-2*pi*i*m/n) rounded from double precision.
void host_twiddles(std::int64_t n, float2* tw) noexcept;

// Bluestein (chirp-z) transforms of a length n that is not a power of two, for n in
// [kMinBluestein, kMaxBluestein]: one kernel per call, both inner length-Mb FFTs
// (Mb = bluestein_length(n), the power of two >= 2n - 1) on chip.  Tables of the
// forward direction: chirp[m] = exp(-pi*i*(m^2 mod 2n)/n), m < n; bhat = FFT(b) / Mb
// with b[m] = b[Mb - m] = conj(chirp[m]) and zeros between; tw_m = exp(-2*pi*i*m/Mb).
// In-place calls (same layout) are allowed; post_tw must be null.
constexpr std::int64_t kMinBluestein = 32;
constexpr std::int64_t kMaxBluestein = 4096;
std::int64_t bluestein_length(std::int64_t n) noexcept;
cudaError_t launch_bluestein(std::int64_t n, int sign, const Batch1D& b, const float2* chirp,
                             const float2* bhat, const float2* tw_m,
                             cudaStream_t stream) noexcept;
// Longer lengths (kMaxBluestein < n <= kMaxBluesteinGlobal) run Bluestein through
// global memory, chunk by chunk of ws_rows transforms: chirp-multiplied gather into
// dense rows of Mb, forward FFT, multiply by bhat, inverse FFT, chirp-multiplied
// scatter.  An inner length above kMaxSinglePass uses the two-pass split
// Mb = n1 * n2 with the scratch rows ws2.  In-place calls are allowed.
// Up to 2^27, so that Mb <= 2^28 = kMaxSinglePass^2 (the two-pass split's limit).
constexpr std::int64_t kMaxBluesteinGlobal = std::int64_t{1} << 27;
// Tables of lengths up to these are built on the host in double precision; longer ones on
// the device (build_twiddles, build_bluestein_tables), where the host work would take
// seconds.
constexpr std::int64_t kMaxHostTwiddles = std::int64_t{1} << 22;
constexpr std::int64_t kMaxHostBluestein = std::int64_t{1} << 20;
struct BluesteinGlobal {
  const float2* chirp;
  const float2* bhat;
  const float2* tw_m;  // exp(-2*pi*i*m/Mb)
  float2* ws;          // ws_rows * Mb
  float2* ws2;         // ws_rows * Mb when Mb > kMaxSinglePass, else null
  std::int64_t ws_rows;
  std::int64_t n1, n2;
  const float2* tw_n1;
  const float2* tw_n2;
};
cudaError_t launch_bluestein_global(std::int64_t n, int sign, const Batch1D& b,
                                    const BluesteinGlobal& g, cudaStream_t stream) noexcept;
// Fills chirp[0 .. n) and bhat[0 .. Mb) in double precision, rounded once.
void host_bluestein_tables(std::int64_t n, std::int64_t mb, float2* chirp, float2* bhat) noexcept;
// Device versions for long lengths: tw[m] = exp(-2*pi*i*m/n) from double sincospi, rounded
// once; chirp as above from double sincospi of the exact (m^2 mod 2n)/n; bhat = the fp32
// FFT of the rounded b, scaled by 1/Mb (exact), computed in place in bhat with g's
// twiddles and scratch (g.tw_m, and for Mb > kMaxSinglePass g.n1, g.n2, g.tw_n1, g.tw_n2,
// g.ws2).  Stream-ordered.
cudaError_t build_twiddles(float2* tw, std::int64_t n, cudaStream_t stream) noexcept;
cudaError_t build_bluestein_tables(std::int64_t n, float2* chirp, float2* bhat,
                                   const BluesteinGlobal& g, cudaStream_t stream) noexcept;

// Real-data transforms of even length L = 2M through a length-M complex FFT of
// the reals read as M complex pairs, z[n] = x[2n] + i x[2n+1].  Rows are indexed
// r = b * prefix + p (b the batch entry, p the position along the leading axes).
// Complex element k of row r of a strided operand sits at
//   base + b * dist + (p * row_len + k) * stride.
struct RealRows {
  std::int64_t rows, prefix;
  std::int64_t M;          // half length
  const float2* tw;        // exp(-2*pi*i*m/L), m in [0, L)
};

// Fused real-data transforms of dense rows (reals of row r at r * 2n, half
// spectrum at r * (n + 1)) for half length n a power of two in [16, 4096]: one
// kernel per direction, the length-n complex FFT with the R2C post-pass in its
// epilogue or the C2R pre-pass in its first pass.  `groups` groups of
// real_bulk_rows_per_group(n) rows each; tw = exp(-2*pi*i*m/n), twl = exp(-2*pi*i*m/(2n)).
// real_bulk_aligned says whether the pointers meet the kernels' alignment (R2C:
// 16-byte reals; C2R: 16-byte reals and, for n <= 2048, 16-byte half spectra);
// input and output must not overlap.
std::int64_t real_bulk_rows_per_group(std::int64_t n) noexcept;
bool real_bulk_aligned(bool r2c, std::int64_t n, const void* in, const void* out) noexcept;
cudaError_t launch_real_bulk(bool r2c, std::int64_t n, const void* in, void* out,
                             long long groups, const float2* tw, const float2* twl,
                             cudaStream_t stream) noexcept;

// R2C post-pass: Z (row r at Z + r * M, dense) -> X[0 .. M] of each row,
// X[k] = (Z[k] + conj(Z[M-k]))/2 - i W^k (Z[k] - conj(Z[M-k]))/2, W = exp(-2*pi*i/L),
// Z[M] = Z[0]; written to out with row_len M + 1.
cudaError_t launch_r2c_post(const RealRows& g, const float2* Z, float2* out, std::int64_t odist,
                            std::int64_t ostride, cudaStream_t stream) noexcept;

// C2R pre-pass: X[0 .. M] of each row (read with row_len M + 1) -> Z' (dense),
// Z'[k] = E[k] + i O[k], E[k] = X[k] + X[k+M], O[k] = (X[k] - X[k+M]) W^-k with
// X[k+M] = conj(X[M-k]) for k > 0, the imaginary parts of X[0] and X[M] ignored
// (the reference expands the half spectrum and keeps the real part of a complex
// inverse, which drops exactly those); the length-M inverse of Z' is then
// x[2n] + i x[2n+1] of the unnormalised real inverse.
cudaError_t launch_c2r_pre(const RealRows& g, const float2* X, std::int64_t idist,
                           std::int64_t istride, float2* Z, cudaStream_t stream) noexcept;

// Real <-> complex layout moves of the general path: gather reals as (x, 0)
// into dense complex rows of length L; scatter the first M + 1 (= L/2 + 1)
// entries of dense complex rows into a strided half-spectrum output; expand a
// dense half spectrum (row_len L/2 + 1) into full rows by conjugate symmetry;
// scatter the real parts of dense complex rows into a strided real output.
cudaError_t launch_gather_real(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                               const float* in, std::int64_t idist, std::int64_t istride,
                               float2* out, cudaStream_t stream) noexcept;
cudaError_t launch_scatter_half(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                                const float2* in, float2* out, std::int64_t odist,
                                std::int64_t ostride, cudaStream_t stream) noexcept;
cudaError_t launch_gather_half(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                               const float2* in, std::int64_t idist, std::int64_t istride,
                               float2* out, cudaStream_t stream) noexcept;
cudaError_t launch_expand_half(std::int64_t rows, std::int64_t L, const float2* in, float2* out,
                               cudaStream_t stream) noexcept;
cudaError_t launch_scatter_real(std::int64_t rows, std::int64_t prefix, std::int64_t L,
                                const float2* in, float* out, std::int64_t odist,
                                std::int64_t ostride, cudaStream_t stream) noexcept;

}  // namespace mb200::fft
