// philox.hpp — launch interface of the Philox4x32-10 fill kernels.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

namespace mb200::rand {

enum class Dist : int {
  kUint32 = 0,
  kUniform = 1,
  kNormal = 2,
  kLogNormal = 3,        // exp of the normal stream
  kUniformDouble = 4,    // two doubles per block
  kNormalDouble = 5,
  kLogNormalDouble = 6,
};

// Fills out[0 .. n) with the Philox stream of (seed, first_block):
//   block i (0-based) uses counter (first_block + i, 0, 0) and key (seed_lo, seed_hi);
//   its four words go to out[4i .. 4i+3] (a partial last block writes only n % 4 words).
// out must be 4-byte aligned; 16-byte alignment selects the vector-store kernel.
cudaError_t launch_philox_fill(Dist dist, void* out, std::uint64_t n, std::uint64_t seed,
                               std::uint64_t first_block, float mean, float stddev,
                               cudaStream_t stream) noexcept;

// Double-precision streams (reference curand_context.mm:115-143, 187-223, 237-247):
// block i uses counter (first_block + i, 0, 0) and gives two values from the 53-bit
// integers m0 = ((r0 << 21) ^ r1) & (2^53 - 1), m1 = ((r2 << 21) ^ r3) & (2^53 - 1):
// uniform u = (m + 1) * 2^-53; normal: r = sqrt(-2 ln u0), theta = 2pi u1,
// (r cos theta * stddev + mean, r sin theta * stddev + mean); log-normal: exp of it.
// out must be 8-byte aligned.
cudaError_t launch_philox_fill_f64(Dist dist, double* out, std::uint64_t n, std::uint64_t seed,
                                   std::uint64_t first_block, double mean, double stddev,
                                   cudaStream_t stream) noexcept;

// Poisson(lambda) counts (reference curand_kernels.metal:212-264): output i uses the
// block (first_block + i, 0, s, 0), s = 0, 1, ... for its successive groups of four
// uniforms.  lambda < 30: Knuth's product of uniforms against exp_neg_lambda, at most
// 1000 factors, count - 1; otherwise floor(lambda + sqrt(lambda) z + 0.5) clamped at
// 0, z = sqrt(-2 ln u0) cos(2pi u1) of the block's first two uniforms (fp32).
cudaError_t launch_philox_poisson(unsigned int* out, std::uint64_t n, std::uint64_t seed,
                                  std::uint64_t first_block, float lambda, float exp_neg_lambda,
                                  cudaStream_t stream) noexcept;

// Number of device kernels one launch_philox_fill call issues (0 for n == 0).
int philox_fill_launch_count(std::uint64_t n, std::uint64_t first_block) noexcept;

}  // namespace mb200::rand
