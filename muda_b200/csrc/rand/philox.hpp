// philox.hpp — launch interface of the Philox4x32-10 fill kernels.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

namespace mb200::rand {

enum class Dist : int { kUint32 = 0, kUniform = 1, kNormal = 2 };

// Fills out[0 .. n) with the Philox stream of (seed, first_block):
//   block i (0-based) uses counter (first_block + i, 0, 0) and key (seed_lo, seed_hi);
//   its four words go to out[4i .. 4i+3] (a partial last block writes only n % 4 words).
// out must be 4-byte aligned; 16-byte alignment selects the vector-store kernel.
cudaError_t launch_philox_fill(Dist dist, void* out, std::uint64_t n, std::uint64_t seed,
                               std::uint64_t first_block, float mean, float stddev,
                               cudaStream_t stream) noexcept;

// Number of device kernels one launch_philox_fill call issues (0 for n == 0).
int philox_fill_launch_count(std::uint64_t n) noexcept;

}  // namespace mb200::rand
