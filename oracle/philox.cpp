// philox.cpp — restatement of the reference's host Philox4x32-10 generator.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Follows libraries/rand/src/curand_context.mm operation by operation:
//   PhiloxHostStep        curand_context.mm:42-73
//   GenerateHostUint      curand_context.mm:75-93
//   GenerateHostUniform   curand_context.mm:95-113
//   GenerateHostNormal    curand_context.mm:145-185
// The only addition is `threads`: the block loop is split across std::threads
// for the multi-core CPU baseline.  Blocks are independent, so the output does
// not depend on the thread count; threads == 1 is the reference's own
// single-threaded loop.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "oracle.h"
#include "parallel.h"

namespace {

constexpr float kTwoPowMinus32 = 2.3283064365386963e-10f;  // curand_context.mm:19
constexpr float kTwoPi = 6.28318530717958647692f;          // curand_context.mm:22

inline float uniform_of(std::uint32_t r) {
  return (static_cast<float>(r) + 1.0f) * kTwoPowMinus32;
}

}  // namespace

extern "C" void oracle_philox_block(uint64_t ctr_idx, uint64_t seed, uint32_t out[4]) {
  std::uint32_t ctr[4] = {static_cast<std::uint32_t>(ctr_idx),
                          static_cast<std::uint32_t>(ctr_idx >> 32), 0u, 0u};
  std::uint32_t key[2] = {static_cast<std::uint32_t>(seed), static_cast<std::uint32_t>(seed >> 32)};
  for (int round = 0; round < 10; ++round) {
    const std::uint64_t p0 = std::uint64_t{0xD2511F53u} * ctr[0];
    const std::uint64_t p1 = std::uint64_t{0xCD9E8D57u} * ctr[2];
    const std::uint32_t n0 = static_cast<std::uint32_t>(p1 >> 32) ^ ctr[1] ^ key[0];
    const std::uint32_t n1 = static_cast<std::uint32_t>(p1);
    const std::uint32_t n2 = static_cast<std::uint32_t>(p0 >> 32) ^ ctr[3] ^ key[1];
    const std::uint32_t n3 = static_cast<std::uint32_t>(p0);
    ctr[0] = n0;
    ctr[1] = n1;
    ctr[2] = n2;
    ctr[3] = n3;
    key[0] += 0x9E3779B9u;
    key[1] += 0xBB67AE85u;
  }
  std::memcpy(out, ctr, sizeof(ctr));
}

extern "C" uint64_t oracle_generate_uint(uint64_t seed, uint64_t offset, uint32_t* out, size_t n,
                                         int threads) {
  const std::int64_t rounds = static_cast<std::int64_t>((n + 3) / 4);
  oracle_detail::parallel_for(0, rounds, threads, [&](std::int64_t i) {
    std::uint32_t r[4];
    oracle_philox_block(static_cast<std::uint64_t>(i) + (offset >> 2), seed, r);
    const std::size_t base = static_cast<std::size_t>(i) * 4;
    for (std::size_t j = 0; j < 4 && base + j < n; ++j) out[base + j] = r[j];
  });
  return offset + static_cast<std::uint64_t>(rounds) * 4;
}

extern "C" uint64_t oracle_generate_uniform(uint64_t seed, uint64_t offset, float* out, size_t n,
                                            int threads) {
  const std::int64_t rounds = static_cast<std::int64_t>((n + 3) / 4);
  oracle_detail::parallel_for(0, rounds, threads, [&](std::int64_t i) {
    std::uint32_t r[4];
    oracle_philox_block(static_cast<std::uint64_t>(i) + (offset >> 2), seed, r);
    const std::size_t base = static_cast<std::size_t>(i) * 4;
    for (std::size_t j = 0; j < 4 && base + j < n; ++j) out[base + j] = uniform_of(r[j]);
  });
  return offset + static_cast<std::uint64_t>(rounds) * 4;
}

extern "C" uint64_t oracle_generate_normal(uint64_t seed, uint64_t offset, float* out, size_t n,
                                           float mean, float stddev, int threads) {
  const std::int64_t rounds = static_cast<std::int64_t>((n + 3) / 4);
  oracle_detail::parallel_for(0, rounds, threads, [&](std::int64_t i) {
    std::uint32_t r[4];
    oracle_philox_block(static_cast<std::uint64_t>(i) + (offset >> 2), seed, r);
    const float u0 = uniform_of(r[0]);
    const float u1 = uniform_of(r[1]);
    const float u2 = uniform_of(r[2]);
    const float u3 = uniform_of(r[3]);
    const float r0 = std::sqrt(-2.0f * std::log(u0));
    const float theta0 = kTwoPi * u1;
    const float z0 = r0 * std::cos(theta0) * stddev + mean;
    const float z1 = r0 * std::sin(theta0) * stddev + mean;
    const float r1 = std::sqrt(-2.0f * std::log(u2));
    const float theta1 = kTwoPi * u3;
    const float z2 = r1 * std::cos(theta1) * stddev + mean;
    const float z3 = r1 * std::sin(theta1) * stddev + mean;
    const std::size_t base = static_cast<std::size_t>(i) * 4;
    if (base < n) out[base] = z0;
    if (base + 1 < n) out[base + 1] = z1;
    if (base + 2 < n) out[base + 2] = z2;
    if (base + 3 < n) out[base + 3] = z3;
  });
  return offset + static_cast<std::uint64_t>(rounds) * 4;
}

// Philox blocks at arbitrary counters (for sampled checks of full-size streams).
extern "C" void oracle_philox_gather(const uint64_t* ctrs, size_t m, uint64_t seed, uint32_t* out,
                                     int threads) {
  oracle_detail::parallel_for(0, static_cast<std::int64_t>(m), threads, [&](std::int64_t i) {
    oracle_philox_block(ctrs[i], seed, out + 4 * i);
  });
}
