// philox.cpp — restatement of the reference's host Philox4x32-10 generator.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Follows libraries/rand/src/curand_context.mm operation by operation:
//   PhiloxHostStep        curand_context.mm:42-73
//   GenerateHostUint      curand_context.mm:75-93
//   GenerateHostUniform   curand_context.mm:95-113
//   GenerateHostNormal    curand_context.mm:145-185
//   GenerateHostUniformDouble / NormalDouble / LogNormal(Double)
//                         curand_context.mm:115-143, 187-247
//   Poisson               curand_kernels.metal:212-264 (device kernel) and
//                         curand_context.mm:249-293 (host path, mode 1)
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

// Counter (ctr_idx low, ctr_idx high, c2, 0).
extern "C" void oracle_philox_block4(uint64_t ctr_idx, uint32_t c2, uint64_t seed, uint32_t out[4]) {
  std::uint32_t ctr[4] = {static_cast<std::uint32_t>(ctr_idx),
                          static_cast<std::uint32_t>(ctr_idx >> 32), c2, 0u};
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

extern "C" void oracle_philox_block(uint64_t ctr_idx, uint64_t seed, uint32_t out[4]) {
  oracle_philox_block4(ctr_idx, 0u, seed, out);
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

// GenerateHostLogNormal (curand_context.mm:225-235): the normal stream, then exp.
extern "C" uint64_t oracle_generate_lognormal(uint64_t seed, uint64_t offset, float* out, size_t n,
                                              float mean, float stddev, int threads) {
  const uint64_t next = oracle_generate_normal(seed, offset, out, n, mean, stddev, threads);
  for (size_t i = 0; i < n; ++i) out[i] = std::exp(out[i]);
  return next;
}

namespace {

constexpr double kTwoPowMinus53 = 1.1102230246251565404236316680908203125e-16;
constexpr double kTwoPiD = 6.283185307179586476925286766559;

inline double uniform53(std::uint32_t hi, std::uint32_t lo) {
  const std::uint64_t m =
      ((static_cast<std::uint64_t>(hi) << 21) ^ static_cast<std::uint64_t>(lo)) &
      0x1FFFFFFFFFFFFFull;
  return (static_cast<double>(m) + 1.0) * kTwoPowMinus53;
}

}  // namespace

// kind 0 uniform, 1 normal, 2 log-normal (curand_context.mm:115-143, 187-223, 237-247):
// block i + offset / 2 gives out[2i], out[2i + 1].
extern "C" uint64_t oracle_generate_double(uint64_t seed, uint64_t offset, double* out, size_t n,
                                           int kind, double mean, double stddev, int threads) {
  const std::int64_t rounds = static_cast<std::int64_t>((n + 1) / 2);
  oracle_detail::parallel_for(0, rounds, threads, [&](std::int64_t i) {
    std::uint32_t r[4];
    oracle_philox_block(static_cast<std::uint64_t>(i) + (offset >> 1), seed, r);
    const double u0 = uniform53(r[0], r[1]);
    const double u1 = uniform53(r[2], r[3]);
    double z0 = u0, z1 = u1;
    if (kind != 0) {
      const double rv = std::sqrt(-2.0 * std::log(u0));
      const double theta = kTwoPiD * u1;
      z0 = rv * std::cos(theta) * stddev + mean;
      z1 = rv * std::sin(theta) * stddev + mean;
      if (kind == 2) {
        z0 = std::exp(z0);
        z1 = std::exp(z1);
      }
    }
    const std::size_t base = static_cast<std::size_t>(i) * 2;
    out[base] = z0;
    if (base + 1 < n) out[base + 1] = z1;
  });
  return offset + static_cast<std::uint64_t>(rounds) * 2;
}

// Poisson counts.  mode 0, the device kernel (curand_kernels.metal:212-264) and this
// library's host generators: output i uses blocks (i + offset, 0, s, 0), fp32
// arithmetic, threshold exp_neg_lambda (the library rounds exp(-lambda) once from
// double).  mode 1, the reference's host path (curand_context.mm:249-293): double
// arithmetic, extra blocks at counter i + offset + s * 2^32.
extern "C" uint64_t oracle_generate_poisson(uint64_t seed, uint64_t offset, uint32_t* out,
                                            size_t n, double lambda, float exp_neg_lambda,
                                            int mode, int threads) {
  oracle_detail::parallel_for(0, static_cast<std::int64_t>(n), threads, [&](std::int64_t i) {
    const std::uint64_t ctr = static_cast<std::uint64_t>(i) + offset;
    std::uint32_t r[4];
    oracle_philox_block(ctr, seed, r);
    if (mode == 0) {
      const float lf = static_cast<float>(lambda);
      if (lf < 30.0f) {
        float p = 1.0f;
        unsigned int k = 0, sub = 0, word = 0;
        while (p > exp_neg_lambda && k < 1000u) {
          ++k;
          p *= uniform_of(r[word]);
          if (++word == 4) {
            word = 0;
            oracle_philox_block4(ctr, ++sub, seed, r);
          }
        }
        out[i] = k > 0 ? k - 1 : 0u;
      } else {
        const float z = std::sqrt(-2.0f * std::log(uniform_of(r[0]))) *
                        std::cos(kTwoPi * uniform_of(r[1]));
        const float val = lf + std::sqrt(lf) * z + 0.5f;
        out[i] = val > 0.0f ? static_cast<unsigned int>(val) : 0u;
      }
    } else {
      const double u32 = 2.3283064365386962890625e-10;
      if (lambda < 30.0) {
        const double L = std::exp(-lambda);
        double p = 1.0;
        unsigned int k = 0, sub = 0;
        std::uint64_t sub_ctr = ctr;
        while (p > L && k < 1000u) {
          ++k;
          p *= (static_cast<double>(r[sub % 4]) + 1.0) * u32;
          ++sub;
          if (sub % 4 == 0) {
            sub_ctr += 0x100000000ull;
            oracle_philox_block(sub_ctr, seed, r);
          }
        }
        out[i] = k > 0 ? k - 1 : 0u;
      } else {
        const double u0 = (static_cast<double>(r[0]) + 1.0) * u32;
        const double u1 = (static_cast<double>(r[1]) + 1.0) * u32;
        const double z = std::sqrt(-2.0 * std::log(u0)) * std::cos(kTwoPiD * u1);
        const double val = lambda + std::sqrt(lambda) * z + 0.5;
        out[i] = val > 0.0 ? static_cast<unsigned int>(val) : 0u;
      }
    }
  });
  return offset + n;
}
