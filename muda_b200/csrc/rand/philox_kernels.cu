// philox_kernels.cu — Philox4x32-10 fill kernels for sm_100a.
//
// Arithmetic follows the reference generator operation by operation so that the
// uint32 and uniform streams are bit-identical to its host path:
//   round:    (hi(M1*c2) ^ c1 ^ k0, lo(M1*c2), hi(M0*c0) ^ c3 ^ k1, lo(M0*c0)),
//             M0 = 0xD2511F53, M1 = 0xCD9E8D57, then key += (0x9E3779B9, 0xBB67AE85)
//             (libraries/rand/src/curand_context.mm:42-73);
//   uniform:  (float(u) + 1.0f) * 2^-32, in (0, 1] (curand_context.mm:95-113);
//   normal:   Box-Muller on (u0,u1) and (u2,u3): r = sqrt(-2 ln u_even),
//             theta = 2pi_f * u_odd, z = (r*cos theta)*stddev + mean, (r*sin theta)*stddev + mean
//             (curand_context.mm:145-185).
// Every float operation of those formulas is issued with an explicit
// round-to-nearest intrinsic so that nvcc cannot contract it into an FMA.
//
// B200 layout: the 10-round key schedule is the same for every thread, so it is
// computed once on the host and read from the kernel parameter bank; each
// thread then owns whole Philox blocks and writes them as one 16-byte store, a
// warp covering 512 contiguous bytes.  The grid is a whole number of waves over
// the 148 SMs and strides over the output.
#include "rand/philox.hpp"

#include <cuda_runtime.h>

#include "common/device.hpp"

namespace mb200::rand {
namespace {

constexpr unsigned kThreads = 256;
constexpr unsigned kCtasPerSm = 8;

struct KeySchedule {
  std::uint32_t k0[10];
  std::uint32_t k1[10];
};

struct FillArgs {
  void* out;
  std::uint64_t n;
  std::uint64_t first_block;
  KeySchedule key;
  float mean;
  float stddev;
};

__device__ __forceinline__ uint4 philox_block(std::uint64_t ctr, const KeySchedule& key) {
  std::uint32_t c0 = static_cast<std::uint32_t>(ctr);
  std::uint32_t c1 = static_cast<std::uint32_t>(ctr >> 32);
  std::uint32_t c2 = 0u;
  std::uint32_t c3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const std::uint32_t hi0 = __umulhi(0xD2511F53u, c0);
    const std::uint32_t lo0 = 0xD2511F53u * c0;
    const std::uint32_t hi1 = __umulhi(0xCD9E8D57u, c2);
    const std::uint32_t lo1 = 0xCD9E8D57u * c2;
    c0 = hi1 ^ c1 ^ key.k0[r];
    c1 = lo1;
    c2 = hi0 ^ c3 ^ key.k1[r];
    c3 = lo0;
  }
  return make_uint4(c0, c1, c2, c3);
}

__device__ __forceinline__ float to_uniform(std::uint32_t u) {
  // (float(u) + 1.0f) * 2^-32 with each step rounded separately.
  return __fmul_rn(__fadd_rn(__uint2float_rn(u), 1.0f), 2.3283064365386963e-10f);
}

__device__ __forceinline__ float2 box_muller(float ua, float ub, float mean, float stddev) {
  const float r = sqrtf(__fmul_rn(-2.0f, logf(ua)));
  const float theta = __fmul_rn(6.28318530717958647692f, ub);
  float s, c;
  sincosf(theta, &s, &c);
  return make_float2(__fadd_rn(__fmul_rn(__fmul_rn(r, c), stddev), mean),
                     __fadd_rn(__fmul_rn(__fmul_rn(r, s), stddev), mean));
}

template <Dist D>
__device__ __forceinline__ uint4 transform(uint4 r, float mean, float stddev) {
  if constexpr (D == Dist::kUint32) {
    return r;
  } else if constexpr (D == Dist::kUniform) {
    return make_uint4(__float_as_uint(to_uniform(r.x)), __float_as_uint(to_uniform(r.y)),
                      __float_as_uint(to_uniform(r.z)), __float_as_uint(to_uniform(r.w)));
  } else {
    const float2 a = box_muller(to_uniform(r.x), to_uniform(r.y), mean, stddev);
    const float2 b = box_muller(to_uniform(r.z), to_uniform(r.w), mean, stddev);
    return make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x),
                      __float_as_uint(b.y));
  }
}

// One thread per Philox block, grid-stride.  Vec16 selects a single 16-byte
// store per block (output 16-byte aligned); otherwise four 4-byte stores.
template <Dist D, bool Vec16>
__global__ void __launch_bounds__(kThreads) philox_fill_kernel(const FillArgs a) {
  const std::uint64_t full_blocks = a.n >> 2;
  const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
  std::uint64_t b = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  std::uint32_t* out = static_cast<std::uint32_t*>(a.out);
  for (; b < full_blocks; b += stride) {
    const uint4 v = transform<D>(philox_block(a.first_block + b, a.key), a.mean, a.stddev);
    if constexpr (Vec16) {
      reinterpret_cast<uint4*>(out)[b] = v;
    } else {
      std::uint32_t* p = out + 4 * b;
      p[0] = v.x;
      p[1] = v.y;
      p[2] = v.z;
      p[3] = v.w;
    }
  }
  // The partial last block (n % 4 words) belongs to the thread whose next
  // grid-stride index is exactly full_blocks.
  const unsigned rem = static_cast<unsigned>(a.n & 3u);
  if (rem != 0 && b == full_blocks) {
    const uint4 v = transform<D>(philox_block(a.first_block + b, a.key), a.mean, a.stddev);
    std::uint32_t* p = out + 4 * b;
    p[0] = v.x;
    if (rem > 1) p[1] = v.y;
    if (rem > 2) p[2] = v.z;
  }
}

template <Dist D>
cudaError_t launch_dist(const FillArgs& a, bool vec16, unsigned grid, cudaStream_t stream) {
  if (vec16) {
    philox_fill_kernel<D, true><<<grid, kThreads, 0, stream>>>(a);
  } else {
    philox_fill_kernel<D, false><<<grid, kThreads, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace

int philox_fill_launch_count(std::uint64_t n) noexcept { return n == 0 ? 0 : 1; }

cudaError_t launch_philox_fill(Dist dist, void* out, std::uint64_t n, std::uint64_t seed,
                               std::uint64_t first_block, float mean, float stddev,
                               cudaStream_t stream) noexcept {
  if (n == 0) return cudaSuccess;
  FillArgs a{};
  a.out = out;
  a.n = n;
  a.first_block = first_block;
  a.mean = mean;
  a.stddev = stddev;
  std::uint32_t k0 = static_cast<std::uint32_t>(seed);
  std::uint32_t k1 = static_cast<std::uint32_t>(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    a.key.k0[r] = k0;
    a.key.k1[r] = k1;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return cudaErrorInvalidDevice;
  const std::uint64_t blocks = (n + 3) / 4;
  const std::uint64_t want = (blocks + kThreads - 1) / kThreads;
  const std::uint64_t cap = static_cast<std::uint64_t>(sms) * kCtasPerSm;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  const bool vec16 = aligned_to(out, 16);
  switch (dist) {
    case Dist::kUint32:
      return launch_dist<Dist::kUint32>(a, vec16, grid, stream);
    case Dist::kUniform:
      return launch_dist<Dist::kUniform>(a, vec16, grid, stream);
    case Dist::kNormal:
      return launch_dist<Dist::kNormal>(a, vec16, grid, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mb200::rand
