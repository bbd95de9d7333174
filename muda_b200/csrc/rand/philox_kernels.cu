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
// round-to-nearest instruction so that nvcc cannot contract it into an FMA.
//
// B200 layout: the 10-round key schedule is the same for every thread, so it is
// computed once on the host and read from the kernel parameter bank; each
// thread then owns whole Philox blocks and writes them as one 16-byte store, a
// warp covering 512 contiguous bytes.  The grid is a whole number of waves over
// the 148 SMs and strides over the output.  A call is cut on the host into segments
// within which the counter's high word is constant (at most 2^31 blocks each, almost
// always one launch): inside a segment the block counter is a 32-bit index, the high
// word a kernel constant that the first round folds, and no carry is propagated.
//
// The normal transform is bound by the FMA pipes, which Philox's twenty 32x32->64
// multiplies per block already hold for 80 of the 91 cycles a warp-block may take at
// the HBM write rate (per-opcode counts: every instruction the transform adds to those
// pipes costs about two cycles of elapsed time).  So its fp32 work is written to leave
// them: the two Box-Muller pairs of a block are the two lanes of sm_100's packed
// add/mul/fma.rn.f32x2 (each lane rounded exactly as the scalar instruction), the
// outputs are formed as (r cos, r sin) pairs that leave in store order, sign folds and
// threshold tests are integer instructions, and -2 ln u, sin and cos come from the
// hardware's approximate lg2 / sin / cos (XU pipe) wherever those are accurate enough,
// with this file's own bounded-range series elsewhere (box_muller.cuh):
//   -2 ln u, u in (0, 1]: u = m 2^e with m in [sqrt(1/2), sqrt(2)), ln m =
//      2 atanh(s) with s = (m-1)/(m+1), |s| <= 0.1716, atanh(s)/s as a quadratic in
//      s^2 (4.7e-7 relative); near u = 1 a series in d = u - 1;
//   cos, sin of theta in [0, 2pi]: Cody-Waite reduction r = theta - j pi/2 with a
//      two-term pi/2 (j <= 4), odd degree-7 and even degree-6 polynomials on
//      |r| <= pi/4 (1e-8 and 3.3e-8 absolute), then the quadrant's swap and signs.
// The polynomial coefficients are this file's own near-minimax fits (weighted
// least squares on Chebyshev nodes, reweighted toward the largest error).
// Against the reference formula evaluated with glibc's float functions the
// result stays within 2e-6 * max(1, |z|).
#include "rand/philox.hpp"

#include <cuda_runtime.h>

#include "common/device.hpp"
#include "rand/box_muller.cuh"

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
  double mean_d, stddev_d;    // double-precision streams
  float lambda, exp_neg_lambda;  // Poisson
  // fp32 segment (philox_fill_kernel): blocks i < nblk use the counter (clo + i, chi, 0, 0)
  // and go to out[4i .. 4i+3]; then `tail` (0..3) words of block nblk
  std::uint32_t nblk, clo, chi, tail;
};

// Counter (ctr_lo, ctr_hi, c2_in, 0): word 2 is 0 except for the Poisson
// stream's extra blocks.
__device__ __forceinline__ uint4 philox_block(std::uint64_t ctr, const KeySchedule& key,
                                              std::uint32_t c2_in = 0u) {
  std::uint32_t c0 = static_cast<std::uint32_t>(ctr);
  std::uint32_t c1 = static_cast<std::uint32_t>(ctr >> 32);
  std::uint32_t c2 = c2_in;
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

// The same rounds for the counter (lo, hi, 0, 0) with hi constant over a segment.
__device__ __forceinline__ uint4 philox_block32(std::uint32_t lo, std::uint32_t hi,
                                                const KeySchedule& key) {
  std::uint32_t c0 = lo, c1 = hi, c2 = 0u, c3 = 0u;
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


// Which stages of the transforms use the packed form (bit set) or scalar pairs.
constexpr unsigned kPackConv = 1u;   // word -> uniform float
constexpr unsigned kPackLog = 2u;    // -2 ln u
constexpr unsigned kPackTrig = 4u;   // reduction and sin/cos polynomials
constexpr unsigned kPackOut = 8u;    // radius products and the affine step

// uint32, uniform and log-normal words of one block.  The log-normal keeps this file's
// bounded-range series for ln / sin / cos (its exp amplifies the normal's error); the
// normal itself runs normal_block_hw (box_muller.cuh).
template <Dist D, bool Scale, unsigned Pack>
__device__ __forceinline__ uint4 transform(uint4 r, float mean, float stddev) {
  constexpr bool PC = (Pack & kPackConv) != 0u, PL = (Pack & kPackLog) != 0u;
  constexpr bool PT = (Pack & kPackTrig) != 0u, PO = (Pack & kPackOut) != 0u;
  if constexpr (D == Dist::kUint32) {
    return r;
  } else if constexpr (D == Dist::kUniform) {
    const Pair a = to_uniform2<PC>(r.x, r.y), b = to_uniform2<PC>(r.z, r.w);
    return make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x),
                      __float_as_uint(b.y));
  } else {
    static_assert(D == Dist::kLogNormal, "normal blocks go through normal_block_hw");
    // lane x is the pair (u0, u1), lane y the pair (u2, u3)
    const Pair ue = to_uniform2<PC>(r.x, r.z), uo = to_uniform2<PC>(r.y, r.w);
    const Pair w = neg2_log<PL>(ue);
    const Pair rad = {sqrt_approx(w.x), sqrt_approx(w.y)};
    const Pair theta = mul<PT>(splat(6.28318530717958647692f), uo);
    Pair zc, zs;
    polar2<PT, PO>(theta, rad, zc, zs);
    if constexpr (Scale) {
      zc = mul<PO>(zc, splat(stddev));
      zs = mul<PO>(zs, splat(stddev));
    }
    // (z * stddev) + mean, rounded separately; with stddev == 1 the product is z
    zc = add<PO>(zc, splat(mean));
    zs = add<PO>(zs, splat(mean));
    return make_uint4(__float_as_uint(expf(zc.x)), __float_as_uint(expf(zs.x)),
                      __float_as_uint(expf(zc.y)), __float_as_uint(expf(zs.y)));
  }
}

// Packing chosen by measurement on B200 (2^30 words, 8 CTAs per SM): the uniform
// conversion packed 0.745 ms, scalar 0.805 ms.  The log-normal (2^28 words, stddev != 1):
// all four stages packed 0.408 ms, all scalar 0.442 ms.
constexpr unsigned kUniformPack = kPackConv;
constexpr unsigned kLogNormalPack = kPackConv | kPackLog | kPackTrig | kPackOut;

// Aff: the affine step of the normal and log-normal words (0: none, mean 0 and stddev 1;
// 1: + mean; 2: * stddev + mean).
template <Dist D, int Aff>
__device__ __forceinline__ uint4 block_words(std::uint32_t lo, std::uint32_t hi,
                                             const FillArgs& a) {
  const uint4 r = philox_block32(lo, hi, a.key);
  if constexpr (D == Dist::kNormal)
    return normal_block_hw<Aff>(r, a.mean, a.stddev);
  else if constexpr (D == Dist::kLogNormal)
    return transform<D, Aff == 2, kLogNormalPack>(r, a.mean, a.stddev);
  else
    return transform<D, false, kUniformPack>(r, a.mean, a.stddev);
}

template <bool Vec16>
__device__ __forceinline__ void store_block(std::uint32_t* p, uint4 v) {
  if constexpr (Vec16) {
    *reinterpret_cast<uint4*>(p) = v;
  } else {
    p[0] = v.x;
    p[1] = v.y;
    p[2] = v.z;
    p[3] = v.w;
  }
}

// One segment (FillArgs::nblk blocks of constant counter high word), one thread per
// Philox block, grid-stride with a 32-bit block index, the output pointer and the
// counter stepped by the stride.  Vec16 selects a single 16-byte store per block
// (output 16-byte aligned); otherwise four 4-byte stores.  The uint32 and uniform
// streams take two blocks (b and b + stride) per loop step.  Measured on 2^30 words
// against the previous 64-bit-counter loop: uniform 0.776 -> 0.664 ms, normal (with
// normal_block_hw's pair layout and integer tests) 1.218 -> 1.057 ms.
template <Dist D, bool Vec16, int Aff>
__global__ void __launch_bounds__(kThreads) philox_fill_kernel(const FillArgs a) {
  constexpr bool kPairs = D == Dist::kUniform || D == Dist::kUint32;
  const std::uint32_t stride = gridDim.x * kThreads;
  std::uint32_t b = blockIdx.x * kThreads + threadIdx.x;
  std::uint32_t* p = static_cast<std::uint32_t*>(a.out) + 4ull * b;
  std::uint32_t c = a.clo + b;
  if constexpr (kPairs) {
    for (; b + stride < a.nblk; b += 2 * stride) {
      const uint4 v0 = block_words<D, Aff>(c, a.chi, a);
      const uint4 v1 = block_words<D, Aff>(c + stride, a.chi, a);
      store_block<Vec16>(p, v0);
      store_block<Vec16>(p + 4ull * stride, v1);
      p += 8ull * stride;
      c += 2 * stride;
    }
  }
  for (; b < a.nblk; b += stride) {
    store_block<Vec16>(p, block_words<D, Aff>(c, a.chi, a));
    p += 4ull * stride;
    c += stride;
  }
  // The partial last block (tail words) belongs to the thread whose next grid-stride
  // index is exactly nblk; the host keeps its counter inside the segment's high word.
  if (a.tail != 0 && b == a.nblk) {
    const uint4 v = block_words<D, Aff>(c, a.chi, a);
    p[0] = v.x;
    if (a.tail > 1) p[1] = v.y;
    if (a.tail > 2) p[2] = v.z;
  }
}

template <Dist D, int Aff>
cudaError_t launch_segment(const FillArgs& a, bool vec16, unsigned grid, cudaStream_t stream) {
  if (vec16)
    philox_fill_kernel<D, true, Aff><<<grid, kThreads, 0, stream>>>(a);
  else
    philox_fill_kernel<D, false, Aff><<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

template <Dist D>
cudaError_t launch_dist(const FillArgs& a, bool vec16, unsigned grid, cudaStream_t stream) {
  if constexpr (D == Dist::kNormal) {
    if (a.stddev != 1.0f) return launch_segment<D, 2>(a, vec16, grid, stream);
    if (a.mean != 0.0f) return launch_segment<D, 1>(a, vec16, grid, stream);
    return launch_segment<D, 0>(a, vec16, grid, stream);
  } else if constexpr (D == Dist::kLogNormal) {
    if (a.stddev != 1.0f) return launch_segment<D, 2>(a, vec16, grid, stream);
    return launch_segment<D, 1>(a, vec16, grid, stream);
  } else {
    return launch_segment<D, 0>(a, vec16, grid, stream);
  }
}

// ------------------------------------------------------ double precision --
// The 53-bit integers and the uniform (m + 1) * 2^-53 are exact, so that stream is
// bit-identical to the reference's; the normal uses the device's double log,
// sqrt and sincos (each within an ulp or two of the host's), every multiply and
// add of the formula rounded separately.
template <Dist D>
__device__ __forceinline__ double2 transform_f64(uint4 r, double mean, double stddev) {
  constexpr unsigned long long kMask = 0x1FFFFFFFFFFFFFull;
  constexpr double kTwoPowMinus53 = 1.1102230246251565404236316680908203125e-16;
  const unsigned long long m0 =
      ((static_cast<unsigned long long>(r.x) << 21) ^ static_cast<unsigned long long>(r.y)) & kMask;
  const unsigned long long m1 =
      ((static_cast<unsigned long long>(r.z) << 21) ^ static_cast<unsigned long long>(r.w)) & kMask;
  const double u0 = __dmul_rn(__dadd_rn(static_cast<double>(m0), 1.0), kTwoPowMinus53);
  const double u1 = __dmul_rn(__dadd_rn(static_cast<double>(m1), 1.0), kTwoPowMinus53);
  if constexpr (D == Dist::kUniformDouble) {
    return make_double2(u0, u1);
  } else {
    const double rad = sqrt(__dmul_rn(-2.0, log(u0)));
    const double theta = __dmul_rn(6.283185307179586476925286766559, u1);
    double sn, cs;
    sincos(theta, &sn, &cs);
    double z0 = __dadd_rn(__dmul_rn(__dmul_rn(rad, cs), stddev), mean);
    double z1 = __dadd_rn(__dmul_rn(__dmul_rn(rad, sn), stddev), mean);
    if constexpr (D == Dist::kLogNormalDouble) {
      z0 = exp(z0);
      z1 = exp(z1);
    }
    return make_double2(z0, z1);
  }
}

template <Dist D, bool Vec16>
__global__ void __launch_bounds__(kThreads) philox_fill_f64_kernel(const FillArgs a) {
  const std::uint64_t full_blocks = a.n >> 1;
  const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
  std::uint64_t b = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  double* out = static_cast<double*>(a.out);
  for (; b < full_blocks; b += stride) {
    const double2 v = transform_f64<D>(philox_block(a.first_block + b, a.key), a.mean_d, a.stddev_d);
    if constexpr (Vec16) {
      reinterpret_cast<double2*>(out)[b] = v;
    } else {
      out[2 * b] = v.x;
      out[2 * b + 1] = v.y;
    }
  }
  if ((a.n & 1u) != 0 && b == full_blocks)
    out[2 * b] = transform_f64<D>(philox_block(a.first_block + b, a.key), a.mean_d, a.stddev_d).x;
}

// --------------------------------------------------------------- Poisson --
__device__ __forceinline__ float uniform_of(std::uint32_t v) {
  return __fmul_rn(__fadd_rn(static_cast<float>(v), 1.0f), 2.3283064365386963e-10f);
}

// Output i draws Knuth's product from its own stream: block ctr = first_block + i,
// then (ctr, c2 = 1, 2, ...) while more words are needed; k counts the factors until
// the product falls to exp(-lambda) or below.  Each step of a thread's loop computes
// one Philox block of its current output and takes up to four factors from it; a
// thread whose output ends writes it and starts its next output at the next step.
// So a warp runs about as many steps as its lanes' own outputs need, instead of the
// longest of 32 outputs each time (the Philox arithmetic never diverges), and no
// block is computed that is not used.
__global__ void __launch_bounds__(kThreads) philox_poisson_kernel(const FillArgs a) {
  const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
  unsigned int* out = static_cast<unsigned int*>(a.out);
  std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (a.lambda >= 30.0f) {
    for (; i < a.n; i += stride) {
      const uint4 r = philox_block(a.first_block + i, a.key);
      const float u0 = uniform_of(r.x), u1 = uniform_of(r.y);
      const float z = __fmul_rn(sqrtf(__fmul_rn(-2.0f, logf(u0))),
                                cosf(__fmul_rn(6.28318530717958647692f, u1)));
      const float val = __fadd_rn(__fadd_rn(a.lambda, __fmul_rn(sqrtf(a.lambda), z)), 0.5f);
      out[i] = val > 0.0f ? static_cast<unsigned int>(val) : 0u;
    }
    return;
  }
  float p = 1.0f;
  unsigned int k = 0, sub = 0;
  while (i < a.n) {
    const uint4 r = philox_block(a.first_block + i, a.key, sub);
    const std::uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (p > a.exp_neg_lambda && k < 1000u) {
        ++k;
        p = __fmul_rn(p, uniform_of(w[j]));
      }
    }
    if (p > a.exp_neg_lambda && k < 1000u) {
      ++sub;  // the same output needs the next block of its stream
    } else {
      out[i] = k > 0 ? k - 1 : 0u;
      i += stride;
      p = 1.0f;
      k = 0;
      sub = 0;
    }
  }
}

KeySchedule key_schedule(std::uint64_t seed) {
  KeySchedule k{};
  std::uint32_t k0 = static_cast<std::uint32_t>(seed);
  std::uint32_t k1 = static_cast<std::uint32_t>(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    k.k0[r] = k0;
    k.k1[r] = k1;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return k;
}

unsigned grid_for(std::uint64_t threads) {
  const int sms = sm_count(current_device());
  const std::uint64_t want = (threads + kThreads - 1) / kThreads;
  const std::uint64_t cap = static_cast<std::uint64_t>(sms > 0 ? sms : 148) * kCtasPerSm;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

template <Dist D>
cudaError_t launch_f64(const FillArgs& a, cudaStream_t stream) {
  const unsigned grid = grid_for((a.n + 1) / 2);
  if (aligned_to(a.out, 16))
    philox_fill_f64_kernel<D, true><<<grid, kThreads, 0, stream>>>(a);
  else
    philox_fill_f64_kernel<D, false><<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}


// The fp32 fill's segments: runs of at most 2^31 blocks whose counters share their high
// word, the partial last block (n % 4 words) inside the last run, or alone when the last
// run ends exactly where the high word changes.  Calls fn(first block, blocks, tail,
// word offset) for each.
template <class Fn>
cudaError_t for_each_segment(std::uint64_t n, std::uint64_t first_block, Fn&& fn) {
  constexpr std::uint64_t kMaxSeg = 1ull << 31;
  std::uint64_t blk = first_block, left = n >> 2, word = 0;
  const auto tail = static_cast<std::uint32_t>(n & 3u);
  for (;;) {
    const std::uint64_t room = (1ull << 32) - (blk & 0xFFFFFFFFull);
    const std::uint64_t seg = left < room ? (left < kMaxSeg ? left : kMaxSeg)
                                          : (room < kMaxSeg ? room : kMaxSeg);
    const bool last = seg == left;
    const bool tail_here = last && tail != 0 && seg < room;
    if (seg > 0 || tail_here) {
      const cudaError_t e = fn(blk, seg, tail_here ? tail : 0u, word);
      if (e != cudaSuccess) return e;
    }
    blk += seg;
    left -= seg;
    word += 4 * seg;
    if (last) {
      if (tail != 0 && !tail_here) return fn(blk, 0, tail, word);
      return cudaSuccess;
    }
  }
}

}  // namespace

int philox_fill_launch_count(std::uint64_t n, std::uint64_t first_block) noexcept {
  int count = 0;
  if (n == 0) return 0;
  for_each_segment(n, first_block, [&](std::uint64_t, std::uint64_t, std::uint32_t,
                                       std::uint64_t) {
    ++count;
    return cudaSuccess;
  });
  return count;
}

cudaError_t launch_philox_fill(Dist dist, void* out, std::uint64_t n, std::uint64_t seed,
                               std::uint64_t first_block, float mean, float stddev,
                               cudaStream_t stream) noexcept {
  if (n == 0) return cudaSuccess;
  FillArgs a{};
  a.n = n;
  a.first_block = first_block;
  a.mean = mean;
  a.stddev = stddev;
  a.key = key_schedule(seed);
  const int dev = current_device();
  const int sms = sm_count(dev);
  if (sms <= 0) return cudaErrorInvalidDevice;
  const std::uint64_t cap = static_cast<std::uint64_t>(sms) * kCtasPerSm;
  const bool vec16 = aligned_to(out, 16);
  return for_each_segment(n, first_block, [&](std::uint64_t blk, std::uint64_t seg,
                                              std::uint32_t tail, std::uint64_t word) {
    FillArgs s = a;
    s.out = static_cast<std::uint32_t*>(out) + word;
    s.nblk = static_cast<std::uint32_t>(seg);
    s.clo = static_cast<std::uint32_t>(blk);
    s.chi = static_cast<std::uint32_t>(blk >> 32);
    s.tail = tail;
    const std::uint64_t want = (seg + (tail != 0 ? 1 : 0) + kThreads - 1) / kThreads;
    const unsigned grid = static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
    switch (dist) {
      case Dist::kUint32:
        return launch_dist<Dist::kUint32>(s, vec16, grid, stream);
      case Dist::kUniform:
        return launch_dist<Dist::kUniform>(s, vec16, grid, stream);
      case Dist::kNormal:
        return launch_dist<Dist::kNormal>(s, vec16, grid, stream);
      case Dist::kLogNormal:
        return launch_dist<Dist::kLogNormal>(s, vec16, grid, stream);
      default:
        return cudaErrorInvalidValue;
    }
  });
}

cudaError_t launch_philox_fill_f64(Dist dist, double* out, std::uint64_t n, std::uint64_t seed,
                                   std::uint64_t first_block, double mean, double stddev,
                                   cudaStream_t stream) noexcept {
  if (n == 0) return cudaSuccess;
  if (!aligned_to(out, 8)) return cudaErrorInvalidValue;
  FillArgs a{};
  a.out = out;
  a.n = n;
  a.first_block = first_block;
  a.mean_d = mean;
  a.stddev_d = stddev;
  a.key = key_schedule(seed);
  switch (dist) {
    case Dist::kUniformDouble:
      return launch_f64<Dist::kUniformDouble>(a, stream);
    case Dist::kNormalDouble:
      return launch_f64<Dist::kNormalDouble>(a, stream);
    case Dist::kLogNormalDouble:
      return launch_f64<Dist::kLogNormalDouble>(a, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_philox_poisson(unsigned int* out, std::uint64_t n, std::uint64_t seed,
                                  std::uint64_t first_block, float lambda, float exp_neg_lambda,
                                  cudaStream_t stream) noexcept {
  if (n == 0) return cudaSuccess;
  FillArgs a{};
  a.out = out;
  a.n = n;
  a.first_block = first_block;
  a.lambda = lambda;
  a.exp_neg_lambda = exp_neg_lambda;
  a.key = key_schedule(seed);
  philox_poisson_kernel<<<grid_for(n), kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mb200::rand
