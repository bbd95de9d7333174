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
// the 148 SMs and strides over the output.
//
// The normal transform is bound by instruction issue and by the heavy FMA pipe, which
// Philox's twenty 32x32->64 multiplies per block already hold for 80 of the 91
// cycles a warp-block may take at the HBM write rate.  So its fp32 work is written
// to leave that pipe: the two Box-Muller pairs of a block are the two lanes of
// sm_100's packed add/mul/fma.rn.f32x2 (each lane rounded exactly as the scalar
// instruction), and -2 ln u, sin and cos come from the hardware's approximate
// lg2 / sin / cos (XU pipe) wherever those are accurate enough, with this file's own
// bounded-range series elsewhere (see kHw below):
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

// A pair of fp32 lanes.  With P (packed) an operation is one add/mul/fma.rn.f32x2
// instruction: one issue slot, but it holds both FMA pipes for two cycles.
// Without P it is two scalar instructions, each free to run on whichever FMA pipe
// is idle.  Philox's wide multiplies keep the heavy FMA pipe busy, so the fastest
// mix of the two forms is a per-stage choice (kPack* below).  Both forms round
// each lane exactly as the scalar round-to-nearest instruction does.
struct Pair {
  float x, y;
};

__device__ __forceinline__ Pair splat(float c) { return {c, c}; }

__device__ __forceinline__ unsigned long long pack(Pair a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
__device__ __forceinline__ Pair unpack(unsigned long long v) {
  Pair r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

template <bool P>
__device__ __forceinline__ Pair add(Pair a, Pair b) {
  if constexpr (P) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack(a)), "l"(pack(b)));
    return unpack(d);
  } else {
    return {__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)};
  }
}
template <bool P>
__device__ __forceinline__ Pair mul(Pair a, Pair b) {
  if constexpr (P) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack(a)), "l"(pack(b)));
    return unpack(d);
  } else {
    return {__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)};
  }
}
template <bool P>
__device__ __forceinline__ Pair fma(Pair a, Pair b, Pair c) {
  if constexpr (P) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pack(a)), "l"(pack(b)), "l"(pack(c)));
    return unpack(d);
  } else {
    return {__fmaf_rn(a.x, b.x, c.x), __fmaf_rn(a.y, b.y, c.y)};
  }
}

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float lg2_approx(float x) {
  float r;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float sin_approx(float x) {
  float r;
  asm("sin.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float cos_approx(float x) {
  float r;
  asm("cos.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Which stages of the transforms use the packed form (bit set) or scalar pairs.
constexpr unsigned kPackConv = 1u;   // word -> uniform float
constexpr unsigned kPackLog = 2u;    // -2 ln u
constexpr unsigned kPackTrig = 4u;   // reduction and sin/cos polynomials
constexpr unsigned kPackOut = 8u;    // radius products and the affine step
// With kHw the normal transform takes -2 ln u and sin / cos from the hardware's
// approximate lg2 / sin / cos (the XU pipe, off the FMA pipes that Philox's
// multiplies fill), keeping this file's series for the inputs where those are not
// accurate enough (see neg2_log_hw and polar2_hw).
constexpr unsigned kHw = 16u;

// (float(u) + 1.0f) * 2^-32 for two words.  Evaluated as fma(float(u), 2^-32, 2^-32):
// scaling by a power of two commutes with rounding (no underflow: the sum is at
// least 1), so the single rounding of the fma equals the reference's rounded add
// followed by its exact multiply, bit for bit.
template <bool P>
__device__ __forceinline__ Pair to_uniform2(std::uint32_t a, std::uint32_t b) {
  return fma<P>({__uint2float_rn(a), __uint2float_rn(b)}, splat(2.3283064365386963e-10f),
                splat(2.3283064365386963e-10f));
}

// -2 ln u for u in (0, 1] in both lanes (u = 1 gives -0, whose square root is
// -0 and whose products become +0 once the mean is added, as in the reference).
// The exponent e (|e| <= 32) is made a float exactly through the 2^23 bias; the
// factor -2 is folded into the series coefficients, which is exact.
template <bool P>
__device__ __forceinline__ Pair neg2_log(Pair u) {
  constexpr std::uint32_t kSqrtHalf = 0x3F3504F3u;  // bits of sqrt(1/2)
  constexpr std::uint32_t kBias = 64u << 23;        // keeps the shifted exponent positive
  const std::uint32_t ba = __float_as_uint(u.x), bb = __float_as_uint(u.y);
  const std::uint32_t ea = (ba - kSqrtHalf + kBias) >> 23;  // e + 64
  const std::uint32_t eb = (bb - kSqrtHalf + kBias) >> 23;
  const Pair e = add<P>({__uint_as_float(0x4B000000u | ea), __uint_as_float(0x4B000000u | eb)},
                        splat(-8388672.0f));  // 2^23 + 64
  const Pair m = {__uint_as_float(ba + kBias - (ea << 23)),
                  __uint_as_float(bb + kBias - (eb << 23))};
  const Pair num = add<P>(m, splat(-1.0f));
  const Pair den = add<P>(m, splat(1.0f));
  const Pair s = mul<P>(num, {rcp_approx(den.x), rcp_approx(den.y)});
  const Pair z = mul<P>(s, s);
  // atanh(s)/s = 1 + z (c1 + c2 z) on z <= 0.02944 (near-minimax fit of this file's
  // own, 4.7e-7 relative error), times -4 so that -2 ln m = s (-4 + z q)
  const Pair q = fma<P>(splat(-4.0f * 0.20429936f), z, splat(-4.0f * 0.33331743f));
  const Pair lnm = mul<P>(s, fma<P>(z, q, splat(-4.0f)));  // -2 ln m
  return fma<P>(e, splat(-1.38629436111989061883f), lnm);  // -2 ln 2 (exactly twice float ln 2)
}

// theta in [0, 2pi] -> x = theta - j pi/2 with |x| <= pi/4 (Cody-Waite, two-term pi/2,
// j <= 4) and the bits of the rounded sum, whose low two bits are j mod 4.
template <bool PT>
__device__ __forceinline__ Pair reduce_quadrant(Pair theta, std::uint32_t (&q)[2]) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
  const Pair magic = fma<PT>(theta, splat(0.636619772367581343076f), splat(kRound));  // 2/pi
  const Pair j = add<PT>(magic, splat(-kRound));
  Pair x = fma<PT>(j, splat(-1.57079637050628662109375f), theta);  // float(pi/2)
  x = fma<PT>(j, splat(4.37113900018624283e-8f), x);               // pi/2 - float(pi/2), negated
  q[0] = __float_as_uint(magic.x);
  q[1] = __float_as_uint(magic.y);
  return x;
}

// sin and cos of |x| <= pi/4 by near-minimax odd / even polynomials (fits of this
// file's own: sin 1e-8, cos 3.3e-8 absolute error).
template <bool PT>
__device__ __forceinline__ void sincos_poly(Pair x, Pair& sn, Pair& cs) {
  const Pair x2 = mul<PT>(x, x);
  Pair p = fma<PT>(splat(-1.958967769e-4f), x2, splat(8.332764730e-3f));
  p = fma<PT>(p, x2, splat(-1.666666567e-1f));
  sn = fma<PT>(mul<PT>(x, x2), p, x);
  Pair c = fma<PT>(splat(-1.359708956e-3f), x2, splat(4.165624082e-2f));
  c = fma<PT>(c, x2, splat(-4.999989271e-1f));
  cs = fma<PT>(c, x2, splat(1.0f));
}

// r*cos(theta) and r*sin(theta) from sin / cos of the reduced angle: quadrant j
// (low bits of q) gives cos = [c, -s, -c, s][j & 3], sin = [s, c, -s, -c][j & 3]; the
// signs are folded into the radius.
template <bool PO>
__device__ __forceinline__ void rotate_quadrant(const std::uint32_t (&q)[2], Pair sn, Pair cs,
                                                Pair r, Pair& zc, Pair& zs) {
  const float csl[2] = {cs.x, cs.y}, snl[2] = {sn.x, sn.y}, rl[2] = {r.x, r.y};
  float cv[2], sv[2], rc[2], rs[2];
#pragma unroll
  for (int l = 0; l < 2; ++l) {
    const bool swap = (q[l] & 1u) != 0u;
    cv[l] = swap ? snl[l] : csl[l];
    sv[l] = swap ? csl[l] : snl[l];
    const std::uint32_t rb = __float_as_uint(rl[l]);
    rs[l] = __uint_as_float(rb ^ ((q[l] << 30) & 0x80000000u));
    rc[l] = __uint_as_float(rb ^ (((q[l] + 1u) << 30) & 0x80000000u));
  }
  zc = mul<PO>({rc[0], rc[1]}, {cv[0], cv[1]});
  zs = mul<PO>({rs[0], rs[1]}, {sv[0], sv[1]});
}

// r*cos(theta) and r*sin(theta), theta in [0, 2pi], both lanes.
template <bool PT, bool PO>
__device__ __forceinline__ void polar2(Pair theta, Pair r, Pair& zc, Pair& zs) {
  std::uint32_t q[2];
  const Pair x = reduce_quadrant<PT>(theta, q);
  Pair sn, cs;
  sincos_poly<PT>(x, sn, cs);
  rotate_quadrant<PO>(q, sn, cs, r, zc, zs);
}

// ---- hardware-approximation variant of the normal transform (kHw) --------------
// The error bound of the transform is 2e-6 * max(1, |z|) against the reference
// formula.  Measured over every fp32 input each step can see (all u in [2^-32, 1],
// all reduced angles |x| <= pi/2):
//   sin.approx / cos.approx of x: at most 3.65e-7 absolute;
//   lg2.approx(u) * -2 ln 2: accurate relative to w = -2 ln u except near u = 1,
//     where lg2 of a mantissa near 2 cancels; for u > kNearOne the series
//     w = d (-2 + d (1 + d (-2/3 + d / 2))) in d = u - 1 (exact) is used instead
//     (2.7e-9 absolute); with that split the radius r = sqrt(w) is within
//     3.5e-7 * max(1, r) of sqrt(-2 ln u).
// z = r cos(theta) then errs by at most 3.5e-7 max(1, r)|cos| + r * 3.65e-7 (+ the
// product's rounding), which stays below 2e-6 max(1, |z|) for r <= kRadHw = 3.75;
// lanes with a larger radius (u < exp(-7.03), one pair in 1100) take this file's
// polynomials for sin / cos.  Both fallbacks are taken per warp only when one of
// its lanes needs them.
constexpr float kNearOne = 0.995f;
constexpr float kRadHw = 3.75f;

template <bool P>
__device__ __forceinline__ Pair neg2_log_hw(Pair u) {
  Pair w = mul<P>({lg2_approx(u.x), lg2_approx(u.y)}, splat(-1.38629436111989061883f));
  const bool nx = u.x > kNearOne, ny = u.y > kNearOne;
  if (__any_sync(__activemask(), nx || ny)) {
    const Pair d = add<P>(u, splat(-1.0f));
    const Pair q = fma<P>(d, splat(0.5f), splat(-0.6666666865f));
    const Pair sr = mul<P>(d, fma<P>(d, fma<P>(d, q, splat(1.0f)), splat(-2.0f)));
    if (nx) w.x = sr.x;
    if (ny) w.y = sr.y;
  }
  return w;
}

// r*cos(theta) and r*sin(theta) with the hardware sin / cos: theta is reduced by
// pi (x = theta - k pi, |x| <= pi/2, two-term pi), so cos and sin of theta are those
// of x with one common sign (-1)^k, folded into the radius.
template <bool PT, bool PO>
__device__ __forceinline__ void polar2_hw(Pair theta, Pair r, Pair& zc, Pair& zs) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
  const Pair magic = fma<PT>(theta, splat(0.318309886183790671538f), splat(kRound));  // 1/pi
  const Pair k = add<PT>(magic, splat(-kRound));
  Pair x = fma<PT>(k, splat(-3.1415927410125732421875f), theta);  // float(pi)
  x = fma<PT>(k, splat(8.74227800037248566e-8f), x);              // pi - float(pi), negated
  const Pair rk = {__uint_as_float(__float_as_uint(r.x) ^ (__float_as_uint(magic.x) << 31)),
                   __uint_as_float(__float_as_uint(r.y) ^ (__float_as_uint(magic.y) << 31))};
  zc = mul<PO>(rk, {cos_approx(x.x), cos_approx(x.y)});
  zs = mul<PO>(rk, {sin_approx(x.x), sin_approx(x.y)});
  const bool fx = r.x > kRadHw, fy = r.y > kRadHw;
  if (__any_sync(__activemask(), fx || fy)) {
    // large radius: this file's polynomials on the pi/2 reduction
    Pair pc, ps;
    polar2<PT, PO>(theta, r, pc, ps);
    if (fx) {
      zc.x = pc.x;
      zs.x = ps.x;
    }
    if (fy) {
      zc.y = pc.y;
      zs.y = ps.y;
    }
  }
}

template <Dist D, bool Scale, unsigned Pack>
__device__ __forceinline__ uint4 transform(uint4 r, float mean, float stddev) {
  constexpr bool PC = (Pack & kPackConv) != 0u, PL = (Pack & kPackLog) != 0u;
  constexpr bool PT = (Pack & kPackTrig) != 0u, PO = (Pack & kPackOut) != 0u;
  if constexpr (D == Dist::kLogNormal) {
    const uint4 z = transform<Dist::kNormal, Scale, Pack>(r, mean, stddev);
    return make_uint4(__float_as_uint(expf(__uint_as_float(z.x))),
                      __float_as_uint(expf(__uint_as_float(z.y))),
                      __float_as_uint(expf(__uint_as_float(z.z))),
                      __float_as_uint(expf(__uint_as_float(z.w))));
  } else if constexpr (D == Dist::kUint32) {
    return r;
  } else if constexpr (D == Dist::kUniform) {
    const Pair a = to_uniform2<PC>(r.x, r.y), b = to_uniform2<PC>(r.z, r.w);
    return make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x),
                      __float_as_uint(b.y));
  } else {
    // lane x is the pair (u0, u1), lane y the pair (u2, u3)
    constexpr bool HW = (Pack & kHw) != 0u;
    const Pair ue = to_uniform2<PC>(r.x, r.z), uo = to_uniform2<PC>(r.y, r.w);
    const Pair w = HW ? neg2_log_hw<PL>(ue) : neg2_log<PL>(ue);
    const Pair rad = {sqrt_approx(w.x), sqrt_approx(w.y)};
    const Pair theta = mul<PT>(splat(6.28318530717958647692f), uo);
    Pair zc, zs;
    if constexpr (HW)
      polar2_hw<PT, PO>(theta, rad, zc, zs);
    else
      polar2<PT, PO>(theta, rad, zc, zs);
    if constexpr (Scale) {
      zc = mul<PO>(zc, splat(stddev));
      zs = mul<PO>(zs, splat(stddev));
    }
    // (z * stddev) + mean, rounded separately; with stddev == 1 the product is z
    zc = add<PO>(zc, splat(mean));
    zs = add<PO>(zs, splat(mean));
    return make_uint4(__float_as_uint(zc.x), __float_as_uint(zs.x), __float_as_uint(zc.y),
                      __float_as_uint(zs.y));
  }
}

// Packing chosen by measurement on B200 (2^30 words, 8 CTAs per SM): the normal's
// 16 mixes ran 1.368 (conversion, log and output packed, trig scalar) to 1.605 ms
// (output and conversion packed only); all-packed 1.400, all-scalar 1.521.  The
// uniform conversion: packed 0.745 ms, scalar 0.805 ms.
// The log-normal (2^28 words, stddev != 1): all four stages packed 0.408 ms, the
// normal's mix 0.418 ms, all scalar 0.442 ms.
constexpr unsigned kUniformPack = kPackConv;
constexpr unsigned kNormalPack = kHw | kPackConv | kPackLog | kPackTrig | kPackOut;
constexpr unsigned kLogNormalPack = kPackConv | kPackLog | kPackTrig | kPackOut;

// Writes one Philox block's four words at block index b.
template <bool Vec16>
__device__ __forceinline__ void store_block(std::uint32_t* out, std::uint64_t b, uint4 v) {
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

// One thread per Philox block, grid-stride.  Vec16 selects a single 16-byte
// store per block (output 16-byte aligned); otherwise four 4-byte stores.
// Scale is false when stddev == 1 (the multiply is then the identity).  The
// uint32 and uniform streams take two blocks (b and b + stride) per loop step,
// which measured 3.4 % faster for the uniform (less loop overhead on the pipe the
// Philox multiplies fill); for the normal it measured slower and is not used.
template <Dist D, bool Vec16, bool Scale = true,
          unsigned Pack = (D == Dist::kNormal      ? kNormalPack
                           : D == Dist::kLogNormal ? kLogNormalPack
                                                   : kUniformPack)>
__global__ void __launch_bounds__(kThreads) philox_fill_kernel(const FillArgs a) {
  constexpr bool kPairs = D == Dist::kUniform || D == Dist::kUint32;
  const std::uint64_t full_blocks = a.n >> 2;
  const std::uint64_t stride = static_cast<std::uint64_t>(gridDim.x) * kThreads;
  std::uint64_t b = static_cast<std::uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  std::uint32_t* out = static_cast<std::uint32_t*>(a.out);
  if constexpr (kPairs) {
    for (; b + stride < full_blocks; b += 2 * stride) {
      const uint4 v0 = transform<D, Scale, Pack>(philox_block(a.first_block + b, a.key), a.mean,
                                                 a.stddev);
      const uint4 v1 = transform<D, Scale, Pack>(philox_block(a.first_block + b + stride, a.key),
                                                 a.mean, a.stddev);
      store_block<Vec16>(out, b, v0);
      store_block<Vec16>(out, b + stride, v1);
    }
  }
  for (; b < full_blocks; b += stride) {
    const uint4 v = transform<D, Scale, Pack>(philox_block(a.first_block + b, a.key), a.mean, a.stddev);
    store_block<Vec16>(out, b, v);
  }
  // The partial last block (n % 4 words) belongs to the thread whose next
  // grid-stride index is exactly full_blocks.
  const unsigned rem = static_cast<unsigned>(a.n & 3u);
  if (rem != 0 && b == full_blocks) {
    const uint4 v = transform<D, Scale, Pack>(philox_block(a.first_block + b, a.key), a.mean, a.stddev);
    std::uint32_t* p = out + 4 * b;
    p[0] = v.x;
    if (rem > 1) p[1] = v.y;
    if (rem > 2) p[2] = v.z;
  }
}

template <Dist D>
cudaError_t launch_dist(const FillArgs& a, bool vec16, unsigned grid, cudaStream_t stream) {
  const bool scale = (D == Dist::kNormal || D == Dist::kLogNormal) && a.stddev != 1.0f;
  if (vec16) {
    if (scale)
      philox_fill_kernel<D, true, true><<<grid, kThreads, 0, stream>>>(a);
    else
      philox_fill_kernel<D, true, false><<<grid, kThreads, 0, stream>>>(a);
  } else {
    if (scale)
      philox_fill_kernel<D, false, true><<<grid, kThreads, 0, stream>>>(a);
    else
      philox_fill_kernel<D, false, false><<<grid, kThreads, 0, stream>>>(a);
  }
  return cudaGetLastError();
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
    case Dist::kLogNormal:
      return launch_dist<Dist::kLogNormal>(a, vec16, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
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
