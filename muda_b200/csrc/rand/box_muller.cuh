// box_muller.cuh — device arithmetic of the cuRAND normal transform (sm_100a).
//
// Shared by the Philox fill kernels (rand/philox_kernels.cu) and the accuracy probe
// (probe/normal_probe.cu), so that the probe measures exactly the shipped code.
// Every function keeps the reference formulas' own roundings where the result must
// be reproduced bit for bit (the uniform conversion) and states its error bound
// where it approximates (ln, sin, cos); see philox_kernels.cu for the transform.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mb200::rand {
namespace {

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
// polynomials for sin / cos.  Both fallbacks are branches that a warp enters only when
// one of its lanes needs them.
constexpr float kNearOne = 0.995f;
constexpr float kRadHw = 3.75f;

// Bit 0 of x moved to bit 31 (a funnel shift: an integer-pipe instruction, which keeps
// the sign fold off the FMA pipes that Philox's multiplies fill).
__device__ __forceinline__ std::uint32_t low_bit_to_sign(std::uint32_t x) {
  std::uint32_t r;
  asm("shf.l.wrap.b32 %0, %1, %1, 31;" : "=r"(r) : "r"(x));
  return r & 0x80000000u;
}

// -2 ln u for u in (0, 1] in both lanes: the hardware lg2 times -2 ln 2, replaced by the
// series in d = u - 1 for u > kNearOne.  u is positive, so its bits order as its values
// and the test is an integer compare.
template <bool P>
__device__ __forceinline__ Pair neg2_log_hw(Pair u) {
  Pair w = mul<P>({lg2_approx(u.x), lg2_approx(u.y)}, splat(-1.38629436111989061883f));
  const bool nx = __float_as_uint(u.x) > __float_as_uint(kNearOne);
  const bool ny = __float_as_uint(u.y) > __float_as_uint(kNearOne);
  if (nx || ny) {
    const Pair d = add<P>(u, splat(-1.0f));
    const Pair q = fma<P>(d, splat(0.5f), splat(-0.6666666865f));
    const Pair sr = mul<P>(d, fma<P>(d, fma<P>(d, q, splat(1.0f)), splat(-2.0f)));
    if (nx) w.x = sr.x;
    if (ny) w.y = sr.y;
  }
  return w;
}

// The two Box-Muller pairs of a block as output pairs: p0 = (r.x cos theta.x,
// r.x sin theta.x), p1 = (r.y cos theta.y, r.y sin theta.y), theta in [0, 2pi], so that
// each product is one packed multiply and the four outputs leave in store order.  theta
// is reduced by pi (x = theta - k pi, |x| <= pi/2, two-term pi): cos and sin of theta are
// those of x with one common sign (-1)^k, folded into the radius.  Radii above kRadHw
// take this file's polynomials on the pi/2 reduction instead.
template <bool P>
__device__ __forceinline__ void polar_pairs_hw(Pair theta, Pair r, Pair& p0, Pair& p1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
  const Pair magic = fma<P>(theta, splat(0.318309886183790671538f), splat(kRound));  // 1/pi
  const Pair k = add<P>(magic, splat(-kRound));
  Pair x = fma<P>(k, splat(-3.1415927410125732421875f), theta);  // float(pi)
  x = fma<P>(k, splat(8.74227800037248566e-8f), x);              // pi - float(pi), negated
  const float rx = __uint_as_float(__float_as_uint(r.x) ^ low_bit_to_sign(__float_as_uint(magic.x)));
  const float ry = __uint_as_float(__float_as_uint(r.y) ^ low_bit_to_sign(__float_as_uint(magic.y)));
  p0 = mul<P>(splat(rx), {cos_approx(x.x), sin_approx(x.x)});
  p1 = mul<P>(splat(ry), {cos_approx(x.y), sin_approx(x.y)});
  // r >= 0, so the threshold test is an integer compare of the bits
  const bool fx = __float_as_uint(r.x) > __float_as_uint(kRadHw);
  const bool fy = __float_as_uint(r.y) > __float_as_uint(kRadHw);
  if (fx || fy) {
    Pair pc, ps;
    polar2<P, P>(theta, r, pc, ps);
    if (fx) p0 = {pc.x, ps.x};
    if (fy) p1 = {pc.y, ps.y};
  }
}

// The normal transform of one Philox block (u0..u3 = the four words as uniforms):
// (r0 cos t0, r0 sin t0, r1 cos t1, r1 sin t1) with r_i = sqrt(-2 ln u_2i), t_i = 2pi u_2i+1,
// then * stddev (Aff 2) and + mean (Aff >= 1), each rounded as in the reference.  Aff 0
// serves mean 0 and stddev 1: the product by 1 is exact and adding 0 only turns a zero
// output's sign from - to +, so both are left out.
template <int Aff>
__device__ __forceinline__ uint4 normal_block_hw(uint4 r, float mean, float stddev) {
  const Pair ue = to_uniform2<true>(r.x, r.z), uo = to_uniform2<true>(r.y, r.w);
  const Pair w = neg2_log_hw<true>(ue);
  const Pair rad = {sqrt_approx(w.x), sqrt_approx(w.y)};
  const Pair theta = mul<true>(splat(6.28318530717958647692f), uo);
  Pair p0, p1;
  polar_pairs_hw<true>(theta, rad, p0, p1);
  if constexpr (Aff == 2) {
    p0 = mul<true>(p0, splat(stddev));
    p1 = mul<true>(p1, splat(stddev));
  }
  if constexpr (Aff >= 1) {
    p0 = add<true>(p0, splat(mean));
    p1 = add<true>(p1, splat(mean));
  }
  return make_uint4(__float_as_uint(p0.x), __float_as_uint(p0.y), __float_as_uint(p1.x),
                    __float_as_uint(p1.y));
}

}  // namespace
}  // namespace mb200::rand
