// stockham_core.cuh — building blocks of the on-chip Stockham FFT kernels:
// complex helpers, in-register R-point DFTs (R = 2, 4, 8, 16), table twiddles and
// the compile-time plan of a power-of-two length.  Included by the C2C / real-data
// kernels (stockham_kernels.cu) and the Bluestein kernel (bluestein_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mb200::fft {
namespace {

// Complex add and subtract as one add / sub.rn.f32x2 on the (re, im) pair: each lane
// rounded as the scalar instruction, one issue slot for both.
__device__ __forceinline__ unsigned long long c_pack(float2 a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
__device__ __forceinline__ float2 c_unpack(unsigned long long v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(c_pack(a)), "l"(c_pack(b)));
  return c_unpack(d);
}
__device__ __forceinline__ float2 csub(float2 a, float2 b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(c_pack(a)), "l"(c_pack(b)));
  return c_unpack(d);
}
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
// multiply by S*i
template <int S>
__device__ __forceinline__ float2 mul_si(float2 a) {
  return S < 0 ? make_float2(a.y, -a.x) : make_float2(-a.y, a.x);
}

// exp(S * 2*pi*i * m / 16) for a compile-time m.
template <int S, int M>
__device__ __forceinline__ float2 rot16(float2 a) {
  constexpr int m = M & 15;
  constexpr float kC[16] = {1.0f, 0.9238795042037964f, 0.7071067690849304f, 0.3826834261417389f,
                            0.0f, -0.3826834261417389f, -0.7071067690849304f, -0.9238795042037964f,
                            -1.0f, -0.9238795042037964f, -0.7071067690849304f, -0.3826834261417389f,
                            0.0f, 0.3826834261417389f, 0.7071067690849304f, 0.9238795042037964f};
  constexpr float kS[16] = {0.0f, 0.3826834261417389f, 0.7071067690849304f, 0.9238795042037964f,
                            1.0f, 0.9238795042037964f, 0.7071067690849304f, 0.3826834261417389f,
                            0.0f, -0.3826834261417389f, -0.7071067690849304f, -0.9238795042037964f,
                            -1.0f, -0.9238795042037964f, -0.7071067690849304f, -0.3826834261417389f};
  if constexpr (m == 0) {
    return a;
  } else if constexpr (m == 4) {
    return mul_si<S>(a);
  } else if constexpr (m == 8) {
    return make_float2(-a.x, -a.y);
  } else if constexpr (m == 12) {
    return mul_si<-S>(a);
  } else {
    return cmul(a, make_float2(kC[m], S * kS[m]));
  }
}

// In-register R-point DFT, natural order in and out: v[k] <- sum_n v[n] W_R^{S n k}.
template <int R, int S>
__device__ __forceinline__ void dft(float2* v);

template <int S, int R, int A, int B, int N2 = 0, int K1 = 0>
__device__ __forceinline__ void twiddle_step(float2 (&y)[R]) {
  if constexpr (N2 < B) {
    if constexpr (K1 < A) {
      y[N2 * A + K1] = rot16<S, (16 / R) * N2 * K1>(y[N2 * A + K1]);
      twiddle_step<S, R, A, B, N2, K1 + 1>(y);
    } else {
      twiddle_step<S, R, A, B, N2 + 1, 0>(y);
    }
  }
}

template <int R, int S>
__device__ __forceinline__ void dft(float2* v) {
  if constexpr (R == 2) {
    const float2 a = v[0], b = v[1];
    v[0] = cadd(a, b);
    v[1] = csub(a, b);
  } else if constexpr (R == 4) {
    const float2 a = cadd(v[0], v[2]), b = csub(v[0], v[2]);
    const float2 c = cadd(v[1], v[3]), d = mul_si<S>(csub(v[1], v[3]));
    v[0] = cadd(a, c);
    v[2] = csub(a, c);
    v[1] = cadd(b, d);
    v[3] = csub(b, d);
  } else {
    // R = A * B; n = B*n1 + n2, k = k1 + A*k2:
    //   Y[n2][k1] = W_R^{n2 k1} * sum_{n1} x[B n1 + n2] W_A^{n1 k1}
    //   X[k1 + A k2] = sum_{n2} Y[n2][k1] W_B^{n2 k2}
    constexpr int A = (R == 8) ? 2 : 4;
    constexpr int B = R / A;
    float2 y[R];
#pragma unroll
    for (int n2 = 0; n2 < B; ++n2) {
      float2 s[A];
#pragma unroll
      for (int n1 = 0; n1 < A; ++n1) s[n1] = v[B * n1 + n2];
      dft<A, S>(s);
#pragma unroll
      for (int k1 = 0; k1 < A; ++k1) y[n2 * A + k1] = s[k1];
    }
    twiddle_step<S, R, A, B>(y);
#pragma unroll
    for (int k1 = 0; k1 < A; ++k1) {
      float2 s[B];
#pragma unroll
      for (int n2 = 0; n2 < B; ++n2) s[n2] = y[n2 * A + k1];
      dft<B, S>(s);
#pragma unroll
      for (int k2 = 0; k2 < B; ++k2) v[k1 + A * k2] = s[k2];
    }
  }
}

template <int S>
__device__ __forceinline__ float2 table_tw(const float2* __restrict__ tw, std::int64_t m) {
  float2 w = __ldg(tw + m);
  if (S > 0) w.y = -w.y;
  return w;
}

// v[r] *= w^r for r = 1..R-1, where w = table[m] (the butterfly's base twiddle,
// conjugated for S > 0).  Only w and w^4 are read from the table; the other powers
// are products of at most three exact-rounded table values (w^2 = w*w,
// w^3 = w^2*w, w^8 = (w^4)^2, w^12 = w^8*w^4, w^r = w^(r mod 4) * w^(r - r mod 4)),
// which keeps the relative error of every twiddle within a few fp32 ulps while
// cutting the table reads per radix-16 butterfly from 15 to 2.
template <int R, int S>
__device__ __forceinline__ void apply_twiddles(float2* v, const float2* __restrict__ tw, int m) {
  if constexpr (R == 2) {
    v[1] = cmul(v[1], table_tw<S>(tw, m));
  } else {
    float2 lo[4], hi[4];
    lo[1] = table_tw<S>(tw, m);
    lo[2] = cmul(lo[1], lo[1]);
    lo[3] = cmul(lo[2], lo[1]);
    if constexpr (R >= 8) {
      hi[1] = table_tw<S>(tw, 4 * m);
      if constexpr (R == 16) {
        hi[2] = cmul(hi[1], hi[1]);
        hi[3] = cmul(hi[2], hi[1]);
      }
    }
#pragma unroll
    for (int r = 1; r < R; ++r) {
      const int a = r & 3, b = r >> 2;
      float2 w;
      if (b == 0) {
        w = lo[a];
      } else if (a == 0) {
        w = hi[b];
      } else {
        w = cmul(lo[a], hi[b]);
      }
      v[r] = cmul(v[r], w);
    }
  }
}

// Compile-time plan of a length-N transform.
template <int LOG2N>
struct Plan {
  static constexpr int N = 1 << LOG2N;
  static constexpr int P = N >= 16 ? 16 : N;                 // points per thread
  static constexpr int T = N / P;                            // threads per transform
  static constexpr int TPC = T >= 256 ? 1 : 256 / T;         // transforms per CTA
  static constexpr int THREADS = T * TPC;
  static constexpr int FIRST_R = (LOG2N % 4 == 0) ? (N >= 16 ? 16 : N) : (1 << (LOG2N % 4));
  static constexpr int PASSES = (LOG2N % 4 == 0) ? LOG2N / 4 : LOG2N / 4 + 1;
  static constexpr int REGION = N + N / 32 + 1;              // padded floats per transform
  static constexpr int SMEM = PASSES > 1 ? TPC * REGION * 2 * 4 : 0;
  // Resident CTAs per SM the register budget is sized for: several CTAs per SM
  // let one CTA's HBM loads overlap another's on-chip passes.
  static constexpr int MIN_CTAS = THREADS >= 1024 ? 1 : (THREADS >= 512 ? 2 : 3);
};

// One pad word per 32: the stride-16 scatter of the first pass and the
// stride-N/16 gathers of the later passes are conflict free.
__device__ __forceinline__ int pad(int i) { return i + (i >> 5); }

__host__ __device__ constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v >> 1); }

}  // namespace
}  // namespace mb200::fft
