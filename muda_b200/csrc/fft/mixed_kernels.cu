// mixed_kernels.cu — C2C transforms of lengths whose prime factors are 2, 3, 5 and 7
// (not powers of two), one CTA per transform, every pass in shared memory (sm_100a).
//
// The reference runs these lengths through its O(N^2) direct DFT
// (cufft_kernels.metal:298-325).  Here the length is factored on the host into a
// radix sequence (16 while possible, then 8 / 4 / 2, then 3, 5, 7) and transformed by
// Stockham autosort passes (Govindaraju et al., SC 2008): pass p with radix R and
// span Ns (the product of the earlier radices) takes v[r] = d[j + r*N/R], multiplies
// v[r] by exp(sign*2*pi*i * r*(j mod Ns) / (Ns*R)) (the exact-rounded N-entry table at
// index r*(j mod Ns)*N/(Ns*R)), runs an R-point DFT in registers and stores
// d'[(j / Ns)*Ns*R + (j mod Ns) + r*Ns].  The transform is read from global memory
// by the first pass straight into registers, the passes exchange through two
// shared-memory buffers (a thread holds one butterfly at a time), and the last pass
// writes the result: one HBM read and one write per element.  Each pass is a template on its radix, so the butterfly
// values stay in registers.
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "common/device.hpp"
#include "fft/fft.hpp"
#include "fft/stockham_core.cuh"

namespace mb200::fft {
namespace {


// The passes run in the order: n16 of radix 16, one of radix r2 (8, 4 or 2; 0 = none),
// then n3, n5 and n7 of radices 3, 5 and 7.
struct MixedPlan {
  int n;
  int threads;  // per transform (a multiple of 32)
  int tpc;      // transforms per CTA
  int n16, r2, n3, n5, n7;
};

// (cos, sin) of 2*pi*m/R for small odd R, from double constants rounded once; the
// index is a compile-time constant after unrolling, so the arrays fold to immediates.
template <int R>
__device__ __forceinline__ float2 odd_root(int m) {
  if constexpr (R == 3) {
    constexpr float c[3] = {1.0f, -0.5f, -0.5f};
    constexpr float s[3] = {0.0f, 0.8660254037844386f, -0.8660254037844386f};
    return make_float2(c[m], s[m]);
  } else if constexpr (R == 5) {
    constexpr float c[5] = {1.0f, 0.30901699437494745f, -0.8090169943749475f,
                            -0.8090169943749475f, 0.30901699437494745f};
    constexpr float s[5] = {0.0f, 0.9510565162951535f, 0.5877852522924732f,
                            -0.5877852522924732f, -0.9510565162951535f};
    return make_float2(c[m], s[m]);
  } else {
    static_assert(R == 7, "odd radix");
    constexpr float c[7] = {1.0f, 0.6234898018587336f, -0.22252093395631434f,
                            -0.9009688679024191f, -0.9009688679024191f,
                            -0.22252093395631434f, 0.6234898018587336f};
    constexpr float s[7] = {0.0f, 0.7818314824680298f, 0.9749279121818236f,
                            0.43388373911755823f, -0.43388373911755823f,
                            -0.9749279121818236f, -0.7818314824680298f};
    return make_float2(c[m], s[m]);
  }
}

// R-point DFT for odd R by pairs: with u_n = v_n + v_{R-n}, w_n = v_n - v_{R-n},
// X_k = v_0 + sum_n (c_{nk} u_n + S i s_{nk} w_n) and X_{R-k} likewise with -S.
template <int R, int S>
__device__ __forceinline__ void odd_dft(float2* v) {
  constexpr int H = R / 2;
  float2 u[H + 1], w[H + 1];
#pragma unroll
  for (int n = 1; n <= H; ++n) {
    u[n] = cadd(v[n], v[R - n]);
    w[n] = csub(v[n], v[R - n]);
  }
  float2 x0 = v[0];
#pragma unroll
  for (int n = 1; n <= H; ++n) x0 = cadd(x0, u[n]);
  float2 out[R];
  out[0] = x0;
#pragma unroll
  for (int k = 1; k <= H; ++k) {
    float2 a = v[0], b = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int n = 1; n <= H; ++n) {
      const int m = (n * k) % R;
      const float2 rt = odd_root<R>(m);
      const float cc = rt.x, ss = rt.y;
      a = make_float2(fmaf(cc, u[n].x, a.x), fmaf(cc, u[n].y, a.y));
      b = make_float2(fmaf(ss, w[n].x, b.x), fmaf(ss, w[n].y, b.y));
    }
    // S*i*b
    const float2 ib = S < 0 ? make_float2(b.y, -b.x) : make_float2(-b.y, b.x);
    out[k] = cadd(a, ib);
    out[R - k] = csub(a, ib);
  }
#pragma unroll
  for (int k = 0; k < R; ++k) v[k] = out[k];
}

template <int R, int S>
__device__ __forceinline__ void small_dft(float2* v) {
  if constexpr (R == 3 || R == 5 || R == 7) {
    odd_dft<R, S>(v);
  } else {
    dft<R, S>(v);
  }
}

__device__ __forceinline__ float2 tw_at(const float2* __restrict__ tw, int m, int sign) {
  float2 w = __ldg(tw + m);
  if (sign > 0) w.y = -w.y;
  return w;
}

// Shared-memory position of element e: one float2 of padding after every 16, so the
// stride-R stores of the first pass (and the unit-stride reads) are free of bank
// conflicts for every radix.
__device__ __forceinline__ int at(int e) { return e + (e >> 4); }
__host__ __device__ constexpr int padded(int n) { return n + (n >> 4) + 1; }

// Where a pass reads and writes: shared to shared, global to shared (the first pass,
// straight from the caller's input) or shared to global (the last pass, straight to
// the caller's output).  Both global sides are coalesced: the first pass reads
// in[j + r*N/R] and the last writes out[j + r*N/R] for consecutive j.
enum Mode { kShared = 0, kFromGlobal = 1, kToGlobal = 2 };

struct Io {
  const float2* in;  // this transform's input (kFromGlobal)
  float2* out;       // this transform's output (kToGlobal)
  std::int64_t in_stride, out_stride;
  bool active;       // false for the padding transforms of the last CTA
};

// Offset of element e of a transform in the caller's buffer: 32-bit for unit stride.
template <bool UNIT>
__device__ __forceinline__ std::int64_t io_offset(int e, std::int64_t stride) {
  if constexpr (UNIT) {
    return e;
  } else {
    return static_cast<std::int64_t>(e) * stride;
  }
}

// One pass of radix R: n complex values from src to dst.  j / ns comes from a float
// reciprocal: trunc((j + 0.5) * rn(1 / ns)) equals the integer quotient for every
// j, ns <= 12288 (checked exhaustively), and keeps the integer divide off the FMA pipe
// the butterflies use.
template <int R, int S, int MODE, bool UNIT>
__device__ __forceinline__ void mixed_pass(const float2* src, float2* dst, int n, int ns,
                                           int tid, int threads,
                                           const float2* __restrict__ tw, const Io& io) {
  const int nb = n / R;
  const int step = n / (ns * R);
  const float inv_ns = __frcp_rn(static_cast<float>(ns));
  for (int j = tid; j < nb; j += threads) {
    float2 v[R];
    if constexpr (MODE == kFromGlobal) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        v[r] = io.active ? io.in[io_offset<UNIT>(j + r * nb, io.in_stride)]
                         : make_float2(0.0f, 0.0f);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) v[r] = src[at(j + r * nb)];
    }
    const int q = __float2int_rz((static_cast<float>(j) + 0.5f) * inv_ns);
    const int k = j - q * ns;
    if (ns > 1) {
#pragma unroll
      for (int r = 1; r < R; ++r) v[r] = cmul(v[r], tw_at(tw, r * k * step, S));
    }
    small_dft<R, S>(v);
    const int o = q * ns * R + k;
    if constexpr (MODE == kToGlobal) {
      if (io.active) {
#pragma unroll
        for (int r = 0; r < R; ++r) io.out[io_offset<UNIT>(o + r * ns, io.out_stride)] = v[r];
      }
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) dst[at(o + r * ns)] = v[r];
    }
  }
  __syncthreads();
}

// The `count` passes of radix R, pass numbers p .. p + count - 1 of `total`.
template <int R, int S, bool UNIT>
__device__ __forceinline__ void run_radix(int count, int& p, int total, float2*& src,
                                          float2*& dst, int n, int& ns, int tid,
                                          int threads, const float2* __restrict__ tw,
                                          const Io& io) {
  for (int i = 0; i < count; ++i, ++p, ns *= R) {
    if (p == 0) {
      mixed_pass<R, S, kFromGlobal, UNIT>(src, dst, n, ns, tid, threads, tw, io);
    } else if (p == total - 1) {
      mixed_pass<R, S, kToGlobal, UNIT>(src, dst, n, ns, tid, threads, tw, io);
    } else {
      mixed_pass<R, S, kShared, UNIT>(src, dst, n, ns, tid, threads, tw, io);
    }
    float2* t = src;
    src = dst;
    dst = t;
  }
}

// R16: the plan has radix-16 passes.  Lengths without them (no factor 16, e.g. 1000 =
// 8 * 5^3) take an instantiation without the radix-16 code, whose registers would
// otherwise spill in every pass; capped at 56 registers, it keeps 9 CTAs of 128 threads
// on an SM instead of 8.
template <int S, bool UNIT, bool R16>
__global__ void __launch_bounds__(512) __maxnreg__(R16 ? 64 : 56)
    mixed_radix_kernel(const Batch1D bt, MixedPlan pl) {
  extern __shared__ float2 sbuf[];
  const int tl = threadIdx.x / pl.threads;  // transform within the CTA
  const int tid = threadIdx.x - tl * pl.threads;
  const int n = pl.n;
  const int total = pl.n16 + (pl.r2 != 0) + pl.n3 + pl.n5 + pl.n7;  // >= 2 for n >= 32
  for (std::int64_t t0 = static_cast<std::int64_t>(blockIdx.x) * pl.tpc; t0 < bt.batch;
       t0 += static_cast<std::int64_t>(gridDim.x) * pl.tpc) {
    const std::int64_t tr = t0 + tl;
    Io io;
    io.active = tr < bt.batch;
    const std::int64_t outer = io.active ? tr / bt.inner_count : 0;
    const std::int64_t inner = io.active ? tr % bt.inner_count : 0;
    io.in = bt.in + outer * bt.in_outer + inner * bt.in_inner;
    io.out = bt.out + outer * bt.out_outer + inner * bt.out_inner;
    io.in_stride = bt.in_stride;
    io.out_stride = bt.out_stride;
    float2* src = sbuf + tl * 2 * padded(n);
    float2* dst = src + padded(n);
    int ns = 1, p = 0;
    if constexpr (R16)
      run_radix<16, S, UNIT>(pl.n16, p, total, src, dst, n, ns, tid, pl.threads, bt.tw, io);
    if (pl.r2 == 8) {
      run_radix<8, S, UNIT>(1, p, total, src, dst, n, ns, tid, pl.threads, bt.tw, io);
    } else if (pl.r2 == 4) {
      run_radix<4, S, UNIT>(1, p, total, src, dst, n, ns, tid, pl.threads, bt.tw, io);
    } else if (pl.r2 == 2) {
      run_radix<2, S, UNIT>(1, p, total, src, dst, n, ns, tid, pl.threads, bt.tw, io);
    }
    run_radix<3, S, UNIT>(pl.n3, p, total, src, dst, n, ns, tid, pl.threads, bt.tw, io);
    run_radix<5, S, UNIT>(pl.n5, p, total, src, dst, n, ns, tid, pl.threads, bt.tw, io);
    run_radix<7, S, UNIT>(pl.n7, p, total, src, dst, n, ns, tid, pl.threads, bt.tw, io);
    // the last pass ended with a barrier, so the buffers are free for the next transform
  }
}

bool plan_for(std::int64_t n, MixedPlan* pl) {
  if (n < 32 || n > kMaxMixed) return false;  // two passes at least
  MixedPlan p{};
  p.n = static_cast<int>(n);
  std::int64_t m = n;
  int a = 0;
  while (m % 2 == 0) {
    m /= 2;
    ++a;
  }
  p.n16 = a / 4;
  p.r2 = a % 4 == 3 ? 8 : a % 4 == 2 ? 4 : a % 4 == 1 ? 2 : 0;
  for (; m % 3 == 0; m /= 3) ++p.n3;
  for (; m % 5 == 0; m /= 5) ++p.n5;
  for (; m % 7 == 0; m /= 7) ++p.n7;
  if (m != 1) return false;
  // threads: one butterfly of the widest pass per thread, 32 to 512
  int widest = p.n / (p.n16 ? 16 : p.r2 ? p.r2 : p.n3 ? 3 : p.n5 ? 5 : 7);
  int threads = 32;
  while (threads < 512 && threads < widest) threads *= 2;
  p.threads = threads;
  // one transform per CTA: measured on B200 for N = 1000 (x 262144), 128 threads a
  // transform, 1 / 2 / 4 transforms per CTA took 1.447 / 1.530 / 1.689 ms (a CTA's
  // barriers then wait only for its own transform, and more CTAs fit an SM); the
  // kernel still takes any tpc
  p.tpc = 1;
  *pl = p;
  return true;
}

}  // namespace

bool mixed_radix_supported(std::int64_t n) noexcept {
  MixedPlan p;
  return (n & (n - 1)) != 0 && plan_for(n, &p);
}

cudaError_t launch_mixed_radix(std::int64_t n, int sign, const Batch1D& b,
                               cudaStream_t stream) noexcept {
  MixedPlan p;
  if (!plan_for(n, &p) || b.post_tw != nullptr) return cudaErrorInvalidValue;
  if (b.batch <= 0) return cudaSuccess;
  const int threads = p.threads * p.tpc;
  const std::size_t smem = static_cast<std::size_t>(p.tpc) * 2 * padded(p.n) * sizeof(float2);
  const bool unit = b.in_stride == 1 && b.out_stride == 1;
  auto pick = [&](auto r16) {
    constexpr bool R = decltype(r16)::value;
    return sign < 0 ? (unit ? mixed_radix_kernel<-1, true, R> : mixed_radix_kernel<-1, false, R>)
                    : (unit ? mixed_radix_kernel<1, true, R> : mixed_radix_kernel<1, false, R>);
  };
  auto kern = p.n16 > 0 ? pick(std::true_type{}) : pick(std::false_type{});
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const std::int64_t ctas = (b.batch + p.tpc - 1) / p.tpc;
  const int sms = sm_count(current_device());
  const std::int64_t per_sm = (2048 / threads) > 1 ? 2048 / threads : 1;
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * per_sm * 4;
  const unsigned grid = static_cast<unsigned>(ctas < cap ? ctas : cap);
  kern<<<grid, threads, smem, stream>>>(b, p);
  return cudaGetLastError();
}

}  // namespace mb200::fft
