// bluestein_kernels.cu — C2C transforms of lengths that are not powers of two
// (sm_100a), by Bluestein's chirp-z algorithm with both inner FFTs on chip.
//
// The reference transforms such an axis with the direct O(N^2) DFT of
// cufft_kernels.metal:298-325 (one thread per output, one sincos per term).
// Here, with nk = (n^2 + k^2 - (k - n)^2) / 2 and w[m] = exp(sign*pi*i*m^2/N)
// (L. Bluestein, "A linear filtering approach to the computation of discrete
// Fourier transform", 1970):
//   X[k] = w[k] * sum_n (x[n] w[n]) conj(w[k - n]),
// a cyclic convolution of a[n] = x[n] w[n] (zero beyond N) with b[m] = conj(w[m])
// (m in (-N, N), wrapped) over a power-of-two length Mb >= 2N - 1, computed as
// IFFT(FFT(a) * Bhat), Bhat = FFT(b) / Mb precomputed in double precision.
//
// One CTA keeps whole length-Mb transforms in shared memory: the forward FFT's
// first pass reads x from global memory and multiplies by w, its last pass leaves
// the spectrum in shared memory, the inverse FFT's first pass multiplies it by
// Bhat, and its last pass multiplies by w and writes the N outputs.  HBM traffic
// is one read and one write per element, as for power-of-two lengths; the work is
// two length-Mb FFTs (Mb < 4N) instead of N^2 products.  The tables hold the
// forward direction; the inverse uses their conjugates (b is symmetric, so
// FFT(conj b) = conj(FFT(b))).
#include <cuda_runtime.h>

#include <cstdint>

#include "common/device.hpp"
#include "fft/fft.hpp"
#include "fft/stockham_core.cuh"

namespace mb200::fft {
namespace {

struct Io {
  const float2* in;
  float2* out;
  std::int64_t in_stride, out_stride;
  bool active;
  int n;
  const float2* chirp;  // w[m] of the forward direction, m < n
  const float2* bhat;   // FFT(b) / Mb of the forward direction
};

template <int DIR>
__device__ __forceinline__ float2 dir_table(const float2* __restrict__ t, int m) {
  float2 v = __ldg(t + m);
  if (DIR > 0) v.y = -v.y;
  return v;
}

enum Src { kFromGlobal, kFromShared, kFromSharedTimesBhat };
enum Dst { kToShared, kToGlobal };

// One Stockham pass of a length-2^LOG2M transform with FFT direction S; the data
// source and sink of the pass are chosen by SRC and DST, every intermediate lives
// in the padded split arrays sre/sim.
template <int LOG2M, int R, int S, int DIR, int SRC, int DST>
__device__ __forceinline__ void bpass(float2 (&v)[Plan<LOG2M>::P], int j, int Ns, int log2Ns,
                                      const Io& io, float* sre, float* sim,
                                      const float2* __restrict__ tw) {
  using PL = Plan<LOG2M>;
  constexpr int M = PL::N;
  constexpr int T = PL::T;
  constexpr int NB = PL::P / R;
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    const int b = j + q * T;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int idx = b + r * (M / R);
      float2 x;
      if constexpr (SRC == kFromGlobal) {
        x = make_float2(0.0f, 0.0f);
        if (io.active && idx < io.n) x = cmul(io.in[idx * io.in_stride], dir_table<DIR>(io.chirp, idx));
      } else {
        x = make_float2(sre[pad(idx)], sim[pad(idx)]);
        if constexpr (SRC == kFromSharedTimesBhat) x = cmul(x, dir_table<DIR>(io.bhat, idx));
      }
      v[q * R + r] = x;
    }
  }
  if constexpr (SRC != kFromGlobal) __syncthreads();  // reads done before the arrays change
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    const int b = j + q * T;
    const int k = b & (Ns - 1);
    if (Ns > 1) apply_twiddles<R, S>(&v[q * R], tw, k << (LOG2M - log2Ns - ilog2(R)));
    dft<R, S>(&v[q * R]);
    const int idxD = ((b >> log2Ns) << (log2Ns + ilog2(R))) + k;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int o = idxD + r * Ns;
      if constexpr (DST == kToGlobal) {
        if (io.active && o < io.n)
          io.out[o * io.out_stride] = cmul(v[q * R + r], dir_table<DIR>(io.chirp, o));
      } else {
        sre[pad(o)] = v[q * R + r].x;
        sim[pad(o)] = v[q * R + r].y;
      }
    }
  }
  if constexpr (DST == kToShared) __syncthreads();
}

// All passes of one inner FFT: FWD = true is FFT(a) (reads x, leaves the spectrum
// in shared memory), FWD = false is IFFT(spectrum * Bhat) (writes the outputs).
template <int LOG2M, int DIR, bool FWD, int PASS = 0>
__device__ __forceinline__ void inner_fft(float2 (&v)[Plan<LOG2M>::P], int j, const Io& io,
                                          float* sre, float* sim, const float2* tw) {
  using PL = Plan<LOG2M>;
  if constexpr (PASS < PL::PASSES) {
    constexpr int R = (PASS == 0) ? PL::FIRST_R : 16;
    constexpr int LOG2NS = (PASS == 0) ? 0 : (ilog2(PL::FIRST_R) + 4 * (PASS - 1));
    constexpr int SRC =
        PASS == 0 ? (FWD ? kFromGlobal : kFromSharedTimesBhat) : kFromShared;
    constexpr int DST = (PASS == PL::PASSES - 1 && !FWD) ? kToGlobal : kToShared;
    bpass<LOG2M, R, FWD ? -1 : 1, DIR, SRC, DST>(v, j, 1 << LOG2NS, LOG2NS, io, sre, sim, tw);
    inner_fft<LOG2M, DIR, FWD, PASS + 1>(v, j, io, sre, sim, tw);
  }
}

// CTA shape of the fused kernel: one transform per CTA once a transform has 64
// threads or more (a CTA's barriers then wait only for its own transform, as the
// mixed-radix kernel measured), else the Stockham plan's packing.  Two inner FFTs
// keep more state live than one: the register budget is 128 a thread, 512 threads
// of resident CTAs per SM, except for 128-thread CTAs (inner length 2048), which fit
// in 96 registers without spilling and so run 5 to an SM (N = 1009: 5.91 -> 5.81 ms;
// 6 CTAs spilled).
template <int LOG2M>
struct BlueShape {
  static constexpr int TPC = Plan<LOG2M>::T >= 64 ? 1 : Plan<LOG2M>::TPC;
  static constexpr int THREADS = Plan<LOG2M>::T * TPC;
  static constexpr int CTAS = THREADS >= 512 ? 1 : (THREADS == 128 ? 5 : 512 / THREADS);
};
template <int LOG2M>
constexpr int kBlueCtas = BlueShape<LOG2M>::CTAS;

template <int LOG2M, int DIR>
__global__ void __launch_bounds__(BlueShape<LOG2M>::THREADS, kBlueCtas<LOG2M>)
    bluestein_kernel(const Batch1D bt, int n, const float2* __restrict__ chirp,
                     const float2* __restrict__ bhat, const float2* __restrict__ tw_m) {
  using PL = Plan<LOG2M>;
  using BS = BlueShape<LOG2M>;
  extern __shared__ float smem[];
  const int tloc = threadIdx.x / PL::T;
  const int j = threadIdx.x % PL::T;
  float* sre = smem + tloc * PL::REGION * 2;
  float* sim = sre + PL::REGION;
  for (std::int64_t t0 = static_cast<std::int64_t>(blockIdx.x) * BS::TPC; t0 < bt.batch;
       t0 += static_cast<std::int64_t>(gridDim.x) * BS::TPC) {
    const std::int64_t tr = t0 + tloc;
    Io io;
    io.active = tr < bt.batch;
    const std::int64_t outer = io.active ? tr / bt.inner_count : 0;
    const std::int64_t inner = io.active ? tr % bt.inner_count : 0;
    io.in = bt.in + outer * bt.in_outer + inner * bt.in_inner;
    io.out = bt.out + outer * bt.out_outer + inner * bt.out_inner;
    io.in_stride = bt.in_stride;
    io.out_stride = bt.out_stride;
    io.n = n;
    io.chirp = chirp;
    io.bhat = bhat;
    float2 v[PL::P];
    inner_fft<LOG2M, DIR, true>(v, j, io, sre, sim, tw_m);
    inner_fft<LOG2M, DIR, false>(v, j, io, sre, sim, tw_m);
  }
}

template <int LOG2M, int DIR>
cudaError_t launch_m(int n, const Batch1D& b, const float2* chirp, const float2* bhat,
                     const float2* tw_m, cudaStream_t stream) {
  using PL = Plan<LOG2M>;
  using BS = BlueShape<LOG2M>;
  auto kern = bluestein_kernel<LOG2M, DIR>;
  constexpr int kSmem = BS::TPC * PL::REGION * 2 * 4;
  if (kSmem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
  }
  const std::int64_t ctas = (b.batch + BS::TPC - 1) / BS::TPC;
  const int sms = sm_count(current_device());
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * kBlueCtas<LOG2M> * 8;
  const unsigned grid = static_cast<unsigned>(ctas < cap ? ctas : cap);
  kern<<<grid, BS::THREADS, kSmem, stream>>>(b, n, chirp, bhat, tw_m);
  return cudaGetLastError();
}

template <int DIR>
cudaError_t dispatch(int log2m, int n, const Batch1D& b, const float2* chirp, const float2* bhat,
                     const float2* tw_m, cudaStream_t st) {
  switch (log2m) {
    case 6: return launch_m<6, DIR>(n, b, chirp, bhat, tw_m, st);
    case 7: return launch_m<7, DIR>(n, b, chirp, bhat, tw_m, st);
    case 8: return launch_m<8, DIR>(n, b, chirp, bhat, tw_m, st);
    case 9: return launch_m<9, DIR>(n, b, chirp, bhat, tw_m, st);
    case 10: return launch_m<10, DIR>(n, b, chirp, bhat, tw_m, st);
    case 11: return launch_m<11, DIR>(n, b, chirp, bhat, tw_m, st);
    case 12: return launch_m<12, DIR>(n, b, chirp, bhat, tw_m, st);
    case 13: return launch_m<13, DIR>(n, b, chirp, bhat, tw_m, st);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// Global-memory Bluestein for lengths above kMaxBluestein.

constexpr int kMoveThreads = 256;

unsigned move_grid(std::int64_t work) {
  const int sms = sm_count(current_device());
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 8;
  const std::int64_t want = (work + kMoveThreads - 1) / kMoveThreads;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

// Address of element 0 of transform t of a Batch1D operand.
__device__ __forceinline__ std::int64_t row_base(std::int64_t t, std::int64_t inner_count,
                                                 std::int64_t outer, std::int64_t inner) {
  return (t / inner_count) * outer + (t % inner_count) * inner;
}

// ws[r][m] = x_{t0+r}[m] * w[m] for m < n, 0 for n <= m < Mb.
template <int DIR>
__global__ void __launch_bounds__(kMoveThreads)
    chirp_gather(const Batch1D bt, std::int64_t t0, std::int64_t rows, std::int64_t n,
                 int log2m, const float2* __restrict__ chirp, float2* __restrict__ ws) {
  const std::int64_t total = rows << log2m;
  const std::int64_t mmask = (std::int64_t{1} << log2m) - 1;
  for (std::int64_t i = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       i < total; i += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = i >> log2m, m = i & mmask;
    float2 v = make_float2(0.0f, 0.0f);
    if (m < n) {
      const float2* x = bt.in + row_base(t0 + r, bt.inner_count, bt.in_outer, bt.in_inner);
      v = cmul(x[m * bt.in_stride], dir_table<DIR>(chirp, static_cast<int>(m)));
    }
    ws[i] = v;
  }
}

template <int DIR>
__global__ void __launch_bounds__(kMoveThreads)
    times_bhat(float2* __restrict__ ws, std::int64_t rows, int log2m,
               const float2* __restrict__ bhat) {
  const std::int64_t total = rows << log2m;
  const std::int64_t mmask = (std::int64_t{1} << log2m) - 1;
  for (std::int64_t i = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       i < total; i += static_cast<std::int64_t>(gridDim.x) * blockDim.x)
    ws[i] = cmul(ws[i], dir_table<DIR>(bhat, static_cast<int>(i & mmask)));
}

// out_{t0+r}[k] = ws[r][k] * w[k] for k < n.
template <int DIR>
__global__ void __launch_bounds__(kMoveThreads)
    chirp_scatter(const Batch1D bt, std::int64_t t0, std::int64_t rows, std::int64_t n,
                  int log2m, const float2* __restrict__ chirp, const float2* __restrict__ ws) {
  const std::int64_t total = rows * n;
  for (std::int64_t i = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       i < total; i += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t r = i / n, k = i - r * n;
    float2* y = bt.out + row_base(t0 + r, bt.inner_count, bt.out_outer, bt.out_inner);
    y[k * bt.out_stride] = cmul(ws[(r << log2m) + k], dir_table<DIR>(chirp, static_cast<int>(k)));
  }
}

// Length-m power-of-two FFT of `rows` dense rows of `data` (in place); above the
// single-pass limit, the two-pass split m = n1 * n2 through `scratch`:
//   pass A, per (row, r2): length-n1 transform over t = n2*r1 + r2, output k1 times
//           W_m^{r2*k1}, stored at scratch[row][k1*n2 + r2];
//   pass B, per (row, k1): length-n2 transform over r2, output k2 at data[row][k1 + n1*k2].
cudaError_t dense_pow2_fft(std::int64_t m, int sign, float2* data, std::int64_t rows,
                           const BluesteinGlobal& g, cudaStream_t st) {
  if (m <= kMaxSinglePass) {
    Batch1D b{};
    b.in = data;
    b.out = data;
    b.in_stride = b.out_stride = 1;
    b.in_outer = b.out_outer = m;
    b.batch = rows;
    b.inner_count = 1;
    b.tw = g.tw_m;
    b.post_n = 1;
    return launch_stockham(m, sign, b, st);
  }
  Batch1D a{};
  a.in = data;
  a.out = g.ws2;
  a.in_stride = g.n2;
  a.in_outer = m;
  a.in_inner = 1;
  a.out_stride = g.n2;
  a.out_outer = m;
  a.out_inner = 1;
  a.batch = rows * g.n2;
  a.inner_count = g.n2;
  a.tw = g.tw_n1;
  a.post_tw = g.tw_m;
  a.post_n = m;
  cudaError_t e = launch_stockham(g.n1, sign, a, st);
  if (e != cudaSuccess) return e;
  Batch1D c{};
  c.in = g.ws2;
  c.out = data;
  c.in_stride = 1;
  c.in_outer = m;
  c.in_inner = g.n2;
  c.out_stride = g.n1;
  c.out_outer = m;
  c.out_inner = 1;
  c.batch = rows * g.n1;
  c.inner_count = g.n1;
  c.tw = g.tw_n2;
  c.post_n = 1;
  return launch_stockham(g.n2, sign, c, st);
}

template <int DIR>
cudaError_t global_dir(std::int64_t n, const Batch1D& b, const BluesteinGlobal& g,
                       cudaStream_t st) {
  const std::int64_t m = bluestein_length(n);
  const int log2m = __builtin_ctzll(static_cast<unsigned long long>(m));
  for (std::int64_t t0 = 0; t0 < b.batch; t0 += g.ws_rows) {
    const std::int64_t rows = (b.batch - t0 < g.ws_rows) ? b.batch - t0 : g.ws_rows;
    chirp_gather<DIR><<<move_grid(rows * m), kMoveThreads, 0, st>>>(b, t0, rows, n, log2m,
                                                                      g.chirp, g.ws);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = dense_pow2_fft(m, -1, g.ws, rows, g, st);
    if (e == cudaSuccess) {
      times_bhat<DIR><<<move_grid(rows * m), kMoveThreads, 0, st>>>(g.ws, rows, log2m, g.bhat);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = dense_pow2_fft(m, 1, g.ws, rows, g, st);
    if (e == cudaSuccess) {
      chirp_scatter<DIR><<<move_grid(rows * n), kMoveThreads, 0, st>>>(b, t0, rows, n, log2m,
                                                                         g.chirp, g.ws);
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_bluestein_global(std::int64_t n, int sign, const Batch1D& b,
                                    const BluesteinGlobal& g, cudaStream_t stream) noexcept {
  if (n <= kMaxBluestein || n > kMaxBluesteinGlobal || b.post_tw != nullptr || g.ws == nullptr ||
      g.ws_rows <= 0 || (bluestein_length(n) > kMaxSinglePass && g.ws2 == nullptr))
    return cudaErrorInvalidValue;
  if (b.batch <= 0) return cudaSuccess;
  return sign < 0 ? global_dir<-1>(n, b, g, stream) : global_dir<1>(n, b, g, stream);
}

namespace {

__global__ void __launch_bounds__(kMoveThreads) twiddle_table(float2* tw, std::int64_t n) {
  for (std::int64_t m = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x; m < n;
       m += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    double s, c;
    sincospi(2.0 * static_cast<double>(m) / static_cast<double>(n), &s, &c);
    tw[m] = make_float2(static_cast<float>(c), static_cast<float>(-s));
  }
}

// chirp[m] = exp(-pi*i*q/n), q = m^2 mod 2n exactly; b[m] = b[mb - m] = conj(chirp[m])
// (b zero-filled beforehand).
__global__ void __launch_bounds__(kMoveThreads)
    chirp_table(std::int64_t n, std::int64_t mb, float2* chirp, float2* b) {
  for (std::int64_t m = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x; m < n;
       m += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long q =
        (static_cast<unsigned long long>(m) * static_cast<unsigned long long>(m)) %
        static_cast<unsigned long long>(2 * n);
    double s, c;
    sincospi(static_cast<double>(q) / static_cast<double>(n), &s, &c);
    const float cf = static_cast<float>(c), sf = static_cast<float>(s);
    chirp[m] = make_float2(cf, -sf);
    b[m] = make_float2(cf, sf);
    if (m > 0) b[mb - m] = make_float2(cf, sf);
  }
}

__global__ void __launch_bounds__(kMoveThreads) scale_table(float2* v, std::int64_t n, float f) {
  for (std::int64_t i = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<std::int64_t>(gridDim.x) * blockDim.x)
    v[i] = make_float2(v[i].x * f, v[i].y * f);
}

}  // namespace

cudaError_t build_twiddles(float2* tw, std::int64_t n, cudaStream_t stream) noexcept {
  if (tw == nullptr || n <= 0) return cudaErrorInvalidValue;
  twiddle_table<<<move_grid(n), kMoveThreads, 0, stream>>>(tw, n);
  return cudaGetLastError();
}

cudaError_t build_bluestein_tables(std::int64_t n, float2* chirp, float2* bhat,
                                   const BluesteinGlobal& g, cudaStream_t stream) noexcept {
  const std::int64_t mb = bluestein_length(n);
  if (chirp == nullptr || bhat == nullptr || g.tw_m == nullptr ||
      (mb > kMaxSinglePass && g.ws2 == nullptr))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(bhat, 0, static_cast<std::size_t>(mb) * sizeof(float2), stream);
  if (e != cudaSuccess) return e;
  chirp_table<<<move_grid(n), kMoveThreads, 0, stream>>>(n, mb, chirp, bhat);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if ((e = dense_pow2_fft(mb, -1, bhat, 1, g, stream)) != cudaSuccess) return e;
  scale_table<<<move_grid(mb), kMoveThreads, 0, stream>>>(bhat, mb,
                                                          1.0f / static_cast<float>(mb));
  return cudaGetLastError();
}

std::int64_t bluestein_length(std::int64_t n) noexcept {
  std::int64_t m = 1;
  while (m < 2 * n - 1) m <<= 1;
  return m;
}

cudaError_t launch_bluestein(std::int64_t n, int sign, const Batch1D& b, const float2* chirp,
                             const float2* bhat, const float2* tw_m,
                             cudaStream_t stream) noexcept {
  if (n < kMinBluestein || n > kMaxBluestein || b.post_tw != nullptr) return cudaErrorInvalidValue;
  if (b.batch <= 0) return cudaSuccess;
  const std::int64_t m = bluestein_length(n);
  const int log2m = __builtin_ctzll(static_cast<unsigned long long>(m));
  const int ni = static_cast<int>(n);
  return sign < 0 ? dispatch<-1>(log2m, ni, b, chirp, bhat, tw_m, stream)
                  : dispatch<1>(log2m, ni, b, chirp, bhat, tw_m, stream);
}

}  // namespace mb200::fft
