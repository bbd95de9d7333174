// stockham_kernels.cu — single-pass batched C2C FFT for power-of-two lengths (sm_100a).
//
// Conventions of the reference (libraries/fft/src/cufft_exec.mm): X[k] =
// sum_n x[n] exp(sign * 2*pi*i * n*k / N), sign -1 forward / +1 inverse, no
// scaling, in-place allowed.  The reference runs one radix-2 Stockham stage per
// launch over global memory (cufft_kernels.metal:255-296, cufft_exec.mm:58-74:
// 12 read+write passes of the whole batch for N = 4096, plus gather and scatter).
//
// Here one CTA owns whole transforms and performs every stage on chip:
//   - mixed-radix Stockham autosort (the formulation of Govindaraju et al.,
//     "High Performance Discrete Fourier Transforms on Graphics Processors",
//     SC 2008): pass p with radix R and span Ns reads v[r] = d[j + r*N/R],
//     multiplies by exp(sign*2*pi*i * r*(j mod Ns) / (Ns*R)), does an R-point DFT in
//     registers, and writes d'[(j / Ns)*Ns*R + (j mod Ns) + r*Ns];
//   - radix 16 (4 x 4 in registers) for all passes but possibly the first, so
//     N = 4096 takes three passes: global -> registers -> shared -> registers ->
//     shared -> registers -> global.  Each element is read from and written to
//     HBM exactly once per transform;
//   - first-pass loads and last-pass stores are coalesced across the threads of a
//     transform for unit stride (thread j touches elements j + r*N/R);
//   - shared memory holds real and imaginary parts in separate arrays with one
//     pad word per 32, which makes the stride-16 scatter of the first pass
//     conflict free;
//   - twiddles come from a table exp(-2*pi*i*m/N) computed in double on the host
//     and rounded once (conjugated for the inverse), not from sincos per
//     butterfly; a radix-16 butterfly reads two table entries (w, w^4) and forms
//     the other powers by products (apply_twiddles), which keeps table traffic
//     through L1 small.
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <mutex>

#include "blas/tc_ptx.cuh"
#include "common/device.hpp"
#include "fft/fft.hpp"
#include "fft/stockham_core.cuh"

namespace mb200::fft {
namespace {

struct Ctx {
  const float2* in;
  float2* out;
  std::int64_t in_stride, out_stride;
  bool active;
  std::int64_t inner;  // b % inner_count (post-twiddle row)
};


// One Stockham pass.  FIRST reads global memory, LAST writes global memory,
// the others go through shared memory (sre/sim).
template <int LOG2N, int R, int S, bool FIRST, bool LAST>
__device__ __forceinline__ void pass(float2 (&v)[Plan<LOG2N>::P], int j, int Ns, int log2Ns,
                                     const Ctx& c, float* sre, float* sim,
                                     const float2* __restrict__ tw,
                                     const float2* __restrict__ post_tw, std::int64_t post_n) {
  using PL = Plan<LOG2N>;
  constexpr int N = PL::N;
  constexpr int T = PL::T;
  constexpr int NB = PL::P / R;  // butterflies per thread
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    const int b = j + q * T;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int idx = b + r * (N / R);
      if constexpr (FIRST) {
        v[q * R + r] = c.active ? c.in[idx * c.in_stride] : make_float2(0.0f, 0.0f);
      } else {
        v[q * R + r] = make_float2(sre[pad(idx)], sim[pad(idx)]);
      }
    }
  }
  if constexpr (!FIRST) __syncthreads();  // all reads done before the region is rewritten
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    const int b = j + q * T;
    const int k = b & (Ns - 1);
    if (Ns > 1) {
      // exp(S*2*pi*i * r*k/(Ns*R)) = table[r*k*N/(Ns*R)]
      apply_twiddles<R, S>(&v[q * R], tw, k << (LOG2N - log2Ns - ilog2(R)));
    }
    dft<R, S>(&v[q * R]);
    const int idxD = ((b >> log2Ns) << (log2Ns + ilog2(R))) + k;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int o = idxD + r * Ns;
      if constexpr (LAST) {
        if (c.active) {
          float2 val = v[q * R + r];
          if (post_tw != nullptr)
            val = cmul(val, table_tw<S>(post_tw, (c.inner * o) % post_n));
          c.out[o * c.out_stride] = val;
        }
      } else {
        sre[pad(o)] = v[q * R + r].x;
        sim[pad(o)] = v[q * R + r].y;
      }
    }
  }
  if constexpr (!LAST) __syncthreads();
}

template <int LOG2N, int S, int PASS = 0>
__device__ __forceinline__ void run_passes(float2 (&v)[Plan<LOG2N>::P], int j, const Ctx& c,
                                           float* sre, float* sim, const float2* tw,
                                           const float2* post_tw, std::int64_t post_n) {
  using PL = Plan<LOG2N>;
  if constexpr (PASS < PL::PASSES) {
    constexpr int R = (PASS == 0) ? PL::FIRST_R : 16;
    constexpr int LOG2NS = (PASS == 0) ? 0 : (ilog2(PL::FIRST_R) + 4 * (PASS - 1));
    pass<LOG2N, R, S, PASS == 0, PASS == PL::PASSES - 1>(v, j, 1 << LOG2NS, LOG2NS, c, sre, sim,
                                                         tw, post_tw, post_n);
    run_passes<LOG2N, S, PASS + 1>(v, j, c, sre, sim, tw, post_tw, post_n);
  }
}

template <int LOG2N, int S>
__global__ void __launch_bounds__(Plan<LOG2N>::THREADS, Plan<LOG2N>::MIN_CTAS)
    stockham_kernel(const Batch1D bt) {
  using PL = Plan<LOG2N>;
  extern __shared__ float smem[];
  const int tloc = threadIdx.x / PL::T;
  const int j = threadIdx.x % PL::T;
  float* sre = smem + tloc * PL::REGION * 2;
  float* sim = sre + PL::REGION;
  for (std::int64_t t0 = static_cast<std::int64_t>(blockIdx.x) * PL::TPC; t0 < bt.batch;
       t0 += static_cast<std::int64_t>(gridDim.x) * PL::TPC) {
    const std::int64_t tr = t0 + tloc;
    Ctx c;
    c.active = tr < bt.batch;
    const std::int64_t outer = c.active ? tr / bt.inner_count : 0;
    c.inner = c.active ? tr % bt.inner_count : 0;
    c.in = bt.in + outer * bt.in_outer + c.inner * bt.in_inner;
    c.out = bt.out + outer * bt.out_outer + c.inner * bt.out_inner;
    c.in_stride = bt.in_stride;
    c.out_stride = bt.out_stride;
    float2 v[PL::P];
    run_passes<LOG2N, S>(v, j, c, sre, sim, bt.tw, bt.post_tw, bt.post_n);
  }
}

template <int LOG2N, int S>
cudaError_t launch_len(const Batch1D& b, cudaStream_t stream) {
  using PL = Plan<LOG2N>;
  auto kern = stockham_kernel<LOG2N, S>;
  if (PL::SMEM > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::SMEM);
    if (e != cudaSuccess) return e;
  }
  const std::int64_t ctas = (b.batch + PL::TPC - 1) / PL::TPC;
  const int sms = sm_count(current_device());
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 64;
  const unsigned grid = static_cast<unsigned>(ctas < cap ? ctas : cap);
  kern<<<grid, PL::THREADS, PL::SMEM, stream>>>(b);
  return cudaGetLastError();
}

template <int S>
cudaError_t dispatch(int log2n, const Batch1D& b, cudaStream_t st) {
  switch (log2n) {
    case 1: return launch_len<1, S>(b, st);
    case 2: return launch_len<2, S>(b, st);
    case 3: return launch_len<3, S>(b, st);
    case 4: return launch_len<4, S>(b, st);
    case 5: return launch_len<5, S>(b, st);
    case 6: return launch_len<6, S>(b, st);
    case 7: return launch_len<7, S>(b, st);
    case 8: return launch_len<8, S>(b, st);
    case 9: return launch_len<9, S>(b, st);
    case 10: return launch_len<10, S>(b, st);
    case 11: return launch_len<11, S>(b, st);
    case 12: return launch_len<12, S>(b, st);
    case 13: return launch_len<13, S>(b, st);
    case 14: return launch_len<14, S>(b, st);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy pipelined variant for contiguous batches (unit stride, dense batch
// distance, 16-byte aligned): each persistent CTA owns a ring of two 32 KB
// staging buffers filled by cp.async.bulk (one copy per group of TPC
// transforms, completing on an mbarrier).  While the passes of group g run, the
// copy of group g + gridDim.x is already in flight, and each finished group leaves
// through one bulk store from the same staging buffer, so loads, compute and
// stores of different groups overlap without any register staging.

__device__ unsigned int g_fft_bulk_timeouts;

// C2R pre-pass value Z'[k] = E[k] + i O[k] of a half-spectrum row X[0 .. n] held
// in shared memory: E[k] = X[k] + Xc, O[k] = (X[k] - Xc) conj(W^k), Xc = conj(X[n-k])
// for k > 0; for k = 0 only the real parts of X[0] and X[n] are used.  W^k is
// twl[k] = exp(-2*pi*i*k/(2n)).
__device__ __forceinline__ float2 c2r_point(const float2* raw, int k, int n, float2 w) {
  float2 xk = raw[k];
  float2 xc;
  if (k == 0) {
    xk.y = 0.0f;
    xc = make_float2(raw[n].x, 0.0f);
  } else {
    const float2 u = raw[n - k];
    xc = make_float2(u.x, -u.y);
  }
  const float2 e = cadd(xk, xc);
  const float2 o = cmul(csub(xk, xc), make_float2(w.x, -w.y));
  return make_float2(e.x - o.y, e.y + o.x);
}

// a * exp(-2*pi*i * m / 32) for m in [0, 16) known at compile time after unrolling.
__device__ __forceinline__ float2 rot32(float2 a, int m) {
  constexpr float kC[16] = {1.0f, 0.9807852506637573f, 0.9238795042037964f, 0.8314695954322815f,
                            0.7071067690849304f, 0.5555702447891235f, 0.3826834261417389f,
                            0.19509032368659973f, 0.0f, -0.19509032368659973f,
                            -0.3826834261417389f, -0.5555702447891235f, -0.7071067690849304f,
                            -0.8314695954322815f, -0.9238795042037964f, -0.9807852506637573f};
  constexpr float kS[16] = {0.0f, 0.19509032368659973f, 0.3826834261417389f, 0.5555702447891235f,
                            0.7071067690849304f, 0.8314695954322815f, 0.9238795042037964f,
                            0.9807852506637573f, 1.0f, 0.9807852506637573f, 0.9238795042037964f,
                            0.8314695954322815f, 0.7071067690849304f, 0.5555702447891235f,
                            0.3826834261417389f, 0.19509032368659973f};
  if (m == 0) return a;
  if (m == 8) return make_float2(a.y, -a.x);  // times -i
  return cmul(a, make_float2(kC[m], -kS[m]));
}

// Pass of the staged kernel: FIRST reads the staging buffer `st` (for PRE, the
// half-spectrum row `raw` through c2r_point), LAST writes `st`; every other read
// and write goes through the padded work arrays.
template <int LOG2N, int R, int S, bool FIRST, bool LAST, bool PRE = false>
__device__ __forceinline__ void spass(float2 (&v)[Plan<LOG2N>::P], int j, int Ns, int log2Ns,
                                      float2* st, float* sre, float* sim,
                                      const float2* __restrict__ tw, const float2* raw = nullptr,
                                      const float2* __restrict__ twl = nullptr) {
  using PL = Plan<LOG2N>;
  constexpr int N = PL::N;
  constexpr int T = PL::T;
  constexpr int NB = PL::P / R;
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    const int b = j + q * T;
    // PRE: the points idx = b + r*N/R of this butterfly need W^idx = W^b * exp(-pi*i*r/R)
    // (W = exp(-2*pi*i/(2N))): one table read, the rest compile-time rotations
    float2 wb = make_float2(1.0f, 0.0f);
    if constexpr (FIRST && PRE) wb = __ldg(twl + b);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int idx = b + r * (N / R);
      if constexpr (FIRST && PRE) {
        v[q * R + r] = c2r_point(raw, idx, N, rot32(wb, r * (16 / R)));
      } else {
        v[q * R + r] = FIRST ? st[idx] : make_float2(sre[pad(idx)], sim[pad(idx)]);
      }
    }
  }
  // The work arrays alias the staging buffer, so every pass finishes its reads
  // before any thread rewrites the buffer.
  __syncthreads();
#pragma unroll
  for (int q = 0; q < NB; ++q) {
    const int b = j + q * T;
    const int k = b & (Ns - 1);
    if (Ns > 1) {
      apply_twiddles<R, S>(&v[q * R], tw, k << (LOG2N - log2Ns - ilog2(R)));
    }
    dft<R, S>(&v[q * R]);
    const int idxD = ((b >> log2Ns) << (log2Ns + ilog2(R))) + k;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int o = idxD + r * Ns;
      if constexpr (LAST) {
        st[o] = v[q * R + r];
      } else {
        sre[pad(o)] = v[q * R + r].x;
        sim[pad(o)] = v[q * R + r].y;
      }
    }
  }
  if constexpr (!LAST) __syncthreads();
}

template <int LOG2N, int S, bool PRE = false, int PASS = 0>
__device__ __forceinline__ void run_spasses(float2 (&v)[Plan<LOG2N>::P], int j, float2* st,
                                            float* sre, float* sim, const float2* tw,
                                            const float2* raw = nullptr,
                                            const float2* twl = nullptr) {
  using PL = Plan<LOG2N>;
  if constexpr (PASS < PL::PASSES) {
    constexpr int R = (PASS == 0) ? PL::FIRST_R : 16;
    constexpr int LOG2NS = (PASS == 0) ? 0 : (ilog2(PL::FIRST_R) + 4 * (PASS - 1));
    spass<LOG2N, R, S, PASS == 0, PASS == PL::PASSES - 1, PRE>(v, j, 1 << LOG2NS, LOG2NS, st, sre,
                                                               sim, tw, raw, twl);
    run_spasses<LOG2N, S, PRE, PASS + 1>(v, j, st, sre, sim, tw, raw, twl);
  }
}

// Each of the two staging buffers holds a group's input (bulk-copied, plain
// interleaved complex values), then — after the first pass has read it into
// registers — that group's padded split work arrays, and finally its output for
// the bulk store: two ~34 KB buffers per CTA, three CTAs per SM.
template <int LOG2N>
struct BulkPlan {
  using PL = Plan<LOG2N>;
  static constexpr int GROUP = PL::TPC * PL::N;                  // complex values per group
  static constexpr int GROUP_BYTES = GROUP * 8;
  static constexpr int WORK_BYTES = PL::TPC * PL::REGION * 2 * 4;
  static constexpr int STAGE_BYTES =
      ((GROUP_BYTES > WORK_BYTES ? GROUP_BYTES : WORK_BYTES) + 127) / 128 * 128;
  static constexpr int SMEM = 2 * STAGE_BYTES + 64;
};

template <int LOG2N, int S>
__global__ void __launch_bounds__(Plan<LOG2N>::THREADS, 3)
    stockham_bulk_kernel(const float2* in, float2* out, long long groups,
                         const float2* __restrict__ tw, unsigned int* timeouts) {
  using PL = Plan<LOG2N>;
  using BP = BulkPlan<LOG2N>;
  extern __shared__ __align__(16) std::uint8_t bsmem[];
  float2* stage0 = reinterpret_cast<float2*>(bsmem);
  float2* stage1 = reinterpret_cast<float2*>(bsmem + BP::STAGE_BYTES);
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(bsmem + 2 * BP::STAGE_BYTES);
  volatile int* ok_flag = reinterpret_cast<volatile int*>(full + 2);
  const int tloc = threadIdx.x / PL::T;
  const int j = threadIdx.x % PL::T;
  const long long stride = gridDim.x;
  std::uint32_t phase[2] = {0u, 0u};
  bool pending[2] = {false, false};

  if (threadIdx.x == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_fence_init();
    for (int s = 0; s < 2; ++s) {
      const long long g = blockIdx.x + s * stride;
      if (g < groups) {
        tc::mbar_arrive_expect_tx(&full[s], BP::GROUP_BYTES);
        tc::bulk_load(s ? stage1 : stage0, in + g * BP::GROUP, BP::GROUP_BYTES, &full[s]);
        pending[s] = true;
      }
    }
  }
  __syncthreads();

  int s = 0;
  for (long long g = blockIdx.x; g < groups; g += stride, s ^= 1) {
    float2* st = (s ? stage1 : stage0);
    if (threadIdx.x == 0) {
      *ok_flag = tc::mbar_wait(&full[s], phase[s]) ? 1 : 0;
      pending[s] = false;
    }
    __syncthreads();
    if (!*ok_flag) {
      if (threadIdx.x == 0) atomicAdd(timeouts, 1u);
      break;
    }
    phase[s] ^= 1u;
    float2 v[PL::P];
    float* sre = reinterpret_cast<float*>(st) + tloc * PL::REGION * 2;
    float* sim = sre + PL::REGION;
    run_spasses<LOG2N, S>(v, j, st + tloc * PL::N, sre, sim, tw);
    tc::fence_proxy_async_smem();
    __syncthreads();  // the whole group is in the staging buffer
    if (threadIdx.x == 0) {
      tc::bulk_store(out + g * BP::GROUP, st, BP::GROUP_BYTES);
      tc::bulk_wait_read_all();  // staging buffer may be refilled
      const long long gn = g + 2 * stride;
      if (gn < groups) {
        tc::mbar_arrive_expect_tx(&full[s], BP::GROUP_BYTES);
        tc::bulk_load(st, in + gn * BP::GROUP, BP::GROUP_BYTES, &full[s]);
        pending[s] = true;
      }
    }
  }
  if (threadIdx.x == 0) {
    // drain: copies still in flight (only after a timeout) and all stores
    for (int q = 0; q < 2; ++q)
      if (pending[q] && !tc::mbar_wait(&full[q], phase[q])) atomicAdd(timeouts, 1u);
    tc::bulk_wait_all();
  }
}

// Three staging buffers, two CTAs per SM: group i computes in buffer i % 3 while group
// i + 1's load has landed or is landing in the next buffer, and the load of group i + 2 goes
// into the buffer whose store (group i - 1) was issued one group earlier, so no thread waits
// for a store to drain before the next group can start.
template <int LOG2N, int S>
__global__ void __launch_bounds__(Plan<LOG2N>::THREADS, 2)
    stockham_bulk3_kernel(const float2* in, float2* out, long long groups,
                          const float2* __restrict__ tw, unsigned int* timeouts) {
  using PL = Plan<LOG2N>;
  using BP = BulkPlan<LOG2N>;
  extern __shared__ __align__(16) std::uint8_t bsmem[];
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(bsmem + 3 * BP::STAGE_BYTES);
  volatile int* ok_flag = reinterpret_cast<volatile int*>(full + 3);
  auto stage = [&](int b) { return reinterpret_cast<float2*>(bsmem + b * BP::STAGE_BYTES); };
  const int tloc = threadIdx.x / PL::T;
  const int j = threadIdx.x % PL::T;
  const long long stride = gridDim.x;
  std::uint32_t phase[3] = {0u, 0u, 0u};
  bool pending[3] = {false, false, false};

  if (threadIdx.x == 0) {
    for (int b = 0; b < 3; ++b) tc::mbar_init(&full[b], 1);
    tc::mbar_fence_init();
    for (int b = 0; b < 2; ++b) {
      const long long g = blockIdx.x + b * stride;
      if (g < groups) {
        tc::mbar_arrive_expect_tx(&full[b], BP::GROUP_BYTES);
        tc::bulk_load(stage(b), in + g * BP::GROUP, BP::GROUP_BYTES, &full[b]);
        pending[b] = true;
      }
    }
  }
  __syncthreads();

  int b = 0;
  for (long long g = blockIdx.x; g < groups; g += stride, b = (b == 2 ? 0 : b + 1)) {
    float2* st = stage(b);
    if (threadIdx.x == 0) {
      *ok_flag = tc::mbar_wait(&full[b], phase[b]) ? 1 : 0;
      pending[b] = false;
    }
    __syncthreads();
    if (!*ok_flag) {
      if (threadIdx.x == 0) atomicAdd(timeouts, 1u);
      break;
    }
    phase[b] ^= 1u;
    float2 v[PL::P];
    float* sre = reinterpret_cast<float*>(st) + tloc * PL::REGION * 2;
    float* sim = sre + PL::REGION;
    run_spasses<LOG2N, S>(v, j, st + tloc * PL::N, sre, sim, tw);
    tc::fence_proxy_async_smem();
    __syncthreads();  // the whole group is in the staging buffer
    if (threadIdx.x == 0) {
      tc::bulk_store(out + g * BP::GROUP, st, BP::GROUP_BYTES);
      tc::bulk_wait_read_but_one();  // the previous group's store has read its buffer
      const long long gn = g + 2 * stride;
      const int bn = b == 0 ? 2 : b - 1;  // (b + 2) % 3: the previous group's buffer
      if (gn < groups) {
        tc::mbar_arrive_expect_tx(&full[bn], BP::GROUP_BYTES);
        tc::bulk_load(stage(bn), in + gn * BP::GROUP, BP::GROUP_BYTES, &full[bn]);
        pending[bn] = true;
      }
    }
  }
  if (threadIdx.x == 0) {
    // drain: copies still in flight (only after a timeout) and all stores
    for (int q = 0; q < 3; ++q)
      if (pending[q] && !tc::mbar_wait(&full[q], phase[q])) atomicAdd(timeouts, 1u);
    tc::bulk_wait_all();
  }
}

template <int LOG2N, int S>
cudaError_t launch_bulk_len(const float2* in, float2* out, long long groups, const float2* tw,
                            unsigned int* timeouts, cudaStream_t stream) {
  using BP = BulkPlan<LOG2N>;
  const int sms = sm_count(current_device());
  if constexpr (LOG2N >= 11) {
    constexpr int smem3 = 3 * BP::STAGE_BYTES + 64;
    auto kern = stockham_bulk3_kernel<LOG2N, S>;
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem3);
    if (e != cudaSuccess) return e;
    const long long cap = static_cast<long long>(sms > 0 ? sms : 148) * 2;
    const unsigned grid = static_cast<unsigned>(groups < cap ? groups : cap);
    kern<<<grid, Plan<LOG2N>::THREADS, smem3, stream>>>(in, out, groups, tw, timeouts);
    return cudaGetLastError();
  }
  auto kern = stockham_bulk_kernel<LOG2N, S>;
  const cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BP::SMEM);
  if (e != cudaSuccess) return e;
  const long long cap = static_cast<long long>(sms > 0 ? sms : 148) * 3;
  const unsigned grid = static_cast<unsigned>(groups < cap ? groups : cap);
  kern<<<grid, Plan<LOG2N>::THREADS, BP::SMEM, stream>>>(in, out, groups, tw, timeouts);
  return cudaGetLastError();
}

template <int S>
cudaError_t dispatch_bulk(int log2n, const float2* in, float2* out, long long groups,
                          const float2* tw, unsigned int* to, cudaStream_t st) {
  switch (log2n) {
    case 4: return launch_bulk_len<4, S>(in, out, groups, tw, to, st);
    case 5: return launch_bulk_len<5, S>(in, out, groups, tw, to, st);
    case 6: return launch_bulk_len<6, S>(in, out, groups, tw, to, st);
    case 7: return launch_bulk_len<7, S>(in, out, groups, tw, to, st);
    case 8: return launch_bulk_len<8, S>(in, out, groups, tw, to, st);
    case 9: return launch_bulk_len<9, S>(in, out, groups, tw, to, st);
    case 10: return launch_bulk_len<10, S>(in, out, groups, tw, to, st);
    case 11: return launch_bulk_len<11, S>(in, out, groups, tw, to, st);
    case 12: return launch_bulk_len<12, S>(in, out, groups, tw, to, st);
    default: return cudaErrorInvalidValue;
  }
}

unsigned int* bulk_timeout_counter() {
  static std::mutex mu;
  static std::array<unsigned int*, 64> addr{};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fft_bulk_timeouts) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    addr[dev] = static_cast<unsigned int*>(p);
  }
  return addr[dev];
}

// ---------------------------------------------------------------------------
// Real-data variants of the bulk kernel: R2C / C2R of even length L = 2N through
// the length-N complex transform of the reals read as N pairs.  Rows are dense on
// both sides (reals at r * L, half spectra at r * (N + 1)).
//
// R2C: the group's reals arrive by bulk copy exactly as a C2C group does; after the
// last pass the TPC rows Z sit in natural order in the staging buffer and the post-
// pass X[k] = E - i W^k D, E = (Z[k] + conj Z[N-k])/2, D = (Z[k] - conj Z[N-k])/2,
// k = 0 .. N (W = exp(-2*pi*i/L), Z[N] = Z[0]) stores the N + 1 entries of each row
// straight to global memory: one HBM read and one HBM write per element, no
// intermediate.  Entries k and N - k come from the same two values: with
// P = W^k D, X[k] = E - i P and, since W^(N-k) = -conj(W^k), X[N-k] = conj(E) -
// i conj(P); so one thread forms both from two shared-memory reads and one twiddle.

__device__ __forceinline__ void r2c_pair(const float2* z, int k, int n,
                                         const float2* __restrict__ twl, float2& xk,
                                         float2& xnk) {
  const float2 a = z[k];
  const float2 c = z[k == 0 ? 0 : n - k];
  const float2 e = make_float2(0.5f * (a.x + c.x), 0.5f * (a.y - c.y));
  const float2 d = make_float2(0.5f * (a.x - c.x), 0.5f * (a.y + c.y));
  const float2 q = cmul(__ldg(twl + k), d);
  xk = make_float2(e.x + q.y, e.y - q.x);
  xnk = make_float2(e.x - q.y, -e.y - q.x);
}

template <int LOG2N>
__global__ void __launch_bounds__(Plan<LOG2N>::THREADS, 3)
    r2c_bulk_kernel(const float* in, float2* out, long long groups, const float2* __restrict__ tw,
                    const float2* __restrict__ twl, unsigned int* timeouts) {
  using PL = Plan<LOG2N>;
  using BP = BulkPlan<LOG2N>;
  constexpr int N = PL::N;
  constexpr int H = N + 1;
  extern __shared__ __align__(16) std::uint8_t bsmem[];
  float2* stage0 = reinterpret_cast<float2*>(bsmem);
  float2* stage1 = reinterpret_cast<float2*>(bsmem + BP::STAGE_BYTES);
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(bsmem + 2 * BP::STAGE_BYTES);
  volatile int* ok_flag = reinterpret_cast<volatile int*>(full + 2);
  const int tloc = threadIdx.x / PL::T;
  const int j = threadIdx.x % PL::T;
  const long long stride = gridDim.x;
  std::uint32_t phase[2] = {0u, 0u};
  bool pending[2] = {false, false};
  const float2* in2 = reinterpret_cast<const float2*>(in);

  if (threadIdx.x == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_fence_init();
    for (int s = 0; s < 2; ++s) {
      const long long g = blockIdx.x + s * stride;
      if (g < groups) {
        tc::mbar_arrive_expect_tx(&full[s], BP::GROUP_BYTES);
        tc::bulk_load(s ? stage1 : stage0, in2 + g * BP::GROUP, BP::GROUP_BYTES, &full[s]);
        pending[s] = true;
      }
    }
  }
  __syncthreads();

  int s = 0;
  for (long long g = blockIdx.x; g < groups; g += stride, s ^= 1) {
    float2* st = (s ? stage1 : stage0);
    if (threadIdx.x == 0) {
      *ok_flag = tc::mbar_wait(&full[s], phase[s]) ? 1 : 0;
      pending[s] = false;
    }
    __syncthreads();
    if (!*ok_flag) {
      if (threadIdx.x == 0) atomicAdd(timeouts, 1u);
      break;
    }
    phase[s] ^= 1u;
    float2 v[PL::P];
    float* sre = reinterpret_cast<float*>(st) + tloc * PL::REGION * 2;
    float* sim = sre + PL::REGION;
    run_spasses<LOG2N, -1>(v, j, st + tloc * N, sre, sim, tw);
    __syncthreads();  // every row of the group is in natural order in `st`
    float2* o = out + g * (PL::TPC * static_cast<long long>(H));
    constexpr int PAIRS = N / 2 + 1;  // k = 0 .. N/2 with partners N .. N/2
    for (int i = threadIdx.x; i < PL::TPC * PAIRS; i += PL::THREADS) {
      const int row = i / PAIRS;
      const int k = i - row * PAIRS;
      float2 xk, xnk;
      r2c_pair(st + row * N, k, N, twl, xk, xnk);
      o[row * H + k] = xk;
      if (2 * k != N) o[row * H + N - k] = xnk;
    }
    __syncthreads();  // staging buffer read completely
    if (threadIdx.x == 0) {
      const long long gn = g + 2 * stride;
      if (gn < groups) {
        tc::mbar_arrive_expect_tx(&full[s], BP::GROUP_BYTES);
        tc::bulk_load(st, in2 + gn * BP::GROUP, BP::GROUP_BYTES, &full[s]);
        pending[s] = true;
      }
    }
  }
  if (threadIdx.x == 0) {
    for (int q = 0; q < 2; ++q)
      if (pending[q] && !tc::mbar_wait(&full[q], phase[q])) atomicAdd(timeouts, 1u);
  }
}

// C2R: the group's half-spectrum rows (N + 1 entries each, not 16-byte aligned in
// general, so 8-byte cp.async copies) are prefetched two groups ahead into the
// staging ring; the first pass forms its butterfly inputs Z'[k] from them
// (c2r_point), and the last pass's output — x[2n] + i x[2n+1] of each row — leaves
// by one bulk store.
__device__ __forceinline__ void cp_async8(void* dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(tc::smem_addr(dst_smem)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_one() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// With an even number of rows per group (half length <= 2048) a group's half
// spectra are 16-byte aligned and a multiple of 16 bytes long, so one bulk copy
// per group completing on an mbarrier replaces the 8-byte copies.
template <int LOG2N, bool BULK>
__global__ void __launch_bounds__(Plan<LOG2N>::THREADS, 3)
    c2r_bulk_kernel(const float2* in, float* out, long long groups, const float2* __restrict__ tw,
                    const float2* __restrict__ twl, unsigned int* timeouts) {
  using PL = Plan<LOG2N>;
  using BP = BulkPlan<LOG2N>;
  constexpr int N = PL::N;
  constexpr int H = N + 1;
  constexpr int ROWS = PL::TPC * H;  // complex values of a group's half spectra
  static_assert(ROWS * 8 <= BP::STAGE_BYTES, "half-spectrum rows exceed the staging buffer");
  static_assert(!BULK || (ROWS * 8) % 16 == 0, "bulk copies need 16-byte multiples");
  extern __shared__ __align__(16) std::uint8_t bsmem[];
  float2* stage[2] = {reinterpret_cast<float2*>(bsmem),
                      reinterpret_cast<float2*>(bsmem + BP::STAGE_BYTES)};
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(bsmem + 2 * BP::STAGE_BYTES);
  volatile int* ok_flag = reinterpret_cast<volatile int*>(full + 2);
  const int tloc = threadIdx.x / PL::T;
  const int j = threadIdx.x % PL::T;
  const long long stride = gridDim.x;
  float2* out2 = reinterpret_cast<float2*>(out);
  std::uint32_t phase[2] = {0u, 0u};
  bool pending[2] = {false, false};

  // BULK: thread 0 issues the copy of group g into stage s; otherwise every thread
  // copies its share and commits one cp.async group (empty or not, which keeps
  // the wait counts aligned).
  auto fetch = [&](int s, long long g) {
    if constexpr (BULK) {
      if (threadIdx.x == 0 && g < groups) {
        tc::mbar_arrive_expect_tx(&full[s], ROWS * 8);
        tc::bulk_load(stage[s], in + g * ROWS, ROWS * 8, &full[s]);
        pending[s] = true;
      }
    } else {
      if (g < groups) {
        const float2* src = in + g * ROWS;
        for (int i = threadIdx.x; i < ROWS; i += PL::THREADS) cp_async8(stage[s] + i, src + i);
      }
      cp_async_commit();
    }
  };
  if constexpr (BULK) {
    if (threadIdx.x == 0) {
      tc::mbar_init(&full[0], 1);
      tc::mbar_init(&full[1], 1);
      tc::mbar_fence_init();
    }
  }
  fetch(0, blockIdx.x);
  fetch(1, blockIdx.x + stride);
  __syncthreads();

  int s = 0;
  for (long long g = blockIdx.x; g < groups; g += stride, s ^= 1) {
    float2* st = stage[s];
    if constexpr (BULK) {
      if (threadIdx.x == 0) {
        *ok_flag = tc::mbar_wait(&full[s], phase[s]) ? 1 : 0;
        pending[s] = false;
      }
      __syncthreads();
      if (!*ok_flag) {
        if (threadIdx.x == 0) atomicAdd(timeouts, 1u);
        break;
      }
      phase[s] ^= 1u;
    } else {
      cp_async_wait_one();  // this thread's copies of group g have landed
      __syncthreads();      // and everyone else's
    }
    float2 v[PL::P];
    float* sre = reinterpret_cast<float*>(st) + tloc * PL::REGION * 2;
    float* sim = sre + PL::REGION;
    run_spasses<LOG2N, 1, true>(v, j, st + tloc * N, sre, sim, tw, st + tloc * H, twl);
    tc::fence_proxy_async_smem();
    __syncthreads();  // the whole group's output is in the staging buffer
    if (threadIdx.x == 0) {
      tc::bulk_store(out2 + g * BP::GROUP, st, BP::GROUP_BYTES);
      tc::bulk_wait_read_all();  // the staging buffer may be refilled
    }
    if constexpr (BULK) {
      fetch(s, g + 2 * stride);
    } else {
      __syncthreads();  // every thread's refill waits for the store's read
      fetch(s, g + 2 * stride);
    }
  }
  if constexpr (BULK) {
    if (threadIdx.x == 0) {
      for (int q = 0; q < 2; ++q)
        if (pending[q] && !tc::mbar_wait(&full[q], phase[q])) atomicAdd(timeouts, 1u);
    }
  } else {
    cp_async_wait_all();
  }
  if (threadIdx.x == 0) tc::bulk_wait_all();
}

template <int LOG2N>
cudaError_t launch_real_bulk_len(bool r2c, const void* in, void* out, long long groups,
                                 const float2* tw, const float2* twl, unsigned int* timeouts,
                                 cudaStream_t stream) {
  using BP = BulkPlan<LOG2N>;
  const int sms = sm_count(current_device());
  const long long cap = static_cast<long long>(sms > 0 ? sms : 148) * 3;
  const unsigned grid = static_cast<unsigned>(groups < cap ? groups : cap);
  if (r2c) {
    auto kern = r2c_bulk_kernel<LOG2N>;
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BP::SMEM);
    if (e != cudaSuccess) return e;
    kern<<<grid, Plan<LOG2N>::THREADS, BP::SMEM, stream>>>(
        static_cast<const float*>(in), static_cast<float2*>(out), groups, tw, twl, timeouts);
  } else {
    constexpr bool kBulk = Plan<LOG2N>::TPC % 2 == 0;
    auto kern = c2r_bulk_kernel<LOG2N, kBulk>;
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BP::SMEM);
    if (e != cudaSuccess) return e;
    kern<<<grid, Plan<LOG2N>::THREADS, BP::SMEM, stream>>>(
        static_cast<const float2*>(in), static_cast<float*>(out), groups, tw, twl, timeouts);
  }
  return cudaGetLastError();
}

}  // namespace

bool single_pass_supported(std::int64_t n) noexcept {
  return n >= 2 && n <= kMaxSinglePass && (n & (n - 1)) == 0;
}

cudaError_t launch_stockham(std::int64_t n, int sign, const Batch1D& b,
                            cudaStream_t stream) noexcept {
  if (!single_pass_supported(n)) return cudaErrorInvalidValue;
  if (b.batch <= 0) return cudaSuccess;
  const int log2n = __builtin_ctzll(static_cast<unsigned long long>(n));
  // Contiguous batches of 16..4096 points take the bulk-copy pipelined kernel for
  // all whole groups; any remainder (and every other layout) the register kernel.
  const bool contiguous = b.in_stride == 1 && b.out_stride == 1 && b.in_outer == n &&
                          b.out_outer == n && b.inner_count == 1 && b.post_tw == nullptr &&
                          aligned_to(b.in, 16) && aligned_to(b.out, 16);
  if (contiguous && n >= 16 && n <= 4096) {
    const long long per_group = 4096 / n;  // TPC transforms of n points = 4096 values
    const long long groups = b.batch / per_group;
    unsigned int* to = bulk_timeout_counter();
    if (groups > 0 && to != nullptr) {
      const cudaError_t e = sign < 0
                                ? dispatch_bulk<-1>(log2n, b.in, b.out, groups, b.tw, to, stream)
                                : dispatch_bulk<1>(log2n, b.in, b.out, groups, b.tw, to, stream);
      if (e != cudaSuccess) return e;
      const long long done = groups * per_group;
      if (done == b.batch) return cudaSuccess;
      Batch1D rest = b;
      rest.in = b.in + done * n;
      rest.out = b.out + done * n;
      rest.batch = b.batch - done;
      return sign < 0 ? dispatch<-1>(log2n, rest, stream) : dispatch<1>(log2n, rest, stream);
    }
  }
  return sign < 0 ? dispatch<-1>(log2n, b, stream) : dispatch<1>(log2n, b, stream);
}

std::int64_t real_bulk_rows_per_group(std::int64_t n) noexcept {
  return (n >= 16 && n <= 4096 && (n & (n - 1)) == 0) ? 4096 / n : 0;
}

bool real_bulk_aligned(bool r2c, std::int64_t n, const void* in, const void* out) noexcept {
  const std::int64_t per = real_bulk_rows_per_group(n);
  if (per == 0) return false;
  // C2R groups of an even number of half-spectrum rows are bulk-copied
  const int in_align = (r2c || per % 2 == 0) ? 16 : 8;
  return aligned_to(in, in_align) && aligned_to(out, r2c ? 8 : 16);
}

cudaError_t launch_real_bulk(bool r2c, std::int64_t n, const void* in, void* out,
                             long long groups, const float2* tw, const float2* twl,
                             cudaStream_t stream) noexcept {
  if (!real_bulk_aligned(r2c, n, in, out)) return cudaErrorInvalidValue;
  if (groups <= 0) return cudaSuccess;
  unsigned int* to = bulk_timeout_counter();
  if (to == nullptr) return cudaErrorInvalidValue;
  switch (__builtin_ctzll(static_cast<unsigned long long>(n))) {
    case 4: return launch_real_bulk_len<4>(r2c, in, out, groups, tw, twl, to, stream);
    case 5: return launch_real_bulk_len<5>(r2c, in, out, groups, tw, twl, to, stream);
    case 6: return launch_real_bulk_len<6>(r2c, in, out, groups, tw, twl, to, stream);
    case 7: return launch_real_bulk_len<7>(r2c, in, out, groups, tw, twl, to, stream);
    case 8: return launch_real_bulk_len<8>(r2c, in, out, groups, tw, twl, to, stream);
    case 9: return launch_real_bulk_len<9>(r2c, in, out, groups, tw, twl, to, stream);
    case 10: return launch_real_bulk_len<10>(r2c, in, out, groups, tw, twl, to, stream);
    case 11: return launch_real_bulk_len<11>(r2c, in, out, groups, tw, twl, to, stream);
    case 12: return launch_real_bulk_len<12>(r2c, in, out, groups, tw, twl, to, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mb200::fft
