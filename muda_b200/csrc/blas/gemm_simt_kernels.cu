// gemm_simt_kernels.cu — register-blocked FFMA GEMM (column-major, any layout).
//
// Per-element arithmetic follows the reference's batched kernels
// (libraries/blas/shaders/cublas_kernels.metal:969-1045): products of op(A) and
// op(B) accumulated with fp32 fma, then C = fma(alpha, acc, beta == 0 ? 0 :
// beta * C), 16-bit outputs rounded to nearest even.  Only the order in which
// the k-products are added differs from the reference's sequential loop.
//
// Blocking: a CTA of 256 threads owns a BM x BN tile of C and walks k in steps
// of BK.  op(A) and op(B) tiles are staged k-major in shared memory (two
// buffers; the next tile is fetched into registers while the current one is
// multiplied), each thread accumulates a TM x TN sub-tile in registers and
// reads its operands as 16-byte vectors, so every shared-memory load feeds
// TM*TN/((TM+TN)/4) FFMAs.  Global loads are coalesced along whichever
// dimension is contiguous for the given transpose.  The tile shape is chosen so
// that the grid covers the 148 SMs (a 1024^3 problem runs as 128 tiles of
// 128 x 64).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "blas/gemm.hpp"
#include "common/device.hpp"

namespace mb200::blas {
namespace {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (sizeof(T) == 4) {
    return v;
  } else if constexpr (std::is_same_v<T, __half>) {
    return __half2float(v);
  } else {
    return __bfloat162float(v);
  }
}

template <typename T>
__device__ __forceinline__ T from_f(float v) {
  if constexpr (sizeof(T) == 4) {
    return v;
  } else if constexpr (std::is_same_v<T, __half>) {
    return __float2half_rn(v);
  } else {
    return __float2bfloat16_rn(v);
  }
}

template <typename T, int BM, int BN, int BK, int TM, int TN, bool TA, bool TB>
__global__ void __launch_bounds__(kThreads) gemm_simt(const GemmArgs g) {
  constexpr int A_PER = BM * BK / kThreads;
  constexpr int B_PER = BN * BK / kThreads;
  constexpr int TX = BM / TM;  // threads along m
  static_assert(TX * (BN / TN) == kThreads, "tile does not match the thread count");
  // Rows padded by 4 words: the transposing stores (8 consecutive k per 8 lanes)
  // land in distinct banks, and rows stay 16-byte aligned for the vector reads.
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN + 4];

  const float alpha = g.alpha_dev ? *g.alpha_dev : g.alpha;
  const float beta = g.beta_dev ? *g.beta_dev : g.beta;
  const int tid = threadIdx.x;
  const int tm = tid % TX;
  const int tn = tid / TX;
  const int m0 = blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;

  for (int z = blockIdx.z; z < g.batch; z += gridDim.z) {
    const T* A = static_cast<const T*>(g.a) + z * g.stride_a;
    const T* B = static_cast<const T*>(g.b) + z * g.stride_b;
    T* Cm = static_cast<T*>(g.c) + z * g.stride_c;

    float ra[A_PER], rb[B_PER];
    auto fetch = [&](int k0) {
#pragma unroll
      for (int s = 0; s < A_PER; ++s) {
        const int idx = tid + s * kThreads;
        const int i = TA ? idx / BK : idx % BM;
        const int p = TA ? idx % BK : idx / BM;
        const int gi = m0 + i, gp = k0 + p;
        ra[s] = (gi < g.m && gp < g.k)
                    ? to_f(TA ? A[gp + static_cast<std::int64_t>(gi) * g.lda]
                              : A[gi + static_cast<std::int64_t>(gp) * g.lda])
                    : 0.0f;
      }
#pragma unroll
      for (int s = 0; s < B_PER; ++s) {
        const int idx = tid + s * kThreads;
        const int j = TB ? idx % BN : idx / BK;
        const int p = TB ? idx / BN : idx % BK;
        const int gj = n0 + j, gp = k0 + p;
        rb[s] = (gj < g.n && gp < g.k)
                    ? to_f(TB ? B[gj + static_cast<std::int64_t>(gp) * g.ldb]
                              : B[gp + static_cast<std::int64_t>(gj) * g.ldb])
                    : 0.0f;
      }
    };
    auto stash = [&](int buf) {
#pragma unroll
      for (int s = 0; s < A_PER; ++s) {
        const int idx = tid + s * kThreads;
        const int i = TA ? idx / BK : idx % BM;
        const int p = TA ? idx % BK : idx / BM;
        As[buf][p][i] = ra[s];
      }
#pragma unroll
      for (int s = 0; s < B_PER; ++s) {
        const int idx = tid + s * kThreads;
        const int j = TB ? idx % BN : idx / BK;
        const int p = TB ? idx / BN : idx % BK;
        Bs[buf][p][j] = rb[s];
      }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

    int buf = 0;
    fetch(0);
    stash(0);
    __syncthreads();
    for (int k0 = 0; k0 < g.k; k0 += BK) {
      const bool more = k0 + BK < g.k;
      if (more) fetch(k0 + BK);
#pragma unroll
      for (int p = 0; p < BK; ++p) {
        float av[TM], bv[TN];
#pragma unroll
        for (int i = 0; i < TM; i += 4) {
          // the thread's rows come in groups of 4 spaced 4*TX apart, so the 16 lanes
          // along m read 16 consecutive float4 (conflict free)
          const float4 t = *reinterpret_cast<const float4*>(&As[buf][p][i * TX + tm * 4]);
          av[i] = t.x;
          av[i + 1] = t.y;
          av[i + 2] = t.z;
          av[i + 3] = t.w;
        }
#pragma unroll
        for (int j = 0; j < TN; j += 4) {
          const float4 t = *reinterpret_cast<const float4*>(&Bs[buf][p][tn * TN + j]);
          bv[j] = t.x;
          bv[j + 1] = t.y;
          bv[j + 2] = t.z;
          bv[j + 3] = t.w;
        }
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      if (more) {
        stash(buf ^ 1);
        __syncthreads();
        buf ^= 1;
      }
    }

#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int gj = n0 + tn * TN + j;
      if (gj >= g.n) continue;
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const int gi = m0 + (i / 4) * 4 * TX + tm * 4 + (i % 4);
        if (gi >= g.m) continue;
        T* cp = Cm + gi + static_cast<std::int64_t>(gj) * g.ldc;
        const float prev = (beta == 0.0f) ? 0.0f : beta * to_f(*cp);
        *cp = from_f<T>(fmaf(alpha, acc[i][j], prev));
      }
    }
    __syncthreads();  // shared tiles are reused by the next batch entry
  }
}

template <typename T, int BM, int BN, int TM, int TN>
cudaError_t launch_tile(const GemmArgs& g, cudaStream_t st) {
  const dim3 grid((g.m + BM - 1) / BM, (g.n + BN - 1) / BN, g.batch < 65535 ? g.batch : 65535);
  if (!g.trans_a && !g.trans_b)
    gemm_simt<T, BM, BN, 8, TM, TN, false, false><<<grid, kThreads, 0, st>>>(g);
  else if (g.trans_a && !g.trans_b)
    gemm_simt<T, BM, BN, 8, TM, TN, true, false><<<grid, kThreads, 0, st>>>(g);
  else if (!g.trans_a && g.trans_b)
    gemm_simt<T, BM, BN, 8, TM, TN, false, true><<<grid, kThreads, 0, st>>>(g);
  else
    gemm_simt<T, BM, BN, 8, TM, TN, true, true><<<grid, kThreads, 0, st>>>(g);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_typed(const GemmArgs& g, cudaStream_t st) {
  const int sms = sm_count(current_device());
  const std::int64_t target = sms > 0 ? sms : 148;
  auto tiles = [&](int bm, int bn) {
    return static_cast<std::int64_t>((g.m + bm - 1) / bm) * ((g.n + bn - 1) / bn) * g.batch;
  };
  if (tiles(128, 128) >= target) return launch_tile<T, 128, 128, 8, 8>(g, st);
  if (tiles(128, 64) >= (target * 3) / 4) return launch_tile<T, 128, 64, 8, 4>(g, st);
  return launch_tile<T, 64, 64, 4, 4>(g, st);
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t stream) noexcept {
  if (g.m <= 0 || g.n <= 0 || g.batch <= 0) return cudaSuccess;
  switch (g.type) {
    case Elem::kF32:
      return launch_typed<float>(g, stream);
    case Elem::kF16:
      return launch_typed<__half>(g, stream);
    case Elem::kBF16:
      return launch_typed<__nv_bfloat16>(g, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mb200::blas
