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
// that the grid covers the 148 SMs.  This generic kernel serves 16-bit types and
// unaligned fp32 operands; aligned fp32 runs gemm_ffma_vec below (whole grid, or
// stream-K when the 128 x 128 tiles number fewer than the SMs).
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

// Split-K form (batch 1): split z = blockIdx.z sums k in [z * kchunk, (z + 1) * kchunk)
// and writes the raw sums, column-major m x n, to ws + z * m * n; simt_split_reduce adds
// the splits in order and applies alpha and beta.
struct SplitK {
  float* ws;
  int kchunk;
};

template <typename T, int BM, int BN, int BK, int TM, int TN, bool TA, bool TB, bool SPLIT = false>
__global__ void __launch_bounds__(kThreads) gemm_simt(const GemmArgs g, const SplitK sk = {}) {
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

  const int k_begin = SPLIT ? static_cast<int>(blockIdx.z) * sk.kchunk : 0;
  const int k_end = SPLIT ? min(g.k, k_begin + sk.kchunk) : g.k;
  for (int z = SPLIT ? 0 : blockIdx.z; z < (SPLIT ? 1 : g.batch); z += gridDim.z) {
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
        ra[s] = (gi < g.m && gp < k_end)
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
        rb[s] = (gj < g.n && gp < k_end)
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
    fetch(k_begin);
    stash(0);
    __syncthreads();
    for (int k0 = k_begin; k0 < k_end; k0 += BK) {
      const bool more = k0 + BK < k_end;
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
        if constexpr (SPLIT) {
          sk.ws[(static_cast<std::int64_t>(blockIdx.z) * g.n + gj) * g.m + gi] = acc[i][j];
          continue;
        }
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

// C = alpha * (sum of the splits in order) + beta * C.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    simt_split_reduce(const GemmArgs g, const float* __restrict__ ws, int splits) {
  const float alpha = g.alpha_dev ? *g.alpha_dev : g.alpha;
  const float beta = g.beta_dev ? *g.beta_dev : g.beta;
  const std::int64_t mn = static_cast<std::int64_t>(g.m) * g.n;
  T* Cm = static_cast<T*>(g.c);
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * kThreads + threadIdx.x; t < mn;
       t += static_cast<std::int64_t>(gridDim.x) * kThreads) {
    float sum = 0.0f;
    for (int z = 0; z < splits; ++z) sum += __ldcs(ws + z * mn + t);
    const std::int64_t gi = t % g.m, gj = t / g.m;
    T* cp = Cm + gi + gj * g.ldc;
    const float prev = (beta == 0.0f) ? 0.0f : beta * to_f(*cp);
    *cp = from_f<T>(fmaf(alpha, sum, prev));
  }
}

// ---------------------------------------------------------------------------------
// fp32 FFMA kernel for 16-byte aligned operands (the cublasSgemm path under
// CUBLAS_PEDANTIC_MATH).  Same per-element arithmetic and tile ownership as
// gemm_simt<float, 128, 128, 8, 8, 8>, with the operand traffic cut down so that the
// FFMA pipe issues nearly every cycle:
//  - k steps of 16 (one barrier per 1024 FFMAs per thread);
//  - an operand whose m (or n) index is contiguous in memory (A untransposed,
//    B transposed) is copied straight into the k-major shared tile with 16-byte
//    cp.async, no registers involved;
//  - an operand whose k index is contiguous (A transposed, B untransposed) is read
//    with 16-byte loads one step ahead and written transposed, lane pairs covering
//    32 contiguous bytes of a column (full sectors) and the stores bank-conflict free
//    (rows of 132 words);
//  - addresses advance by pointer increments; only tiles at the matrix edge test
//    bounds (whole 4-element chunks, so m, n and k must be multiples of 4);
//  - at most 128 registers, two CTAs (16 warps) per SM.
// Output columns are written with 16-byte stores when C allows it.
namespace vec {

constexpr int BM = 128, BN = 128, BK = 16;
constexpr int LDS = BM + 4;              // words per k row of a shared tile
constexpr int kTile = BK * LDS;          // words per operand tile

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  const int bytes = valid ? 16 : 0;  // 0: the 16 bytes are zero-filled, nothing is read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// One operand tile: element (r, p) of op(X), r along m (or n), p along k.
// KCONTIG: X[p + r * ld] (k contiguous), else X[r + p * ld].
template <bool KCONTIG>
struct Operand {
  const float* base;  // element (r0, k_begin) of this CTA's panel
  std::int64_t ld;
  int rows_left;      // valid rows from r0 (may exceed 128)

  // chunk s (0, 1) of this thread: 4 consecutive elements along the contiguous index
  __device__ __forceinline__ void chunk(int s, int tid, int& r, int& p) const {
    if constexpr (KCONTIG) {
      r = (tid >> 1) & (BM - 1);     // 128 rows, lane pairs share a row
      p = ((tid & 1) + 2 * s) * 4;   // k chunks 0..3
    } else {
      const int c = tid + 256 * s;
      r = (c & 31) * 4;              // 32 chunks of 4 along m
      p = c >> 5;                    // 16 k rows
    }
  }
  __device__ __forceinline__ const float* at(int r, int p, int k0) const {
    return KCONTIG ? base + (k0 + p) + static_cast<std::int64_t>(r) * ld
                   : base + r + static_cast<std::int64_t>(k0 + p) * ld;
  }
};

// Stream-K form for a batch-1 problem with fewer tiles than SMs.  The k steps of all
// tiles, tile after tile (tile t = m tile t % tiles_m, n tile t / tiles_m), are cut
// into `ctas` equal runs, CTA c taking steps [c*total/ctas, (c+1)*total/ctas); every
// SM then gets the same work.  A run covers the end of one tile and the start of the
// following ones: each piece's raw sums go to workspace slot c + t (128 x 128,
// column-major; slots are distinct because t never decreases with c), and
// ffma_stream_reduce adds the pieces of each tile in CTA order, i.e. in k order, so
// the result does not depend on scheduling.
struct StreamK {
  int tiles_m;
  int ktiles;          // k steps of BK per tile
  long long total;     // tiles * ktiles
  int ctas;
};
constexpr int kSlot = BM * BN;

__device__ __forceinline__ long long run_begin(long long c, const StreamK& sk) {
  return c * sk.total / sk.ctas;
}
// The CTA whose run holds k step s.
__device__ __forceinline__ int cta_of(long long s, const StreamK& sk) {
  return static_cast<int>(((s + 1) * sk.ctas - 1) / sk.total);
}

// STREAM false: one 128 x 128 tile of C per CTA (grid x, y), batch entries along grid
// z, C = alpha * op(A) op(B) + beta * C (beta == 0: C not read), 16-byte stores when C
// allows.  STREAM true: the CTA's run of k steps (StreamK), raw sums to the workspace.
// Row tm*4 + r + 64*h of a tile is held in acc[4h + r][.], column tn*8 + j in acc[.][j].
// (One kernel body for both forms: the tile loop compiles measurably faster inline
// than behind a helper function.)
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

template <bool TA, bool TB, bool STREAM>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_ffma_vec(const GemmArgs g, float* __restrict__ ws, const StreamK sk) {
  __shared__ __align__(16) float smem[2][2][kTile];  // [buffer][A, B][k][m or n]

  const float alpha = g.alpha_dev ? *g.alpha_dev : g.alpha;
  const float beta = g.beta_dev ? *g.beta_dev : g.beta;
  const int tid = threadIdx.x;
  const int tm = tid % 16, tn = tid / 16;
  long long s = STREAM ? run_begin(blockIdx.x, sk) : 0;
  const long long s_end = STREAM ? run_begin(blockIdx.x + 1, sk) : 0;

  for (int z = STREAM ? 0 : blockIdx.z; STREAM ? s < s_end : z < g.batch;
       z += STREAM ? 0 : gridDim.z) {
    int m0, n0, k_begin, k_end, t = 0;
    long long seg_end = 0;
    if constexpr (STREAM) {
      t = static_cast<int>(s / sk.ktiles);
      const long long t0 = static_cast<long long>(t) * sk.ktiles;
      seg_end = min(s_end, t0 + sk.ktiles);
      m0 = (t % sk.tiles_m) * BM;
      n0 = (t / sk.tiles_m) * BN;
      k_begin = static_cast<int>(s - t0) * BK;
      k_end = min(g.k, static_cast<int>(seg_end - t0) * BK);
    } else {
      m0 = blockIdx.x * BM;
      n0 = blockIdx.y * BN;
      k_begin = 0;
      k_end = g.k;
    }
    const float* A = static_cast<const float*>(g.a) + z * g.stride_a;
    const float* B = static_cast<const float*>(g.b) + z * g.stride_b;
    // op(A)(i, p): A[i + p*lda] untransposed (m contiguous), A[p + i*lda] transposed
    const Operand<TA> opa{TA ? A + k_begin + static_cast<std::int64_t>(m0) * g.lda
                             : A + m0 + static_cast<std::int64_t>(k_begin) * g.lda,
                          g.lda, g.m - m0};
    // op(B)(p, j): B[p + j*ldb] untransposed (k contiguous), B[j + p*ldb] transposed
    const Operand<!TB> opb{!TB ? B + k_begin + static_cast<std::int64_t>(n0) * g.ldb
                               : B + n0 + static_cast<std::int64_t>(k_begin) * g.ldb,
                           g.ldb, g.n - n0};
    const int klen = k_end - k_begin;

    float4 ra[2], rb[2];  // k-contiguous operands, one step ahead
    auto issue = [&](int k0, int buf) {
      const bool full_k = k0 + BK <= klen;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        int r, p;
        opa.chunk(q, tid, r, p);
        const bool ok = r < opa.rows_left && (full_k || k0 + p < klen);
        if constexpr (TA) {
          ra[q] = ok ? __ldg(reinterpret_cast<const float4*>(opa.at(r, p, k0)))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
          cp_async16(&smem[buf][0][p * LDS + r], ok ? opa.at(r, p, k0) : opa.base, ok);
        }
        opb.chunk(q, tid, r, p);
        const bool okb = r < opb.rows_left && (full_k || k0 + p < klen);
        if constexpr (!TB) {
          rb[q] = okb ? __ldg(reinterpret_cast<const float4*>(opb.at(r, p, k0)))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
          cp_async16(&smem[buf][1][p * LDS + r], okb ? opb.at(r, p, k0) : opb.base, okb);
        }
      }
      cp_async_commit();
    };
    auto stash = [&](int buf) {  // the k-contiguous operands, written k-major
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        int r, p;
        if constexpr (TA) {
          opa.chunk(q, tid, r, p);
          float* d = &smem[buf][0][p * LDS + r];
          d[0] = ra[q].x;
          d[LDS] = ra[q].y;
          d[2 * LDS] = ra[q].z;
          d[3 * LDS] = ra[q].w;
        }
        if constexpr (!TB) {
          opb.chunk(q, tid, r, p);
          float* d = &smem[buf][1][p * LDS + r];
          d[0] = rb[q].x;
          d[LDS] = rb[q].y;
          d[2 * LDS] = rb[q].z;
          d[3 * LDS] = rb[q].w;
        }
      }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    if (klen > 0) {
      issue(0, 0);
      stash(0);
      cp_async_wait_all();
      __syncthreads();
    }
    int buf = 0;
    for (int k0 = 0; k0 < klen; k0 += BK) {
      const bool more = k0 + BK < klen;
      if (more) issue(k0 + BK, buf ^ 1);
      const float* As = smem[buf][0];
      const float* Bs = smem[buf][1];
#pragma unroll
      for (int p = 0; p < BK; ++p) {
        const float4 a0 = *reinterpret_cast<const float4*>(As + p * LDS + tm * 4);
        const float4 a1 = *reinterpret_cast<const float4*>(As + p * LDS + 64 + tm * 4);
        const float4 b0 = *reinterpret_cast<const float4*>(Bs + p * LDS + tn * 8);
        const float4 b1 = *reinterpret_cast<const float4*>(Bs + p * LDS + tn * 8 + 4);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        // two columns per fma.rn.f32x2 (each lane the scalar fma, rounded alike): half
        // the issue slots of the scalar form for the same FMA-pipe work
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const unsigned long long a2 = pack2(av[i], av[i]);
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            unsigned long long c2 = pack2(acc[i][j], acc[i][j + 1]);
            asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c2) : "l"(a2), "l"(pack2(bv[j], bv[j + 1])));
            unpack2(c2, acc[i][j], acc[i][j + 1]);
          }
        }
      }
      if (more) {
        stash(buf ^ 1);
        cp_async_wait_all();
      }
      __syncthreads();
      buf ^= 1;
    }

    float* Cm = static_cast<float*>(g.c) + z * g.stride_c;
    const bool vec_c = STREAM || ((reinterpret_cast<std::uintptr_t>(Cm) & 15) == 0 &&
                                  (g.ldc & 3) == 0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gj = n0 + tn * 8 + j;
      if (!STREAM && gj >= g.n) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gi = m0 + h * 64 + tm * 4;  // m % 4 == 0: the 4 rows are valid together
        if (!STREAM && gi >= g.m) continue;
        const float4 v = make_float4(acc[4 * h][j], acc[4 * h + 1][j], acc[4 * h + 2][j],
                                     acc[4 * h + 3][j]);
        if constexpr (STREAM) {  // the whole 128 x 128 piece (zeros past the edge)
          *reinterpret_cast<float4*>(ws + static_cast<std::int64_t>(blockIdx.x + t) * kSlot +
                                     (tn * 8 + j) * BM + h * 64 + tm * 4) = v;
          continue;
        }
        float* cp = Cm + gi + static_cast<std::int64_t>(gj) * g.ldc;
        float4 prev = make_float4(0.f, 0.f, 0.f, 0.f);
        if (beta != 0.0f) {
          const float4 c = vec_c ? *reinterpret_cast<const float4*>(cp)
                                 : make_float4(cp[0], cp[1], cp[2], cp[3]);
          prev = make_float4(beta * c.x, beta * c.y, beta * c.z, beta * c.w);
        }
        const float4 out = make_float4(fmaf(alpha, v.x, prev.x), fmaf(alpha, v.y, prev.y),
                                       fmaf(alpha, v.z, prev.z), fmaf(alpha, v.w, prev.w));
        if (vec_c) {
          *reinterpret_cast<float4*>(cp) = out;
        } else {
          cp[0] = out.x;
          cp[1] = out.y;
          cp[2] = out.z;
          cp[3] = out.w;
        }
      }
    }
    if constexpr (STREAM) s = seg_end;
  }
}

// C = alpha * (pieces of the tile added in CTA order) + beta * C, 4 rows per thread.
__global__ void __launch_bounds__(kThreads)
    ffma_stream_reduce(const GemmArgs g, const float* __restrict__ ws, const StreamK sk) {
  const float alpha = g.alpha_dev ? *g.alpha_dev : g.alpha;
  const float beta = g.beta_dev ? *g.beta_dev : g.beta;
  float* Cm = static_cast<float*>(g.c);
  const bool vec_c = (reinterpret_cast<std::uintptr_t>(Cm) & 15) == 0 && (g.ldc & 3) == 0;
  const int m4 = g.m / 4;
  const std::int64_t count = static_cast<std::int64_t>(m4) * g.n;
  for (std::int64_t q = static_cast<std::int64_t>(blockIdx.x) * kThreads + threadIdx.x; q < count;
       q += static_cast<std::int64_t>(gridDim.x) * kThreads) {
    const int gi = static_cast<int>(q % m4) * 4, gj = static_cast<int>(q / m4);
    const int t = gi / BM + (gj / BN) * sk.tiles_m;
    const long long t0 = static_cast<long long>(t) * sk.ktiles;
    const int c0 = cta_of(t0, sk), c1 = cta_of(t0 + sk.ktiles - 1, sk);
    const std::int64_t off = (gj % BN) * BM + gi % BM;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = c0; c <= c1; ++c) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(
          ws + static_cast<std::int64_t>(c + t) * kSlot + off));
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    float* cp = Cm + gi + static_cast<std::int64_t>(gj) * g.ldc;
    float4 prev = make_float4(0.f, 0.f, 0.f, 0.f);
    if (beta != 0.0f) {
      const float4 cv = vec_c ? *reinterpret_cast<const float4*>(cp)
                              : make_float4(cp[0], cp[1], cp[2], cp[3]);
      prev = make_float4(beta * cv.x, beta * cv.y, beta * cv.z, beta * cv.w);
    }
    const float4 out = make_float4(fmaf(alpha, sum.x, prev.x), fmaf(alpha, sum.y, prev.y),
                                   fmaf(alpha, sum.z, prev.z), fmaf(alpha, sum.w, prev.w));
    if (vec_c) {
      *reinterpret_cast<float4*>(cp) = out;
    } else {
      cp[0] = out.x;
      cp[1] = out.y;
      cp[2] = out.z;
      cp[3] = out.w;
    }
  }
}

// The aligned-fp32 conditions of these kernels: 16-byte aligned A and B (base, leading
// dimensions and batch strides), m, n, k multiples of 4.
bool usable(const GemmArgs& g) {
  auto al = [](const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15) == 0; };
  return g.type == Elem::kF32 && al(g.a) && al(g.b) && (g.lda & 3) == 0 && (g.ldb & 3) == 0 &&
         (g.batch == 1 || ((g.stride_a & 3) == 0 && (g.stride_b & 3) == 0)) &&
         (g.m & 3) == 0 && (g.n & 3) == 0 && (g.k & 3) == 0;
}

std::int64_t tile_count(const GemmArgs& g) {
  return static_cast<std::int64_t>((g.m + BM - 1) / BM) * ((g.n + BN - 1) / BN);
}

// Stream-K plan for a batch-1 problem with fewer 128 x 128 tiles than SMs: two CTAs per
// SM, each with at least 4 k steps (ctas 0: not used).
StreamK stream_plan(const GemmArgs& g) {
  StreamK sk{};
  const int sms = sm_count(current_device());
  const std::int64_t sm = sms > 0 ? sms : 148;
  const std::int64_t tiles = tile_count(g);
  if (!usable(g) || g.batch != 1 || g.k <= 0 || tiles >= sm) return sk;
  sk.tiles_m = (g.m + BM - 1) / BM;
  sk.ktiles = (g.k + BK - 1) / BK;
  sk.total = tiles * sk.ktiles;
  std::int64_t ctas = std::min<std::int64_t>(2 * sm, sk.total / 4);
  if (ctas <= tiles) return StreamK{};  // one CTA per tile is as good
  sk.ctas = static_cast<int>(ctas);
  return sk;
}

std::size_t stream_workspace(const StreamK& sk, const GemmArgs& g) {
  return sk.ctas == 0 ? 0
                      : static_cast<std::size_t>(sk.ctas + tile_count(g) - 1) * kSlot *
                            sizeof(float);
}

cudaError_t launch_whole(const GemmArgs& g, cudaStream_t st) {
  const dim3 grid((g.m + BM - 1) / BM, (g.n + BN - 1) / BN,
                  static_cast<unsigned>(g.batch < 65535 ? g.batch : 65535));
  const StreamK none{};
  if (!g.trans_a && !g.trans_b)
    gemm_ffma_vec<false, false, false><<<grid, kThreads, 0, st>>>(g, nullptr, none);
  else if (g.trans_a && !g.trans_b)
    gemm_ffma_vec<true, false, false><<<grid, kThreads, 0, st>>>(g, nullptr, none);
  else if (!g.trans_a && g.trans_b)
    gemm_ffma_vec<false, true, false><<<grid, kThreads, 0, st>>>(g, nullptr, none);
  else
    gemm_ffma_vec<true, true, false><<<grid, kThreads, 0, st>>>(g, nullptr, none);
  return cudaGetLastError();
}

cudaError_t launch_stream(const GemmArgs& g, const StreamK& sk, float* ws, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>(sk.ctas));
  if (!g.trans_a && !g.trans_b)
    gemm_ffma_vec<false, false, true><<<grid, kThreads, 0, st>>>(g, ws, sk);
  else if (g.trans_a && !g.trans_b)
    gemm_ffma_vec<true, false, true><<<grid, kThreads, 0, st>>>(g, ws, sk);
  else if (!g.trans_a && g.trans_b)
    gemm_ffma_vec<false, true, true><<<grid, kThreads, 0, st>>>(g, ws, sk);
  else
    gemm_ffma_vec<true, true, true><<<grid, kThreads, 0, st>>>(g, ws, sk);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int sms = sm_count(current_device());
  const std::int64_t count = static_cast<std::int64_t>(g.m / 4) * g.n;
  std::int64_t blocks = (count + kThreads - 1) / kThreads;
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  ffma_stream_reduce<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(g, ws, sk);
  return cudaGetLastError();
}

}  // namespace vec

// Splits of K for a batch-1 problem whose 128 x 128 tiles cannot fill the GPU twice
// (0: no split): enough splits for two CTAs per SM, each at least 256 deep.
int simt_splits(const GemmArgs& g) {
  if (g.batch != 1 || g.k < 512) return 0;
  const int sms = sm_count(current_device());
  const std::int64_t target = 2 * static_cast<std::int64_t>(sms > 0 ? sms : 148);
  const std::int64_t tiles = static_cast<std::int64_t>((g.m + 127) / 128) * ((g.n + 127) / 128);
  if (tiles >= target / 2) return 0;
  std::int64_t s = (target + tiles - 1) / tiles;
  const std::int64_t by_k = g.k / 256;
  if (s > by_k) s = by_k;
  if (s > 16) s = 16;
  return s >= 2 ? static_cast<int>(s) : 0;
}

template <typename T, bool TA, bool TB>
void launch_split_kernel(const GemmArgs& g, const SplitK& sk, int splits, cudaStream_t st) {
  const dim3 grid((g.m + 127) / 128, (g.n + 127) / 128, static_cast<unsigned>(splits));
  gemm_simt<T, 128, 128, 8, 8, 8, TA, TB, true><<<grid, kThreads, 0, st>>>(g, sk);
}

template <typename T>
cudaError_t launch_split(const GemmArgs& g, float* ws, int splits, cudaStream_t st) {
  SplitK sk{ws, ((g.k + splits - 1) / splits + 15) / 16 * 16};
  splits = (g.k + sk.kchunk - 1) / sk.kchunk;
  if (!g.trans_a && !g.trans_b)
    launch_split_kernel<T, false, false>(g, sk, splits, st);
  else if (g.trans_a && !g.trans_b)
    launch_split_kernel<T, true, false>(g, sk, splits, st);
  else if (!g.trans_a && g.trans_b)
    launch_split_kernel<T, false, true>(g, sk, splits, st);
  else
    launch_split_kernel<T, true, true>(g, sk, splits, st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int sms = sm_count(current_device());
  const std::int64_t mn = static_cast<std::int64_t>(g.m) * g.n;
  std::int64_t grid = (mn + kThreads - 1) / kThreads;
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 8;
  if (grid > cap) grid = cap;
  simt_split_reduce<T><<<static_cast<unsigned>(grid), kThreads, 0, st>>>(g, ws, splits);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_typed(const GemmArgs& g, cudaStream_t st) {
  const int sms = sm_count(current_device());
  const std::int64_t target = sms > 0 ? sms : 148;
  auto tiles = [&](int bm, int bn) {
    return static_cast<std::int64_t>((g.m + bm - 1) / bm) * ((g.n + bn - 1) / bn) * g.batch;
  };
  if (std::is_same_v<T, float> && vec::usable(g) && tiles(128, 128) >= target)
    return vec::launch_whole(g, st);
  if (tiles(128, 128) >= target) return launch_tile<T, 128, 128, 8, 8>(g, st);
  if (tiles(128, 64) >= (target * 3) / 4) return launch_tile<T, 128, 64, 8, 4>(g, st);
  return launch_tile<T, 64, 64, 4, 4>(g, st);
}

}  // namespace

std::size_t gemm_simt_workspace(const GemmArgs& g) noexcept {
  const vec::StreamK sk = vec::stream_plan(g);
  if (sk.ctas > 0) return vec::stream_workspace(sk, g);
  const int s = simt_splits(g);
  return s == 0 ? 0 : static_cast<std::size_t>(s) * g.m * g.n * sizeof(float);
}

cudaError_t launch_gemm_simt_split(const GemmArgs& g, void* workspace, std::size_t ws_bytes,
                                   cudaStream_t stream) noexcept {
  const vec::StreamK sk = vec::stream_plan(g);
  if (sk.ctas > 0) {
    if (workspace == nullptr || ws_bytes < vec::stream_workspace(sk, g))
      return launch_gemm_simt(g, stream);
    return vec::launch_stream(g, sk, static_cast<float*>(workspace), stream);
  }
  const int s = simt_splits(g);
  if (s == 0 || workspace == nullptr || ws_bytes < gemm_simt_workspace(g))
    return launch_gemm_simt(g, stream);
  float* ws = static_cast<float*>(workspace);
  switch (g.type) {
    case Elem::kF32:
      return launch_split<float>(g, ws, s, stream);
    case Elem::kF16:
      return launch_split<__half>(g, ws, s, stream);
    case Elem::kBF16:
      return launch_split<__nv_bfloat16>(g, ws, s, stream);
  }
  return cudaErrorInvalidValue;
}

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
