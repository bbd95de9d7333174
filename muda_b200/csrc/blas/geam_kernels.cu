// geam_kernels.cu — cuBLAS geam, C = alpha * op(A) + beta * op(B) (HBM-bound).
//
// Per-element arithmetic follows the reference.  Sgeam (libraries/blas/shaders/
// cublas_kernels.metal:1047-1076): each term is rounded on its own, a zero
// scalar's term is +0 and its operand is not read, then C = term_a + term_b.
// Dgeam (libraries/blas/src/cublas_level3.mm:906-927, a host loop there):
// val = 0; val += alpha * a when alpha != 0; val += beta * b when beta != 0.
// Both are evaluated here with explicit round-to-nearest multiplies and adds, so
// nothing is contracted into an fma and the results are bit-identical to the CPU
// restatement built with -ffp-contract=off.
//
// B200 layout: the m x n output is cut into 64 x 64 tiles (32 x 64 for fp64), walked grid-stride by
// one wave of CTAs (256 threads each, as many per SM as fit).  A warp writes 64
// consecutive rows of one column of C (two 128-byte lines for fp32, adjacent in
// DRAM).  An untransposed operand is read the same way, into registers.  A
// transposed operand is read along its own columns (rows of op(X)), 64 elements
// at a time, into a 64 x 65 (fp64: 32 x 65) shared tile and read back across it, so both its
// global reads and the writes of C stay coalesced.  All of a tile's loads (up to 32
// per thread) are issued before its one barrier, so the tile waits on memory once.
#include "blas/geam.hpp"

#include <cuda_runtime.h>

#include "common/device.hpp"

namespace mb200::blas {
namespace {

constexpr int kLanes = 32;
constexpr int kCols = 64;         // columns of C per tile
constexpr int kRowsPerPass = 8;   // blockDim.y
constexpr int kColSteps = kCols / kRowsPerPass;
// Rows of C per tile: 256 bytes of a column (64 fp32, 32 fp64), one or two per lane.
template <typename T>
constexpr int kTile = 256 / static_cast<int>(sizeof(T));
template <typename T>
constexpr int kRowReps = kTile<T> / kLanes;

template <typename T>
struct GeamArgs {
  const T* A;
  const T* B;
  T* C;
  const T* alpha_dev;
  const T* beta_dev;
  long long lda, ldb, ldc;
  int m, n;
  int tiles_m;
  long long tiles;
  T alpha, beta;
};

__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }

// Sgeam: term_a + term_b, each term +0 when its scalar is zero.
__device__ __forceinline__ float combine(bool use_a, float ta, bool use_b, float tb) {
  return add_rn(use_a ? ta : 0.0f, use_b ? tb : 0.0f);
}
// Dgeam: 0 + term_a (when used) + term_b (when used), in that order.
__device__ __forceinline__ double combine(bool use_a, double ta, bool use_b, double tb) {
  double v = 0.0;
  if (use_a) v = add_rn(v, ta);
  if (use_b) v = add_rn(v, tb);
  return v;
}

// One operand's values for the thread's kRowReps x kColSteps outputs of a tile
// (rows r0 + lane + 32i, columns c0 + ty + 8k).  Transposed: rows [r0, r0+kTile) x
// cols [c0, c0+64) of op(X) = X^T go through s[row][col] first; X[c + r * ldx] is
// op(X)[r][c], so the loads walk c (contiguous in X).  Untransposed: read straight
// into registers.  Every global load of the tile is issued before the caller's
// barrier.
template <typename T, bool TRANS>
__device__ __forceinline__ void load_operand(T (*s)[kCols + 1], T (&v)[kRowReps<T>][kColSteps],
                                             const T* X, long long ldx, int m, int n, int r0,
                                             int c0) {
  if constexpr (TRANS) {
#pragma unroll
    for (int k = 0; k < kTile<T> / kRowsPerPass; ++k) {
      const int rr = threadIdx.y + k * kRowsPerPass;
      const int r = r0 + rr;
#pragma unroll
      for (int j = 0; j < kCols / kLanes; ++j) {
        const int c = c0 + threadIdx.x + j * kLanes;
        if (r < m && c < n)
          s[rr][threadIdx.x + j * kLanes] = X[c + static_cast<long long>(r) * ldx];
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < kColSteps; ++k) {
      const int c = c0 + threadIdx.y + k * kRowsPerPass;
#pragma unroll
      for (int i = 0; i < kRowReps<T>; ++i) {
        const int r = r0 + threadIdx.x + i * kLanes;
        v[i][k] = (r < m && c < n) ? X[r + static_cast<long long>(c) * ldx] : T(0);
      }
    }
  }
}

template <typename T, bool TRANS>
__device__ __forceinline__ T operand_at(T (*s)[kCols + 1], const T (&v)[kRowReps<T>][kColSteps],
                                        int i, int k) {
  if constexpr (TRANS) return s[threadIdx.x + i * kLanes][threadIdx.y + k * kRowsPerPass];
  else return v[i][k];
}

template <typename T, bool TA, bool TB>
// Without a transposed operand the 2 x 8 values of A and of B a thread holds in flight
// need more than 64 registers (4 CTAs per SM spilled them, 3 still did): 2 CTAs per SM there.
__global__ void __launch_bounds__(kLanes* kRowsPerPass, (TA || TB) ? 4 : 2)
    geam_kernel(GeamArgs<T> g) {
  __shared__ T sa[TA ? kTile<T> : 1][kCols + 1];
  __shared__ T sb[TB ? kTile<T> : 1][kCols + 1];
  const T alpha = g.alpha_dev ? *g.alpha_dev : g.alpha;
  const T beta = g.beta_dev ? *g.beta_dev : g.beta;
  const bool use_a = alpha != T(0);
  const bool use_b = beta != T(0);
  for (long long t = blockIdx.x; t < g.tiles; t += gridDim.x) {
    const int r0 = static_cast<int>(t % g.tiles_m) * kTile<T>;
    const int c0 = static_cast<int>(t / g.tiles_m) * kCols;
    T va[kRowReps<T>][kColSteps], vb[kRowReps<T>][kColSteps];
    if (use_a) load_operand<T, TA>(sa, va, g.A, g.lda, g.m, g.n, r0, c0);
    if (use_b) load_operand<T, TB>(sb, vb, g.B, g.ldb, g.m, g.n, r0, c0);
    if constexpr (TA || TB) __syncthreads();
#pragma unroll
    for (int k = 0; k < kColSteps; ++k) {
      const int c = c0 + threadIdx.y + k * kRowsPerPass;
#pragma unroll
      for (int i = 0; i < kRowReps<T>; ++i) {
        const int r = r0 + threadIdx.x + i * kLanes;
        if (r < g.m && c < g.n) {
          const T ta = use_a ? mul_rn(alpha, operand_at<T, TA>(sa, va, i, k)) : T(0);
          const T tb = use_b ? mul_rn(beta, operand_at<T, TB>(sb, vb, i, k)) : T(0);
          g.C[r + static_cast<long long>(c) * g.ldc] = combine(use_a, ta, use_b, tb);
        }
      }
    }
    if constexpr (TA || TB) __syncthreads();  // the next tile overwrites the staging tiles
  }
}

// Exactly one transposed operand: its staging tile is double-buffered and filled by
// cp.async one tile ahead (element copies, skipped outside the matrix), so the copy of
// tile t + 1 is in flight while tile t is combined and stored; the untransposed
// operand is read into registers as in geam_kernel.
template <typename T>
__device__ __forceinline__ void cp_async_elem(T* dst, const T* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(static_cast<unsigned>(
                   __cvta_generic_to_shared(dst))),
               "l"(src), "n"(static_cast<int>(sizeof(T)))
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Rows [r0, r0 + kTile) x cols [c0, c0 + 64) of op(X) = X^T into s (X[c + r * ldx] is
// op(X)[r][c]; the copies walk c, contiguous in X), as one cp.async group.
template <typename T>
__device__ __forceinline__ void copy_transposed(T (*s)[kCols + 1], const T* X, long long ldx,
                                                int m, int n, int r0, int c0) {
#pragma unroll
  for (int k = 0; k < kTile<T> / kRowsPerPass; ++k) {
    const int rr = threadIdx.y + k * kRowsPerPass;
    const int r = r0 + rr;
#pragma unroll
    for (int j = 0; j < kCols / kLanes; ++j) {
      const int c = c0 + threadIdx.x + j * kLanes;
      if (r < m && c < n)
        cp_async_elem(&s[rr][threadIdx.x + j * kLanes], X + c + static_cast<long long>(r) * ldx);
    }
  }
  cp_async_commit();
}

template <typename T, bool TA>
__global__ void __launch_bounds__(kLanes* kRowsPerPass, 4) geam_kernel_db(GeamArgs<T> g) {
  __shared__ T st[2][kTile<T>][kCols + 1];
  const T alpha = g.alpha_dev ? *g.alpha_dev : g.alpha;
  const T beta = g.beta_dev ? *g.beta_dev : g.beta;
  const bool use_a = alpha != T(0);
  const bool use_b = beta != T(0);
  const bool use_t = TA ? use_a : use_b;  // the transposed operand is read
  const bool use_n = TA ? use_b : use_a;
  const T* xt = TA ? g.A : g.B;
  const T* xn = TA ? g.B : g.A;
  const long long ldt = TA ? g.lda : g.ldb;
  const long long ldn = TA ? g.ldb : g.lda;
  auto corner = [&](long long t, int& r0, int& c0) {
    r0 = static_cast<int>(t % g.tiles_m) * kTile<T>;
    c0 = static_cast<int>(t / g.tiles_m) * kCols;
  };
  int r0, c0;
  corner(blockIdx.x, r0, c0);
  if (use_t && blockIdx.x < g.tiles) {
    copy_transposed(st[0], xt, ldt, g.m, g.n, r0, c0);
  } else {
    cp_async_commit();
  }
  int buf = 0;
  for (long long t = blockIdx.x; t < g.tiles; t += gridDim.x, buf ^= 1) {
    corner(t, r0, c0);
    const long long tn = t + gridDim.x;
    if (use_t && tn < g.tiles) {
      int rn, cn;
      corner(tn, rn, cn);
      copy_transposed(st[buf ^ 1], xt, ldt, g.m, g.n, rn, cn);
    } else {
      cp_async_commit();  // an empty group keeps the wait counts aligned
    }
    T vn[kRowReps<T>][kColSteps];
    if (use_n) load_operand<T, false>(nullptr, vn, xn, ldn, g.m, g.n, r0, c0);
    cp_async_wait<1>();  // this thread's copies of tile t have landed
    __syncthreads();     // and everyone's
#pragma unroll
    for (int k = 0; k < kColSteps; ++k) {
      const int c = c0 + threadIdx.y + k * kRowsPerPass;
#pragma unroll
      for (int i = 0; i < kRowReps<T>; ++i) {
        const int r = r0 + threadIdx.x + i * kLanes;
        if (r < g.m && c < g.n) {
          const T xtv = st[buf][threadIdx.x + i * kLanes][threadIdx.y + k * kRowsPerPass];
          const T xa = TA ? xtv : vn[i][k];
          const T xb = TA ? vn[i][k] : xtv;
          const T ta = use_a ? mul_rn(alpha, xa) : T(0);
          const T tb = use_b ? mul_rn(beta, xb) : T(0);
          g.C[r + static_cast<long long>(c) * g.ldc] = combine(use_a, ta, use_b, tb);
        }
      }
    }
    __syncthreads();  // st[buf] is refilled by the next iteration's copy
  }
  cp_async_wait<0>();
}

// Neither operand transposed, every column 16-byte aligned (pointers aligned, m and the
// leading dimensions multiples of 16 / sizeof(T)): a CTA takes whole columns and its
// threads stream them in 16-byte vectors, four vectors of each operand in flight per
// thread, the arithmetic per element as in geam_kernel.
template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  using V = float4;
  static constexpr int kN = 4;
};
template <>
struct Vec16<double> {
  using V = double2;
  static constexpr int kN = 2;
};

template <typename T>
__device__ __forceinline__ T lane_of(const typename Vec16<T>::V& v, int e) {
  if constexpr (Vec16<T>::kN == 4) {
    return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
  } else {
    return e == 0 ? v.x : v.y;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) geam_nn_vec(GeamArgs<T> g) {
  using VT = typename Vec16<T>::V;
  constexpr int kN = Vec16<T>::kN;
  constexpr int kU = 4;
  const T alpha = g.alpha_dev ? *g.alpha_dev : g.alpha;
  const T beta = g.beta_dev ? *g.beta_dev : g.beta;
  const bool use_a = alpha != T(0);
  const bool use_b = beta != T(0);
  const int mv = g.m / kN;  // vectors per column
  for (long long c = blockIdx.x; c < g.n; c += gridDim.x) {
    const VT* a = reinterpret_cast<const VT*>(g.A + c * g.lda);
    const VT* b = reinterpret_cast<const VT*>(g.B + c * g.ldb);
    VT* out = reinterpret_cast<VT*>(g.C + c * g.ldc);
    for (int v0 = threadIdx.x; v0 < mv; v0 += kU * blockDim.x) {
      VT va[kU], vb[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int v = v0 + u * blockDim.x;
        if (v < mv) {
          if (use_a) va[u] = __ldcs(a + v);
          if (use_b) vb[u] = __ldcs(b + v);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int v = v0 + u * blockDim.x;
        if (v < mv) {
          T r[kN];
#pragma unroll
          for (int e = 0; e < kN; ++e) {
            const T ta = use_a ? mul_rn(alpha, lane_of<T>(va[u], e)) : T(0);
            const T tb = use_b ? mul_rn(beta, lane_of<T>(vb[u], e)) : T(0);
            r[e] = combine(use_a, ta, use_b, tb);
          }
          VT o;
          if constexpr (kN == 4) {
            o = make_float4(r[0], r[1], r[2], r[3]);
          } else {
            o = make_double2(r[0], r[1]);
          }
          __stcs(out + v, o);
        }
      }
    }
  }
}

// One wave: as many CTAs as the SMs hold at this instance's occupancy (its register
// and shared-memory use differ by type and transposition), so that no CTA of the
// grid-stride loop waits for a second wave.
template <typename T, bool TA, bool TB>
cudaError_t launch(const GeamArgs<T>& g, cudaStream_t stream) {
  constexpr bool kDb = TA != TB;
  auto kern = [] {
    if constexpr (kDb) return geam_kernel_db<T, TA>;
    else return geam_kernel<T, TA, TB>;
  }();
  static const int per_sm = [&] {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, kLanes * kRowsPerPass, 0) !=
        cudaSuccess)
      b = 0;
    return b > 0 ? b : 1;
  }();
  const long long wave = static_cast<long long>(sm_count(current_device())) * per_sm;
  const unsigned grid = static_cast<unsigned>(g.tiles < wave ? g.tiles : wave);
  kern<<<grid, dim3(kLanes, kRowsPerPass), 0, stream>>>(g);
  return cudaGetLastError();
}

}  // namespace

template <typename T>
cudaError_t launch_geam(bool trans_a, bool trans_b, int m, int n, T alpha, const T* alpha_dev,
                        const T* A, int lda, T beta, const T* beta_dev, const T* B, int ldb,
                        T* C, int ldc, cudaStream_t stream) noexcept {
  if (m <= 0 || n <= 0) return cudaSuccess;
  GeamArgs<T> g{};
  g.A = A;
  g.B = B;
  g.C = C;
  g.alpha_dev = alpha_dev;
  g.beta_dev = beta_dev;
  g.lda = lda;
  g.ldb = ldb;
  g.ldc = ldc;
  g.m = m;
  g.n = n;
  g.tiles_m = (m + kTile<T> - 1) / kTile<T>;
  g.tiles = static_cast<long long>(g.tiles_m) * ((n + kCols - 1) / kCols);
  g.alpha = alpha;
  g.beta = beta;
  constexpr int kVec = 16 / static_cast<int>(sizeof(T));
  if (!trans_a && !trans_b && m % kVec == 0 && lda % kVec == 0 && ldb % kVec == 0 &&
      ldc % kVec == 0 && aligned_to(A, 16) && aligned_to(B, 16) && aligned_to(C, 16)) {
    // a null operand is never read (its scalar is zero), so its alignment does not matter
    const long long wave = static_cast<long long>(sm_count(current_device())) * 8;
    const unsigned grid = static_cast<unsigned>(n < wave ? n : wave);
    geam_nn_vec<T><<<grid, 256, 0, stream>>>(g);
    return cudaGetLastError();
  }
  if (trans_a)
    return trans_b ? launch<T, true, true>(g, stream) : launch<T, true, false>(g, stream);
  return trans_b ? launch<T, false, true>(g, stream) : launch<T, false, false>(g, stream);
}

template cudaError_t launch_geam<float>(bool, bool, int, int, float, const float*, const float*,
                                        int, float, const float*, const float*, int, float*,
                                        int, cudaStream_t) noexcept;
template cudaError_t launch_geam<double>(bool, bool, int, int, double, const double*,
                                         const double*, int, double, const double*,
                                         const double*, int, double*, int,
                                         cudaStream_t) noexcept;

}  // namespace mb200::blas
