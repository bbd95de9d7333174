// dblas_kernels.cu — cuBLAS double-precision kernels (sm_100a).
//
// The reference runs cublasD* on the host through the platform CBLAS
// (libraries/blas/src/cublas_level1.mm:658-979, cublas_level2.mm:135-200,
// cublas_level3.mm:714-819); the results here follow the reference-BLAS
// definitions those calls implement:
//   daxpy  y(i) = y(i) + alpha*x(i), the product and the sum rounded separately;
//   dscal  x(i) = alpha*x(i);  dcopy, dswap elementwise;
//   ddot / dasum / dnrm2 sums over i (any order; nrm2 with Blue's scaling so that
//          no square overflows or underflows);  idamax the first largest |x(i)|;
//   dgemv  y = alpha*op(A)*x + beta*y;  dgemm C = alpha*op(A)*op(B) + beta*C, with
//          beta == 0 not reading y / C and alpha == 0 not reading A, B, x.
// A stride of 0 in y (or in either vector of dswap) means every element updates the
// same location one after another; those calls run on one thread in element order,
// as the sequential reference loop does.
//
// B200 layout: elementwise and reduction kernels are grid-stride over a whole number
// of waves with 16-byte (double2) accesses on unit-stride aligned vectors;
// reductions are one launch whose last CTA adds the per-CTA partials in CTA order
// (deterministic).  dgemv gives every thread one row (op N, columns streamed in
// order) or every warp one column (op T), splitting the inner dimension into chunks
// when the outer one cannot fill the GPU.  dgemm runs on the fp64 tensor-core MMA
// (mma.m8n8k4 .f64): a CTA owns a 128 x 64 tile (64 x 64 for problems with fewer
// tiles than twice the SM count), each warp 32 x 32, k in stages staged through a
// cp.async ring in shared memory.
#include "blas/dblas.hpp"

#include <cuda_runtime.h>

#include <cstdint>

#include "common/device.hpp"

namespace mb200::blas {
namespace {

constexpr int kThreads = 256;
constexpr int kCtasPerSm = 8;
constexpr int kMaxPartials = 1024;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ long long vidx(long long i, int n, int inc) {
  return inc >= 0 ? i * inc : (i - n + 1) * static_cast<long long>(inc);
}

unsigned grid_for(long long work) {
  const int sms = sm_count(current_device());
  const long long cap = static_cast<long long>(sms > 0 ? sms : 148) * kCtasPerSm;
  const long long want = (work + kThreads - 1) / kThreads;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

// ------------------------------------------------------------------ elementwise

enum class Elt : int { kAxpy, kCopy, kScal, kSwap };

template <Elt E>
__device__ __forceinline__ void apply(double a, double* x, double* y, long long ix, long long iy) {
  if constexpr (E == Elt::kAxpy) {
    y[iy] = __dadd_rn(y[iy], __dmul_rn(a, x[ix]));
  } else if constexpr (E == Elt::kCopy) {
    y[iy] = x[ix];
  } else if constexpr (E == Elt::kScal) {
    x[ix] = __dmul_rn(a, x[ix]);
  } else {
    const double t = x[ix];
    x[ix] = y[iy];
    y[iy] = t;
  }
}

template <Elt E>
__device__ __forceinline__ void apply2(double a, double2* x, double2* y, long long i) {
  if constexpr (E == Elt::kAxpy) {
    const double2 u = x[i];
    double2 v = y[i];
    v.x = __dadd_rn(v.x, __dmul_rn(a, u.x));
    v.y = __dadd_rn(v.y, __dmul_rn(a, u.y));
    y[i] = v;
  } else if constexpr (E == Elt::kCopy) {
    y[i] = x[i];
  } else if constexpr (E == Elt::kScal) {
    double2 v = x[i];
    v.x = __dmul_rn(a, v.x);
    v.y = __dmul_rn(a, v.y);
    x[i] = v;
  } else {
    const double2 t = x[i];
    x[i] = y[i];
    y[i] = t;
  }
}

// Vec: unit strides and 16-byte aligned vectors: n / 2 double2 plus a scalar tail.
// Seq: one thread walks the elements in order (a zero stride on a written vector).
template <Elt E, bool Vec, bool Seq>
__global__ void __launch_bounds__(kThreads)
    elementwise(int n, double alpha, const double* alpha_dev, double* x, int incx, double* y,
                int incy) {
  const double a = alpha_dev ? *alpha_dev : alpha;
  if (E == Elt::kAxpy && a == 0.0) return;
  if constexpr (Seq) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    for (long long i = 0; i < n; ++i) apply<E>(a, x, y, vidx(i, n, incx), vidx(i, n, incy));
    return;
  }
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if constexpr (Vec) {
    const long long n2 = n / 2;
    for (long long i = t0; i < n2; i += stride)
      apply2<E>(a, reinterpret_cast<double2*>(x), reinterpret_cast<double2*>(y), i);
    if ((n & 1) != 0 && t0 == 0) apply<E>(a, x, y, n - 1, n - 1);
  } else {
    for (long long i = t0; i < n; i += stride) apply<E>(a, x, y, vidx(i, n, incx), vidx(i, n, incy));
  }
}

template <Elt E>
cudaError_t launch_elt(int n, double alpha, const double* alpha_dev, const double* x, int incx,
                       double* y, int incy, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  double* xm = const_cast<double*>(x);
  const bool seq = n > 1 && ((E != Elt::kScal && incy == 0) || (E == Elt::kSwap && incx == 0));
  const bool unit = incx == 1 && (E == Elt::kScal || incy == 1);
  const bool vec = unit && aligned_to(x, 16) && (E == Elt::kScal || aligned_to(y, 16));
  if (seq)
    elementwise<E, false, true><<<1, 32, 0, stream>>>(n, alpha, alpha_dev, xm, incx, y, incy);
  else if (vec)
    elementwise<E, true, false><<<grid_for((n + 1) / 2), kThreads, 0, stream>>>(
        n, alpha, alpha_dev, xm, incx, y, incy);
  else
    elementwise<E, false, false><<<grid_for(n), kThreads, 0, stream>>>(n, alpha, alpha_dev, xm,
                                                                       incx, y, incy);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ reductions

// Blue's scaled sums of squares (the reference-BLAS dnrm2): values above kTbig are
// summed scaled by kSbig, values below kTsml scaled by kSsml, the rest as they are.
constexpr double kTsml = 0x1p-511;
constexpr double kTbig = 0x1p+486;
constexpr double kSsml = 0x1p+537;
constexpr double kSbig = 0x1p-538;

struct Acc {
  double a, b, c;  // dot / asum: a; nrm2: small, medium, big sums; amax: a = |x|, b = index
};

struct Scratch {
  unsigned counter;  // CTAs finished; the last one resets it to 0 (same word as level12's)
  unsigned pad[7];
  Acc partial[kMaxPartials];
};

template <Reduce R>
__device__ __forceinline__ Acc zero_acc() {
  if constexpr (R == Reduce::kAmax) return Acc{-1.0, 0.0, 0.0};
  return Acc{0.0, 0.0, 0.0};
}

template <Reduce R>
__device__ __forceinline__ void add_elem(Acc& s, double u, double v, long long i) {
  if constexpr (R == Reduce::kDot) {
    s.a = fma(u, v, s.a);
  } else if constexpr (R == Reduce::kAsum) {
    s.a += fabs(u);
  } else if constexpr (R == Reduce::kNrm2) {
    const double ax = fabs(u);
    if (ax > kTbig) {
      const double t = ax * kSbig;
      s.c = fma(t, t, s.c);
    } else if (ax < kTsml) {
      const double t = ax * kSsml;
      s.a = fma(t, t, s.a);
    } else {
      s.b = fma(ax, ax, s.b);  // NaN lands here and propagates
    }
  } else {
    const double ax = fabs(u);
    if (ax > s.a) {  // ascending i within a thread: strict > keeps the first; NaN never wins
      s.a = ax;
      s.b = static_cast<double>(i + 1);
    }
  }
}

template <Reduce R>
__device__ __forceinline__ Acc combine(Acc p, Acc q) {
  if constexpr (R == Reduce::kAmax) {
    if (q.b == 0.0) return p;
    if (p.b == 0.0) return q;
    if (q.a > p.a || (q.a == p.a && q.b < p.b)) return q;
    return p;
  } else {
    return Acc{p.a + q.a, p.b + q.b, p.c + q.c};
  }
}

template <Reduce R>
__device__ __forceinline__ Acc warp_combine(Acc s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Acc t{__shfl_xor_sync(kFull, s.a, o), __shfl_xor_sync(kFull, s.b, o),
          __shfl_xor_sync(kFull, s.c, o)};
    // fixed pairing order: the lower lane's value first
    s = (threadIdx.x & o) ? combine<R>(t, s) : combine<R>(s, t);
  }
  return s;
}

// Block-wide combine in warp order; the result is valid in thread 0.
template <Reduce R>
__device__ __forceinline__ Acc block_combine(Acc mine, Acc* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  Acc s = warp_combine<R>(mine);
  if (lane == 0) sh[warp] = s;
  __syncthreads();
  if (warp == 0) {
    s = lane < kThreads / 32 ? sh[lane] : zero_acc<R>();
    s = warp_combine<R>(s);
  }
  __syncthreads();
  return s;
}

// The reference-BLAS dnrm2 finish of Blue's three sums.
__device__ __forceinline__ double nrm2_finish(double asml, double amed, double abig) {
  if (abig > 0.0) {
    if (amed > 0.0 || isnan(amed)) abig += (amed * kSbig) * kSbig;
    return sqrt(abig) / kSbig;
  }
  if (asml > 0.0) {
    if (amed > 0.0 || isnan(amed)) {
      const double m = sqrt(amed), s = sqrt(asml) / kSsml;
      const double ymin = s > m ? m : s, ymax = s > m ? s : m;
      const double r = ymin / ymax;
      return sqrt(ymax * ymax * (1.0 + r * r));
    }
    return sqrt(asml) / kSsml;
  }
  return sqrt(amed);
}

template <Reduce R, bool Vec>
__global__ void __launch_bounds__(kThreads)
    dreduce_kernel(int n, const double* __restrict__ x, int incx, const double* __restrict__ y,
                   int incy, void* out, Scratch* scratch) {
  __shared__ Acc sh[kThreads / 32];
  __shared__ int last;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  Acc s = zero_acc<R>();
  if constexpr (Vec) {
    const long long n2 = n / 2;
    const double2* x2 = reinterpret_cast<const double2*>(x);
    const double2* y2 = reinterpret_cast<const double2*>(y);
    for (long long i = t0; i < n2; i += stride) {
      const double2 u = __ldcs(x2 + i);
      double2 v = make_double2(0.0, 0.0);
      if constexpr (R == Reduce::kDot) v = __ldcs(y2 + i);
      add_elem<R>(s, u.x, v.x, 2 * i);
      add_elem<R>(s, u.y, v.y, 2 * i + 1);
    }
    if ((n & 1) != 0 && t0 == 0)
      add_elem<R>(s, x[n - 1], R == Reduce::kDot ? y[n - 1] : 0.0, n - 1);
  } else {
    for (long long i = t0; i < n; i += stride)
      add_elem<R>(s, x[vidx(i, n, incx)], R == Reduce::kDot ? y[vidx(i, n, incy)] : 0.0, i);
  }
  Acc part = block_combine<R>(s, sh);
  if (threadIdx.x == 0) {
    scratch->partial[blockIdx.x] = part;
    __threadfence();
    last = atomicAdd(&scratch->counter, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // the last CTA: thread t adds partials t, t + 256, ... in order, then the block combines
  Acc m = zero_acc<R>();
  for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
    const volatile Acc* p = &scratch->partial[b];
    m = combine<R>(m, Acc{p->a, p->b, p->c});
  }
  part = block_combine<R>(m, sh);
  if (threadIdx.x == 0) {
    if constexpr (R == Reduce::kAmax) {
      // the reference idamax starts from the first element's magnitude: a NaN there
      // is never exceeded
      *static_cast<int*>(out) = isnan(x[0]) ? 1 : static_cast<int>(part.b);
    } else if constexpr (R == Reduce::kNrm2) {
      *static_cast<double*>(out) = nrm2_finish(part.a, part.b, part.c);
    } else {
      *static_cast<double*>(out) = part.a;
    }
    scratch->counter = 0u;
  }
}

template <Reduce R>
cudaError_t launch_r(int n, const double* x, int incx, const double* y, int incy, void* out,
                     Scratch* scratch, cudaStream_t stream) {
  const bool vec = incx == 1 && aligned_to(x, 16) &&
                   (R != Reduce::kDot || (incy == 1 && aligned_to(y, 16)));
  const long long per_thread = 8;
  long long g = (static_cast<long long>(n) + kThreads * per_thread - 1) / (kThreads * per_thread);
  const int sms = sm_count(current_device());
  const long long cap = static_cast<long long>(sms > 0 ? sms : 148) * 4;
  if (g > cap) g = cap;
  if (g > kMaxPartials) g = kMaxPartials;
  if (g < 1) g = 1;
  if (vec)
    dreduce_kernel<R, true><<<static_cast<unsigned>(g), kThreads, 0, stream>>>(n, x, incx, y,
                                                                               incy, out, scratch);
  else
    dreduce_kernel<R, false><<<static_cast<unsigned>(g), kThreads, 0, stream>>>(n, x, incx, y,
                                                                                incy, out, scratch);
  return cudaGetLastError();
}

__global__ void dreduce_empty(void* out, int is_index) {
  if (is_index)
    *static_cast<int*>(out) = 0;
  else
    *static_cast<double*>(out) = 0.0;
}

// ------------------------------------------------------------------ gemv

__device__ __forceinline__ double scalar_of(double host, const double* dev) {
  return dev ? *dev : host;
}

// y(i) = alpha*sum + beta*y(i) (beta == 0: y not read).
__device__ __forceinline__ void gemv_write(double* yp, double al, double sum, double be) {
  const double prev = be == 0.0 ? 0.0 : be * *yp;
  *yp = fma(al, sum, prev);
}

// op(A) = A: thread per row, columns [j0, j1) in order; gridDim.y chunks write raw
// sums to partial[chunk * m + i].
__global__ void __launch_bounds__(kThreads)
    dgemv_n_kernel(int m, int n, const double* __restrict__ A, int lda,
                   const double* __restrict__ x, int incx, int cols_per_chunk,
                   double* __restrict__ partial, double alpha, const double* alpha_dev,
                   double beta, const double* beta_dev, double* y, int incy) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const double al = scalar_of(alpha, alpha_dev);
  double sum = 0.0;
  if (al != 0.0) {
    const int j0 = blockIdx.y * cols_per_chunk;
    const int j1 = min(n, j0 + cols_per_chunk);
    const double* a = A + i + static_cast<long long>(j0) * lda;
    int j = j0;
    for (; j + 3 < j1; j += 4) {
      double v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcs(a + u * static_cast<long long>(lda));
#pragma unroll
      for (int u = 0; u < 4; ++u) sum = fma(v[u], __ldg(x + vidx(j + u, n, incx)), sum);
      a += 4ll * lda;
    }
    for (; j < j1; ++j, a += lda) sum = fma(__ldcs(a), __ldg(x + vidx(j, n, incx)), sum);
  }
  if (gridDim.y > 1) {
    partial[static_cast<long long>(blockIdx.y) * m + i] = sum;
    return;
  }
  gemv_write(y + vidx(i, m, incy), al, sum, scalar_of(beta, beta_dev));
}

// op(A) = A^T: warp per column c, lanes striding the rows [r0, r1).
__global__ void __launch_bounds__(kThreads)
    dgemv_t_kernel(int m, int n, const double* __restrict__ A, int lda,
                   const double* __restrict__ x, int incx, int rows_per_chunk,
                   double* __restrict__ partial, double alpha, const double* alpha_dev,
                   double beta, const double* beta_dev, double* y, int incy) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (c >= n) return;
  const double al = scalar_of(alpha, alpha_dev);
  double s0 = 0.0, s1 = 0.0;
  if (al != 0.0) {
    const int r0 = blockIdx.y * rows_per_chunk;
    const int r1 = min(m, r0 + rows_per_chunk);
    const double* col = A + static_cast<long long>(c) * lda;
    int r = r0 + lane;
    for (; r + 32 < r1; r += 64) {
      const double a0 = __ldcs(col + r), a1 = __ldcs(col + r + 32);
      s0 = fma(a0, __ldg(x + vidx(r, m, incx)), s0);
      s1 = fma(a1, __ldg(x + vidx(r + 32, m, incx)), s1);
    }
    if (r < r1) s0 = fma(__ldcs(col + r), __ldg(x + vidx(r, m, incx)), s0);
  }
  double sum = s0 + s1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  if (lane != 0) return;
  if (gridDim.y > 1) {
    partial[static_cast<long long>(blockIdx.y) * n + c] = sum;
    return;
  }
  gemv_write(y + vidx(c, n, incy), al, sum, scalar_of(beta, beta_dev));
}

__global__ void __launch_bounds__(kThreads)
    dgemv_finish(int len, int chunks, const double* __restrict__ partial, double alpha,
                 const double* alpha_dev, double beta, const double* beta_dev, double* y,
                 int incy) {
  const double al = scalar_of(alpha, alpha_dev);
  const double be = scalar_of(beta, beta_dev);
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < len;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    double s = 0.0;
    for (int c = 0; c < chunks; ++c) s += __ldcs(partial + static_cast<long long>(c) * len + i);
    gemv_write(y + vidx(i, len, incy), al, s, be);
  }
}

int dgemv_chunks(bool trans, int m, int n) {
  const int sms = sm_count(current_device());
  const long long target = static_cast<long long>(sms > 0 ? sms : 148) * kCtasPerSm;
  const long long outer_blocks = trans ? (n + kThreads / 32 - 1) / (kThreads / 32)
                                       : (m + kThreads - 1) / kThreads;
  if (2 * outer_blocks >= target) return 1;
  const int inner = trans ? m : n;
  long long c = target / outer_blocks;
  const long long max_c = (inner + 255) / 256;
  if (c > max_c) c = max_c;
  return c < 1 ? 1 : static_cast<int>(c);
}

// ------------------------------------------------------------------ gemm

// fp64 tensor-core MMA, D(8x8) = A(8x4) B(4x8) + D.  Fragments (PTX ISA, mma.m8n8k4 with
// .f64 operands): lane l holds A(l/4, l%4), B(l%4, l/4) and D(l/4, 2(l%4)) and
// D(l/4, 2(l%4) + 1).
__device__ __forceinline__ void dmma(double (&d)[2], double a, double b) {
  asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
      : "+d"(d[0]), "+d"(d[1])
      : "d"(a), "d"(b));
}

// 8-byte asynchronous copy global -> shared; `ok` false writes zero and reads nothing.
__device__ __forceinline__ void cp_async8(double* dst, const double* src, bool ok) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(s), "l"(src),
               "r"(ok ? 8 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kDBK = 32;     // k per stage: eight MMA k-steps
constexpr int kDStages = 2;  // the copy of stage kt + 1 flies while stage kt computes

// One operand's stage in shared memory: element (i, kk), i along M (or N) and kk along
// K, sits at kk * (ROWS + 4) + i when the operand is contiguous along M / N in global
// memory and at i * (kDBK + 4) + kk when it is contiguous along K, so the copies write
// contiguous runs.  Both strides are 4 (mod 16) doubles: the 16 (i, kk) pairs a
// half-warp reads for one fragment (4 consecutive i by 4 consecutive kk) land in 16
// different bank pairs.
template <int ROWS, bool MN_CONTIG>
struct DTile {
  static constexpr int kElems = MN_CONTIG ? kDBK * (ROWS + 4) : ROWS * (kDBK + 4);
  __device__ static int at(int i, int kk) {
    return MN_CONTIG ? kk * (ROWS + 4) + i : i * (kDBK + 4) + kk;
  }
};

// Stage sizes: the larger of the two layouts of each operand, so one size serves every
// transpose.
template <int BM, int BN>
struct DStage {
  static constexpr int kA = DTile<BM, true>::kElems > DTile<BM, false>::kElems
                                ? DTile<BM, true>::kElems
                                : DTile<BM, false>::kElems;
  static constexpr int kB = DTile<BN, true>::kElems > DTile<BN, false>::kElems
                                ? DTile<BN, true>::kElems
                                : DTile<BN, false>::kElems;
  static constexpr int kSmemBytes = kDStages * (kA + kB) * 8;
};

// Copies rows r0 .. r0 + ROWS - 1 (i) by k0 .. k0 + kDBK - 1 (kk) of an operand into
// `dst`: element (i, kk) of op(X) is X[r + k * ld] when X is contiguous along M / N and
// X[k + r * ld] otherwise; rows >= R and k >= K read as zero.
template <int ROWS, int THREADS, bool MN_CONTIG>
__device__ __forceinline__ void dgemm_stage_copy(double* dst, const double* X, long long ld,
                                                 int r0, int R, int k0, int K, int tid) {
  using TL = DTile<ROWS, MN_CONTIG>;
#pragma unroll
  for (int p = 0; p < ROWS * kDBK / THREADS; ++p) {
    const int e = tid + THREADS * p;
    const int i = MN_CONTIG ? e % ROWS : e / kDBK;
    const int kk = MN_CONTIG ? e / ROWS : e % kDBK;
    const bool ok = r0 + i < R && k0 + kk < K;
    const double* src =
        !ok ? X
            : (MN_CONTIG ? X + (r0 + i) + static_cast<long long>(k0 + kk) * ld
                         : X + (k0 + kk) + static_cast<long long>(r0 + i) * ld);
    cp_async8(dst + TL::at(i, kk), src, ok);
  }
}

// CTA tile BM x 64 (BM = 128: 8 warps as 4 x 2; BM = 64: 4 warps as 2 x 2), warp tile
// 32 x 32 = 4 x 4 MMA tiles (32 accumulators per lane), k in stages through a cp.async
// ring.  Per k-step a warp reads 8 fragments (one double per lane each) for 16 MMAs of
// 256 FMAs: shared-memory traffic is a small fraction of the fp64 pipe's time, where a
// register-blocked DFMA kernel is bound by its operand reads.
template <int BM, int BN, bool TA, bool TB>
__global__ void __launch_bounds__(BM * BN / 32, BM * BN >= 128 * 128 ? 1 : (BM == 128 ? 2 : 3))
    dgemm_kernel(const DgemmArgs g) {
  constexpr int THREADS = BM * BN / 32;
  using TileA = DTile<BM, !TA>;
  using TileB = DTile<BN, TB>;
  constexpr int kStageA = DStage<BM, BN>::kA, kStageB = DStage<BM, BN>::kB;
  extern __shared__ __align__(16) double dsm[];
  double* As = dsm;
  double* Bs = dsm + kDStages * kStageA;

  const double alpha = scalar_of(g.alpha, g.alpha_dev);
  const double beta = scalar_of(g.beta, g.beta_dev);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp % (BM / 32), wn = warp / (BM / 32);
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int kt_count = (g.k + kDBK - 1) / kDBK;

  for (int z = blockIdx.z; z < g.batch; z += gridDim.z) {
    const double* A = g.a + z * g.stride_a;
    const double* B = g.b + z * g.stride_b;
    double* Cm = g.c + z * g.stride_c;
    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;

    if (alpha != 0.0 && g.k > 0) {
      auto load = [&](int slot, int kt) {
        dgemm_stage_copy<BM, THREADS, !TA>(As + slot * kStageA, A, g.lda, m0, g.m, kt * kDBK,
                                           g.k, tid);
        dgemm_stage_copy<BN, THREADS, TB>(Bs + slot * kStageB, B, g.ldb, n0, g.n, kt * kDBK,
                                            g.k, tid);
      };
#pragma unroll
      for (int s = 0; s < kDStages - 1; ++s) {
        if (s < kt_count) load(s, s);
        cp_async_commit();
      }
      for (int kt = 0; kt < kt_count; ++kt) {
        cp_async_wait<kDStages - 2>();  // stage kt has landed (this thread's copies)
        __syncthreads();                // everyone's, and stage kt - 1 is no longer read
        const int nk = kt + kDStages - 1;
        if (nk < kt_count) load(nk % kDStages, nk);
        cp_async_commit();
        const double* as = As + (kt % kDStages) * kStageA;
        const double* bs = Bs + (kt % kDStages) * kStageB;
#pragma unroll
        for (int ks = 0; ks < kDBK / 4; ++ks) {
          const int kk = ks * 4 + (lane & 3);
          double a[4], b[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) a[i] = as[TileA::at(wm * 32 + i * 8 + (lane >> 2), kk)];
#pragma unroll
          for (int j = 0; j < 4; ++j) b[j] = bs[TileB::at(wn * 32 + j * 8 + (lane >> 2), kk)];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) dmma(acc[i][j], a[i], b[j]);
        }
      }
      cp_async_wait<0>();
      __syncthreads();  // the next batch entry refills the ring
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gm = m0 + wm * 32 + i * 8 + (lane >> 2);
      if (gm >= g.m) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int gn = n0 + wn * 32 + j * 8 + 2 * (lane & 3) + e;
          if (gn >= g.n) continue;
          double* cp = Cm + gm + static_cast<long long>(gn) * g.ldc;
          const double prev = beta == 0.0 ? 0.0 : beta * *cp;
          *cp = fma(alpha, acc[i][j][e], prev);
        }
      }
    }
  }
}

template <int BM, int BN, bool TA, bool TB>
cudaError_t launch_dgemm_kernel(const DgemmArgs& g, dim3 grid, cudaStream_t stream) {
  constexpr int smem = DStage<BM, BN>::kSmemBytes;
  auto kern = dgemm_kernel<BM, BN, TA, TB>;
  const cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, BM * BN / 32, smem, stream>>>(g);
  return cudaGetLastError();
}

template <int BM, int BN>
cudaError_t launch_dgemm_tiles(const DgemmArgs& g, cudaStream_t stream) {
  const dim3 grid((g.m + BM - 1) / BM, (g.n + BN - 1) / BN,
                  static_cast<unsigned>(g.batch < 65535 ? g.batch : 65535));
  if (g.trans_a) {
    return g.trans_b ? launch_dgemm_kernel<BM, BN, true, true>(g, grid, stream)
                     : launch_dgemm_kernel<BM, BN, true, false>(g, grid, stream);
  }
  return g.trans_b ? launch_dgemm_kernel<BM, BN, false, true>(g, grid, stream)
                   : launch_dgemm_kernel<BM, BN, false, false>(g, grid, stream);
}

}  // namespace

cudaError_t launch_daxpy(int n, double alpha, const double* alpha_dev, const double* x, int incx,
                         double* y, int incy, cudaStream_t stream) noexcept {
  return launch_elt<Elt::kAxpy>(n, alpha, alpha_dev, x, incx, y, incy, stream);
}
cudaError_t launch_dcopy(int n, const double* x, int incx, double* y, int incy,
                         cudaStream_t stream) noexcept {
  return launch_elt<Elt::kCopy>(n, 0.0, nullptr, x, incx, y, incy, stream);
}
cudaError_t launch_dscal(int n, double alpha, const double* alpha_dev, double* x, int incx,
                         cudaStream_t stream) noexcept {
  if (incx <= 0) return cudaSuccess;
  return launch_elt<Elt::kScal>(n, alpha, alpha_dev, x, incx, x, incx, stream);
}
cudaError_t launch_dswap(int n, double* x, int incx, double* y, int incy,
                         cudaStream_t stream) noexcept {
  return launch_elt<Elt::kSwap>(n, 0.0, nullptr, x, incx, y, incy, stream);
}

std::size_t dreduce_scratch_bytes() noexcept { return sizeof(Scratch); }

cudaError_t launch_dreduce(Reduce op, int n, const double* x, int incx, const double* y, int incy,
                           void* out, void* scratch, cudaStream_t stream) noexcept {
  const bool empty = n <= 0 || (op != Reduce::kDot && incx <= 0);
  if (empty) {
    dreduce_empty<<<1, 1, 0, stream>>>(out, op == Reduce::kAmax ? 1 : 0);
    return cudaGetLastError();
  }
  Scratch* s = static_cast<Scratch*>(scratch);
  switch (op) {
    case Reduce::kDot:
      return launch_r<Reduce::kDot>(n, x, incx, y, incy, out, s, stream);
    case Reduce::kNrm2:
      return launch_r<Reduce::kNrm2>(n, x, incx, nullptr, 0, out, s, stream);
    case Reduce::kAsum:
      return launch_r<Reduce::kAsum>(n, x, incx, nullptr, 0, out, s, stream);
    case Reduce::kAmax:
      return launch_r<Reduce::kAmax>(n, x, incx, nullptr, 0, out, s, stream);
  }
  return cudaErrorInvalidValue;
}

std::size_t dgemv_workspace_bytes(bool trans, int m, int n) noexcept {
  if (m <= 0 || n <= 0) return 0;
  const int chunks = dgemv_chunks(trans, m, n);
  return chunks > 1 ? static_cast<std::size_t>(chunks) * (trans ? n : m) * sizeof(double) : 0;
}

cudaError_t launch_dgemv(bool trans, int m, int n, double alpha, const double* alpha_dev,
                         const double* A, int lda, const double* x, int incx, double beta,
                         const double* beta_dev, double* y, int incy, void* workspace,
                         std::size_t ws_bytes, cudaStream_t stream) noexcept {
  if (m <= 0 || n <= 0) return cudaSuccess;
  int chunks = dgemv_chunks(trans, m, n);
  if (chunks > 1 && (workspace == nullptr || ws_bytes < dgemv_workspace_bytes(trans, m, n)))
    chunks = 1;
  double* part = static_cast<double*>(workspace);
  const int out_len = trans ? n : m;
  if (!trans) {
    const int per = (n + chunks - 1) / chunks;
    const dim3 grid((m + kThreads - 1) / kThreads, static_cast<unsigned>((n + per - 1) / per));
    dgemv_n_kernel<<<grid, kThreads, 0, stream>>>(m, n, A, lda, x, incx, per, part, alpha,
                                                  alpha_dev, beta, beta_dev, y, incy);
    chunks = static_cast<int>(grid.y);
  } else {
    const int per = (m + chunks - 1) / chunks;
    const dim3 grid((n + kThreads / 32 - 1) / (kThreads / 32),
                    static_cast<unsigned>((m + per - 1) / per));
    dgemv_t_kernel<<<grid, kThreads, 0, stream>>>(m, n, A, lda, x, incx, per, part, alpha,
                                                  alpha_dev, beta, beta_dev, y, incy);
    chunks = static_cast<int>(grid.y);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || chunks == 1) return e;
  dgemv_finish<<<grid_for(out_len), kThreads, 0, stream>>>(out_len, chunks, part, alpha,
                                                           alpha_dev, beta, beta_dev, y, incy);
  return cudaGetLastError();
}

cudaError_t launch_dgemm(const DgemmArgs& g, cudaStream_t stream) noexcept {
  if (g.m <= 0 || g.n <= 0 || g.batch <= 0) return cudaSuccess;
  const int sms = sm_count(current_device());
  // 128 x 64 tiles (two CTAs per SM) when they fill the GPU twice, else 64 x 64
  const long long big_tiles = static_cast<long long>((g.m + 127) / 128) * ((g.n + 63) / 64) *
                              g.batch;
  if (big_tiles >= 2ll * (sms > 0 ? sms : 148)) return launch_dgemm_tiles<128, 64>(g, stream);
  return launch_dgemm_tiles<64, 64>(g, stream);
}

}  // namespace mb200::blas
