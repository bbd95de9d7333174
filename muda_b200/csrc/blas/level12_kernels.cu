// level12_kernels.cu — cuBLAS level-1 and level-2 fp32 kernels (HBM-bound).
//
// Per-element arithmetic follows the reference kernels (libraries/blas/shaders/
// cublas_kernels.metal): axpy y = fma(alpha, x, y) (:11-33), scal
// x = alpha == 0 ? 0 : alpha * x (:57-76), dot / nrm2 accumulate with fma and
// asum with adds (:93-338), isamax keeps the first largest |x| and never picks a
// NaN (:364-495), gemv accumulates fma over the inner index and finishes with
// fma(alpha, sum, beta == 0 ? 0 : beta * y) (:497-592).  Only the order in which
// partial sums of the reductions are combined differs.
//
// B200 layout: elementwise kernels are grid-stride over a whole number of waves
// (8 CTAs x 148 SMs), with 16-byte vectors on unit-stride, aligned vectors.
// Reductions are one launch: each CTA reduces a fixed slice into a partial, and
// the last CTA to finish (a counter in the scratch) adds the partials in CTA
// order, so results are deterministic and nothing waits on another CTA.  gemv N
// gives every thread one row (coalesced column reads, x broadcast from L1) and,
// when m is too small to fill the GPU, splits the columns into chunks whose
// partial rows are added in chunk order by a second pass; gemv T gives every
// warp one column, splitting the rows the same way when n is small.
#include "blas/level12.hpp"

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
__device__ __forceinline__ void apply(float a, const float* x, float* y, long long ix, long long iy) {
  if constexpr (E == Elt::kAxpy) {
    y[iy] = fmaf(a, x[ix], y[iy]);
  } else if constexpr (E == Elt::kCopy) {
    y[iy] = x[ix];
  } else if constexpr (E == Elt::kScal) {
    float* xx = const_cast<float*>(x);
    xx[ix] = (a == 0.0f) ? 0.0f : a * xx[ix];
  } else {
    float* xx = const_cast<float*>(x);
    const float t = xx[ix];
    xx[ix] = y[iy];
    y[iy] = t;
  }
}

template <Elt E>
__device__ __forceinline__ void apply4(float a, const float4* x, float4* y, long long i) {
  if constexpr (E == Elt::kAxpy) {
    const float4 u = x[i];
    float4 v = y[i];
    v.x = fmaf(a, u.x, v.x);
    v.y = fmaf(a, u.y, v.y);
    v.z = fmaf(a, u.z, v.z);
    v.w = fmaf(a, u.w, v.w);
    y[i] = v;
  } else if constexpr (E == Elt::kCopy) {
    y[i] = x[i];
  } else if constexpr (E == Elt::kScal) {
    float4* xx = const_cast<float4*>(x);
    float4 v = xx[i];
    if (a == 0.0f) {
      v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    } else {
      v.x *= a;
      v.y *= a;
      v.z *= a;
      v.w *= a;
    }
    xx[i] = v;
  } else {
    float4* xx = const_cast<float4*>(x);
    const float4 t = xx[i];
    xx[i] = y[i];
    y[i] = t;
  }
}

// Vec: unit strides and 16-byte aligned x (and y): n / 4 vectors plus a scalar tail.
template <Elt E, bool Vec>
__global__ void __launch_bounds__(kThreads)
    elementwise(int n, float alpha, const float* alpha_dev, const float* x, int incx, float* y,
                int incy) {
  const float a = alpha_dev ? *alpha_dev : alpha;
  if (E == Elt::kAxpy && a == 0.0f) return;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if constexpr (Vec) {
    const long long n4 = n / 4;
    for (long long i = t0; i < n4; i += stride)
      apply4<E>(a, reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), i);
    const long long tail = n4 * 4 + t0;
    if (tail < n) apply<E>(a, x, y, tail, tail);
  } else {
    for (long long i = t0; i < n; i += stride) apply<E>(a, x, y, vidx(i, n, incx), vidx(i, n, incy));
  }
}

template <Elt E>
cudaError_t launch_elt(int n, float alpha, const float* alpha_dev, const float* x, int incx,
                       float* y, int incy, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const bool unit = incx == 1 && (E == Elt::kScal || incy == 1);
  const bool vec = unit && aligned_to(x, 16) && (E == Elt::kScal || aligned_to(y, 16));
  if (vec)
    elementwise<E, true><<<grid_for((n + 3) / 4), kThreads, 0, stream>>>(n, alpha, alpha_dev, x,
                                                                          incx, y, incy);
  else
    elementwise<E, false><<<grid_for(n), kThreads, 0, stream>>>(n, alpha, alpha_dev, x, incx, y,
                                                                incy);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ reductions

struct Scratch {
  unsigned counter;  // CTAs finished; the last one resets it to 0
  unsigned pad[3];
  float2 partial[kMaxPartials];  // (value, index bits) per CTA
};

struct Best {
  float v;
  int i;  // 1-based, 0 = none
};

__device__ __forceinline__ Best better(Best a, Best b) {
  if (b.i == 0) return a;
  if (a.i == 0) return b;
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ __forceinline__ void consider(Best& b, float v, long long i) {
  // ascending i within a thread: strict > keeps the first of equal values; NaN never wins
  if (v > b.v) {
    b.v = v;
    b.i = static_cast<int>(i + 1);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ Best warp_best(Best b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best other{__shfl_xor_sync(kFull, b.v, o), __shfl_xor_sync(kFull, b.i, o)};
    b = better(b, other);
  }
  return b;
}

// Block-wide combine of one value per thread (fixed order); result valid in thread 0.
template <Reduce R>
__device__ __forceinline__ float2 block_combine(float2 mine, float2* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float2 r = mine;
  if constexpr (R == Reduce::kAmax) {
    Best b{r.x, __float_as_int(r.y)};
    b = warp_best(b);
    r = make_float2(b.v, __int_as_float(b.i));
  } else {
    r.x = warp_sum(r.x);
  }
  if (lane == 0) sh[warp] = r;
  __syncthreads();
  if (warp == 0) {
    r = lane < kThreads / 32 ? sh[lane] : (R == Reduce::kAmax ? make_float2(-1.0f, 0.0f)
                                                               : make_float2(0.0f, 0.0f));
    if constexpr (R == Reduce::kAmax) {
      Best b{r.x, __float_as_int(r.y)};
      b = warp_best(b);
      r = make_float2(b.v, __int_as_float(b.i));
    } else {
      r.x = warp_sum(r.x);
    }
  }
  __syncthreads();
  return r;
}

template <Reduce R, bool Vec>
__global__ void __launch_bounds__(kThreads)
    reduce_kernel(int n, const float* __restrict__ x, int incx, const float* __restrict__ y,
                  int incy, void* out, Scratch* scratch) {
  __shared__ float2 sh[kThreads / 32];
  __shared__ int last;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  float acc = 0.0f;
  Best best{-1.0f, 0};
  if constexpr (Vec) {
    const long long n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* y4 = reinterpret_cast<const float4*>(y);
    for (long long i = t0; i < n4; i += stride) {
      const float4 u = __ldcs(x4 + i);
      if constexpr (R == Reduce::kDot) {
        const float4 v = __ldcs(y4 + i);
        acc = fmaf(u.x, v.x, acc);
        acc = fmaf(u.y, v.y, acc);
        acc = fmaf(u.z, v.z, acc);
        acc = fmaf(u.w, v.w, acc);
      } else if constexpr (R == Reduce::kNrm2) {
        acc = fmaf(u.x, u.x, acc);
        acc = fmaf(u.y, u.y, acc);
        acc = fmaf(u.z, u.z, acc);
        acc = fmaf(u.w, u.w, acc);
      } else if constexpr (R == Reduce::kAsum) {
        acc += fabsf(u.x);
        acc += fabsf(u.y);
        acc += fabsf(u.z);
        acc += fabsf(u.w);
      } else {
        consider(best, fabsf(u.x), 4 * i);
        consider(best, fabsf(u.y), 4 * i + 1);
        consider(best, fabsf(u.z), 4 * i + 2);
        consider(best, fabsf(u.w), 4 * i + 3);
      }
    }
    const long long tail = n4 * 4 + t0;
    if (tail < n) {
      const float u = x[tail];
      if constexpr (R == Reduce::kDot) acc = fmaf(u, y[tail], acc);
      else if constexpr (R == Reduce::kNrm2) acc = fmaf(u, u, acc);
      else if constexpr (R == Reduce::kAsum) acc += fabsf(u);
      else consider(best, fabsf(u), tail);
    }
  } else {
    for (long long i = t0; i < n; i += stride) {
      const float u = x[vidx(i, n, incx)];
      if constexpr (R == Reduce::kDot) acc = fmaf(u, y[vidx(i, n, incy)], acc);
      else if constexpr (R == Reduce::kNrm2) acc = fmaf(u, u, acc);
      else if constexpr (R == Reduce::kAsum) acc += fabsf(u);
      else consider(best, fabsf(u), i);
    }
  }
  float2 mine = R == Reduce::kAmax ? make_float2(best.v, __int_as_float(best.i))
                                   : make_float2(acc, 0.0f);
  float2 part = block_combine<R>(mine, sh);
  if (threadIdx.x == 0) {
    scratch->partial[blockIdx.x] = part;
    __threadfence();
    last = atomicAdd(&scratch->counter, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (!last) return;
  // the last CTA: add the partials in CTA order (thread t takes t, t + 256, ...)
  __threadfence();
  float2 m2 = R == Reduce::kAmax ? make_float2(-1.0f, 0.0f) : make_float2(0.0f, 0.0f);
  for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
    const float2 p = __ldcg(&scratch->partial[b]);
    if constexpr (R == Reduce::kAmax) {
      const Best c = better(Best{m2.x, __float_as_int(m2.y)}, Best{p.x, __float_as_int(p.y)});
      m2 = make_float2(c.v, __int_as_float(c.i));
    } else {
      m2.x += p.x;
    }
  }
  part = block_combine<R>(m2, sh);
  if (threadIdx.x == 0) {
    if constexpr (R == Reduce::kAmax)
      *static_cast<int*>(out) = __float_as_int(part.y);
    else if constexpr (R == Reduce::kNrm2)
      *static_cast<float*>(out) = sqrtf(part.x);
    else
      *static_cast<float*>(out) = part.x;
    scratch->counter = 0u;
  }
}

template <Reduce R>
cudaError_t launch_r(int n, const float* x, int incx, const float* y, int incy, void* out,
                     Scratch* scratch, cudaStream_t stream) {
  const bool vec = incx == 1 && aligned_to(x, 16) &&
                   (R != Reduce::kDot || (incy == 1 && aligned_to(y, 16)));
  const long long per_thread = 16;
  long long g = (static_cast<long long>(n) + kThreads * per_thread - 1) / (kThreads * per_thread);
  const int sms = sm_count(current_device());
  const long long cap = static_cast<long long>(sms > 0 ? sms : 148) * 4;
  if (g > cap) g = cap;
  if (g > kMaxPartials) g = kMaxPartials;
  if (g < 1) g = 1;
  if (vec)
    reduce_kernel<R, true><<<static_cast<unsigned>(g), kThreads, 0, stream>>>(n, x, incx, y, incy,
                                                                              out, scratch);
  else
    reduce_kernel<R, false><<<static_cast<unsigned>(g), kThreads, 0, stream>>>(n, x, incx, y,
                                                                               incy, out, scratch);
  return cudaGetLastError();
}

// Writes the empty-vector result (0, or index 0) to `out`.
__global__ void reduce_empty(void* out, int is_index) {
  if (is_index)
    *static_cast<int*>(out) = 0;
  else
    *static_cast<float*>(out) = 0.0f;
}

// ------------------------------------------------------------------ gemv

// op(A) = A: thread per row i, sequential fma over the columns [j0, j1).  chunks == 1
// finishes y in place; otherwise the raw sums go to partial[chunk * m + i].
__global__ void __launch_bounds__(kThreads)
    gemv_n_kernel(int m, int n, const float* __restrict__ A, int lda, const float* __restrict__ x,
                  int incx, int cols_per_chunk, float* __restrict__ partial, float alpha,
                  const float* alpha_dev, float beta, const float* beta_dev, float* y, int incy) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const int j0 = blockIdx.y * cols_per_chunk;
  const int j1 = min(n, j0 + cols_per_chunk);
  const float* a = A + i + static_cast<long long>(j0) * lda;
  float sum = 0.0f;
  int j = j0;
  // eight columns per step: the eight loads of A are independent and in flight
  // together (the sums still run in column order)
  for (; j + 7 < j1; j += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __ldcs(a + u * static_cast<long long>(lda));
#pragma unroll
    for (int u = 0; u < 8; ++u) sum = fmaf(v[u], __ldg(x + vidx(j + u, n, incx)), sum);
    a += 8ll * lda;
  }
  for (; j < j1; ++j, a += lda) sum = fmaf(__ldcs(a), __ldg(x + vidx(j, n, incx)), sum);
  if (gridDim.y > 1) {
    partial[static_cast<long long>(blockIdx.y) * m + i] = sum;
    return;
  }
  const float al = alpha_dev ? *alpha_dev : alpha;
  const float be = beta_dev ? *beta_dev : beta;
  float* yp = y + vidx(i, m, incy);
  const float prev = (be == 0.0f) ? 0.0f : be * *yp;
  *yp = fmaf(al, sum, prev);
}

// op(A) = A with 16-byte aligned columns (lda % 4 == 0, m % 4 == 0): thread per 4
// consecutive rows read as one float4 per column, so a CTA streams 4 KB of every
// column; each row's sum still runs over the columns in order.
__global__ void __launch_bounds__(kThreads)
    gemv_n4_kernel(int m, int n, const float* __restrict__ A, int lda, const float* __restrict__ x,
                   int incx, int cols_per_chunk, float* __restrict__ partial, float alpha,
                   const float* alpha_dev, float beta, const float* beta_dev, float* y, int incy) {
  const int i4 = blockIdx.x * blockDim.x + threadIdx.x;  // rows 4*i4 .. 4*i4 + 3
  if (4 * i4 >= m) return;
  const int j0 = blockIdx.y * cols_per_chunk;
  const int j1 = min(n, j0 + cols_per_chunk);
  const float4* a = reinterpret_cast<const float4*>(A + static_cast<long long>(j0) * lda) + i4;
  const long long step = lda / 4;
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  int j = j0;
  for (; j + 3 < j1; j += 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcs(a + u * step);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float xv = __ldg(x + vidx(j + u, n, incx));
      s0 = fmaf(v[u].x, xv, s0);
      s1 = fmaf(v[u].y, xv, s1);
      s2 = fmaf(v[u].z, xv, s2);
      s3 = fmaf(v[u].w, xv, s3);
    }
    a += 4 * step;
  }
  for (; j < j1; ++j, a += step) {
    const float4 v = __ldcs(a);
    const float xv = __ldg(x + vidx(j, n, incx));
    s0 = fmaf(v.x, xv, s0);
    s1 = fmaf(v.y, xv, s1);
    s2 = fmaf(v.z, xv, s2);
    s3 = fmaf(v.w, xv, s3);
  }
  const float sums[4] = {s0, s1, s2, s3};
  if (gridDim.y > 1) {
#pragma unroll
    for (int r = 0; r < 4; ++r) partial[static_cast<long long>(blockIdx.y) * m + 4 * i4 + r] = sums[r];
    return;
  }
  const float al = alpha_dev ? *alpha_dev : alpha;
  const float be = beta_dev ? *beta_dev : beta;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float* yp = y + vidx(4 * i4 + r, m, incy);
    const float prev = (be == 0.0f) ? 0.0f : be * *yp;
    *yp = fmaf(al, sums[r], prev);
  }
}

// op(A) = A^T: warp per column c, lanes striding the rows [r0, r1) (float4 along the
// column with Vec); the column's sum goes to y in place or to partial[chunk * n + c].
template <bool Vec>
__global__ void __launch_bounds__(kThreads)
    gemv_t_kernel(int m, int n, const float* __restrict__ A, int lda, const float* __restrict__ x,
                  int incx, int rows_per_chunk, float* __restrict__ partial, float alpha,
                  const float* alpha_dev, float beta, const float* beta_dev, float* y, int incy) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (c >= n) return;
  const int r0 = blockIdx.y * rows_per_chunk;
  const int r1 = min(m, r0 + rows_per_chunk);
  const float* col = A + static_cast<long long>(c) * lda;
  float s0 = 0.0f, s1 = 0.0f;
  if constexpr (Vec) {
    // r0, r1 are multiples of 4 except the final r1 == m, handled by the tail loop
    const int v1 = r0 + ((r1 - r0) & ~3);
    const float4* c4 = reinterpret_cast<const float4*>(col + r0);
    const float4* x4 = reinterpret_cast<const float4*>(x + r0);
    const int nv = (v1 - r0) / 4;
    int k = lane;
    for (; k + 32 < nv; k += 64) {
      const float4 a = __ldcs(c4 + k), b = __ldcs(c4 + k + 32);
      const float4 u = __ldg(x4 + k), w = __ldg(x4 + k + 32);
      s0 = fmaf(a.x, u.x, s0);
      s0 = fmaf(a.y, u.y, s0);
      s0 = fmaf(a.z, u.z, s0);
      s0 = fmaf(a.w, u.w, s0);
      s1 = fmaf(b.x, w.x, s1);
      s1 = fmaf(b.y, w.y, s1);
      s1 = fmaf(b.z, w.z, s1);
      s1 = fmaf(b.w, w.w, s1);
    }
    for (; k < nv; k += 32) {
      const float4 a = __ldcs(c4 + k);
      const float4 u = __ldg(x4 + k);
      s0 = fmaf(a.x, u.x, s0);
      s0 = fmaf(a.y, u.y, s0);
      s0 = fmaf(a.z, u.z, s0);
      s0 = fmaf(a.w, u.w, s0);
    }
    for (int r = v1 + lane; r < r1; r += 32) s0 = fmaf(col[r], x[r], s0);
  } else {
    for (int r = r0 + lane; r < r1; r += 32) s0 = fmaf(__ldcs(col + r), __ldg(x + vidx(r, m, incx)), s0);
  }
  const float sum = warp_sum(s0 + s1);
  if (lane != 0) return;
  if (gridDim.y > 1) {
    partial[static_cast<long long>(blockIdx.y) * n + c] = sum;
    return;
  }
  const float al = alpha_dev ? *alpha_dev : alpha;
  const float be = beta_dev ? *beta_dev : beta;
  float* yp = y + vidx(c, n, incy);
  const float prev = (be == 0.0f) ? 0.0f : be * *yp;
  *yp = fmaf(al, sum, prev);
}

// y[i] = fma(alpha, sum over chunks of partial[chunk * len + i] (chunk order), beta*y[i]).
__global__ void __launch_bounds__(kThreads)
    gemv_finish(int len, int chunks, const float* __restrict__ partial, float alpha,
                const float* alpha_dev, float beta, const float* beta_dev, float* y, int incy) {
  const float al = alpha_dev ? *alpha_dev : alpha;
  const float be = beta_dev ? *beta_dev : beta;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < len;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float s = 0.0f;
    for (int c = 0; c < chunks; ++c) s += __ldcs(partial + static_cast<long long>(c) * len + i);
    float* yp = y + vidx(i, len, incy);
    const float prev = (be == 0.0f) ? 0.0f : be * *yp;
    *yp = fmaf(al, s, prev);
  }
}

// Chunks of the inner dimension so that the CTAs fill, but do not overflow, one wave
// of 8 CTAs per SM (a partial second wave would run alone for a whole CTA time).
int gemv_chunks(bool trans, int m, int n) {
  const int sms = sm_count(current_device());
  const long long target = static_cast<long long>(sms > 0 ? sms : 148) * kCtasPerSm;
  const long long rows_per_block = m % 4 == 0 ? 4 * kThreads : kThreads;  // gemv_n4_kernel
  const long long outer_blocks = trans ? (n + kThreads / 32 - 1) / (kThreads / 32)
                                       : (m + rows_per_block - 1) / rows_per_block;
  if (2 * outer_blocks >= target) return 1;
  const int inner = trans ? m : n;
  long long c = target / outer_blocks;
  const long long max_c = (inner + 255) / 256;  // keep at least 256 inner elements per chunk
  if (c > max_c) c = max_c;
  return c < 1 ? 1 : static_cast<int>(c);
}

}  // namespace

cudaError_t launch_saxpy(int n, float alpha, const float* alpha_dev, const float* x, int incx,
                         float* y, int incy, cudaStream_t stream) noexcept {
  return launch_elt<Elt::kAxpy>(n, alpha, alpha_dev, x, incx, y, incy, stream);
}
cudaError_t launch_scopy(int n, const float* x, int incx, float* y, int incy,
                         cudaStream_t stream) noexcept {
  return launch_elt<Elt::kCopy>(n, 0.0f, nullptr, x, incx, y, incy, stream);
}
cudaError_t launch_sscal(int n, float alpha, const float* alpha_dev, float* x, int incx,
                         cudaStream_t stream) noexcept {
  if (incx <= 0) return cudaSuccess;
  return launch_elt<Elt::kScal>(n, alpha, alpha_dev, x, incx, x, incx, stream);
}
cudaError_t launch_sswap(int n, float* x, int incx, float* y, int incy,
                         cudaStream_t stream) noexcept {
  return launch_elt<Elt::kSwap>(n, 0.0f, nullptr, x, incx, y, incy, stream);
}

std::size_t reduce_scratch_bytes() noexcept { return sizeof(Scratch); }

cudaError_t launch_reduce(Reduce op, int n, const float* x, int incx, const float* y, int incy,
                          void* out, void* scratch, cudaStream_t stream) noexcept {
  const bool empty = n <= 0 || (op != Reduce::kDot && incx <= 0);
  if (empty) {
    reduce_empty<<<1, 1, 0, stream>>>(out, op == Reduce::kAmax ? 1 : 0);
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

std::size_t gemv_workspace_bytes(bool trans, int m, int n) noexcept {
  if (m <= 0 || n <= 0) return 0;
  const int chunks = gemv_chunks(trans, m, n);
  return chunks > 1 ? static_cast<std::size_t>(chunks) * (trans ? n : m) * sizeof(float) : 0;
}

cudaError_t launch_sgemv(bool trans, int m, int n, float alpha, const float* alpha_dev,
                         const float* A, int lda, const float* x, int incx, float beta,
                         const float* beta_dev, float* y, int incy, void* workspace,
                         std::size_t ws_bytes, cudaStream_t stream) noexcept {
  if (m <= 0 || n <= 0) return cudaSuccess;
  int chunks = gemv_chunks(trans, m, n);
  if (chunks > 1 && (workspace == nullptr || ws_bytes < gemv_workspace_bytes(trans, m, n)))
    chunks = 1;
  float* part = static_cast<float*>(workspace);
  const int out_len = trans ? n : m;
  if (!trans) {
    const int per = (n + chunks - 1) / chunks;
    const bool vec = m % 4 == 0 && lda % 4 == 0 && aligned_to(A, 16);
    const int rows_per_block = vec ? 4 * kThreads : kThreads;
    const dim3 grid((m + rows_per_block - 1) / rows_per_block,
                    static_cast<unsigned>((n + per - 1) / per));
    if (vec)
      gemv_n4_kernel<<<grid, kThreads, 0, stream>>>(m, n, A, lda, x, incx, per, part, alpha,
                                                    alpha_dev, beta, beta_dev, y, incy);
    else
      gemv_n_kernel<<<grid, kThreads, 0, stream>>>(m, n, A, lda, x, incx, per, part, alpha,
                                                   alpha_dev, beta, beta_dev, y, incy);
    chunks = static_cast<int>(grid.y);
  } else {
    int per = (m + chunks - 1) / chunks;
    per = (per + 3) & ~3;  // chunk starts stay 16-byte aligned for the vector loads
    const bool vec = incx == 1 && lda % 4 == 0 && aligned_to(A, 16) && aligned_to(x, 16);
    const dim3 grid((n + kThreads / 32 - 1) / (kThreads / 32),
                    static_cast<unsigned>((m + per - 1) / per));
    if (vec)
      gemv_t_kernel<true><<<grid, kThreads, 0, stream>>>(m, n, A, lda, x, incx, per, part, alpha,
                                                         alpha_dev, beta, beta_dev, y, incy);
    else
      gemv_t_kernel<false><<<grid, kThreads, 0, stream>>>(m, n, A, lda, x, incx, per, part, alpha,
                                                          alpha_dev, beta, beta_dev, y, incy);
    chunks = static_cast<int>(grid.y);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || chunks == 1) return e;
  gemv_finish<<<grid_for(out_len), kThreads, 0, stream>>>(out_len, chunks, part, alpha, alpha_dev,
                                                          beta, beta_dev, y, incy);
  return cudaGetLastError();
}

}  // namespace mb200::blas
