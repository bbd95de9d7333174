// blas12.cpp — restatement of the reference's cuBLAS level-1 / level-2 fp32 arithmetic.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Follows libraries/blas/shaders/cublas_kernels.metal and the host rules of
// libraries/blas/src/cublas_level1.mm / cublas_level2.mm:
//   index of element i with increment inc: inc >= 0 ? i*inc : (i - n + 1)*inc (:19-20);
//   axpy  y = fma(alpha, x, y), nothing when alpha == 0 (cublas_level1.mm:239-241);
//   scal  x = alpha == 0 ? 0 : alpha * x, nothing when incx <= 0 (:65-66);
//   copy, swap elementwise (:35-91);
//   dot   sequential fma over i (:93-130), nrm2 sqrt of the sequential fma of x*x
//         (:185-215), asum the sequential sum of |x| (:264-293); the reference's
//         parallel order differs, so these also return the double-precision value
//         and the sum of magnitudes for error bounds;
//   isamax the 1-based index of the first largest |x|, NaN never chosen, 0 when
//         n <= 0 or incx <= 0 (:452-495);
//   gemv  per output, sequential fma over the inner index, then
//         fma(alpha, sum, beta == 0 ? 0 : beta * y) (:497-524).
#include <cmath>
#include <cstdint>

#include "oracle.h"
#include "parallel.h"

namespace {

inline int64_t vidx(int64_t i, int n, int inc) {
  return inc >= 0 ? i * inc : (i - n + 1) * static_cast<int64_t>(inc);
}

}  // namespace

extern "C" {

void oracle_saxpy(int n, float alpha, const float* x, int incx, float* y, int incy) {
  if (n <= 0 || alpha == 0.0f) return;
  for (int64_t i = 0; i < n; ++i) {
    float* yp = y + vidx(i, n, incy);
    *yp = std::fma(alpha, x[vidx(i, n, incx)], *yp);
  }
}

void oracle_scopy(int n, const float* x, int incx, float* y, int incy) {
  for (int64_t i = 0; i < n; ++i) y[vidx(i, n, incy)] = x[vidx(i, n, incx)];
}

void oracle_sscal(int n, float alpha, float* x, int incx) {
  if (n <= 0 || incx <= 0) return;
  for (int64_t i = 0; i < n; ++i) {
    float* p = x + i * incx;
    *p = (alpha == 0.0f) ? 0.0f : alpha * *p;
  }
}

void oracle_sswap(int n, float* x, int incx, float* y, int incy) {
  for (int64_t i = 0; i < n; ++i) {
    float* a = x + vidx(i, n, incx);
    float* b = y + vidx(i, n, incy);
    const float t = *a;
    *a = *b;
    *b = t;
  }
}

/* op 0 dot, 1 nrm2, 2 asum.  out_f32: the reference formula in sequential fp32;
 * out_f64: the same in double; out_abs: sum of |terms| in double (dot: |x*y|,
 * nrm2: x*x, asum: |x|), for error bounds. */
void oracle_sreduce(int op, int n, const float* x, int incx, const float* y, int incy,
                    float* out_f32, double* out_f64, double* out_abs) {
  float acc = 0.0f;
  double acc64 = 0.0, mag = 0.0;
  const bool empty = n <= 0 || (op != 0 && incx <= 0);
  if (!empty) {
    for (int64_t i = 0; i < n; ++i) {
      const float u = x[vidx(i, n, incx)];
      if (op == 0) {
        const float v = y[vidx(i, n, incy)];
        acc = std::fma(u, v, acc);
        acc64 += static_cast<double>(u) * v;
        mag += std::fabs(static_cast<double>(u) * v);
      } else if (op == 1) {
        acc = std::fma(u, u, acc);
        acc64 += static_cast<double>(u) * u;
        mag += static_cast<double>(u) * u;
      } else {
        acc += std::fabs(u);
        acc64 += std::fabs(static_cast<double>(u));
        mag += std::fabs(static_cast<double>(u));
      }
    }
  }
  if (op == 1) {
    acc = std::sqrt(acc);
    acc64 = std::sqrt(acc64);
  }
  if (out_f32) *out_f32 = acc;
  if (out_f64) *out_f64 = acc64;
  if (out_abs) *out_abs = mag;
}

int oracle_isamax(int n, const float* x, int incx) {
  if (n <= 0 || incx <= 0) return 0;
  float best = -1.0f;
  int idx = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float v = std::fabs(x[i * incx]);
    if (v > best) {
      best = v;
      idx = static_cast<int>(i + 1);
    }
  }
  return idx;
}

/* exact (optional): alpha * op(A) x + beta * y in double per output;
 * absv (optional): |alpha| * |op(A)| |x| + |beta * y| in double per output. */
void oracle_sgemv(int trans, int m, int n, float alpha, const float* A, int64_t lda,
                  const float* x, int incx, float beta, float* y, int incy, double* exact,
                  double* absv, int threads) {
  const int out_len = trans ? n : m;
  const int inner = trans ? m : n;
  oracle_detail::parallel_for(0, out_len, threads, [&](std::int64_t r) {
    float sum = 0.0f;
    double s64 = 0.0, a64 = 0.0;
    for (int64_t j = 0; j < inner; ++j) {
      const float a = trans ? A[j + r * lda] : A[r + j * lda];
      const float u = x[vidx(j, inner, incx)];
      sum = std::fma(a, u, sum);
      s64 += static_cast<double>(a) * u;
      a64 += std::fabs(static_cast<double>(a) * u);
    }
    float* yp = y + vidx(r, out_len, incy);
    const double y0 = *yp;
    const float prev = (beta == 0.0f) ? 0.0f : beta * *yp;
    if (exact) exact[r] = alpha * s64 + (beta == 0.0f ? 0.0 : beta * y0);
    if (absv) absv[r] = std::fabs(alpha) * a64 + (beta == 0.0f ? 0.0 : std::fabs(beta * y0));
    *yp = std::fma(alpha, sum, prev);
  });
}

}  // extern "C"

/* Sgeam, restated from libraries/blas/shaders/cublas_kernels.metal:1047-1076:
 * term = scalar != 0 ? scalar * x : +0 for each operand (the operand is not read
 * when its scalar is 0), C = term_a + term_b.  Column-major, op T reads X[c + r*ldx]. */
void oracle_sgeam(int transa, int transb, int m, int n, float alpha, const float* A,
                  int64_t lda, float beta, const float* B, int64_t ldb, float* C, int64_t ldc,
                  int threads) {
  // columns are independent; `threads` splits them for the multi-core CPU baseline
  oracle_detail::parallel_for(0, n, threads, [&](std::int64_t c) {
    for (int64_t r = 0; r < m; ++r) {
      float ta = 0.0f, tb = 0.0f;
      if (alpha != 0.0f) ta = alpha * (transa ? A[c + r * lda] : A[r + c * lda]);
      if (beta != 0.0f) tb = beta * (transb ? B[c + r * ldb] : B[r + c * ldb]);
      C[r + c * ldc] = ta + tb;
    }
  });
}

/* Dgeam, restated from the host loop at libraries/blas/src/cublas_level3.mm:906-927:
 * val = 0; val += alpha * a when alpha != 0; val += beta * b when beta != 0. */
void oracle_dgeam(int transa, int transb, int m, int n, double alpha, const double* A,
                  int64_t lda, double beta, const double* B, int64_t ldb, double* C,
                  int64_t ldc, int threads) {
  oracle_detail::parallel_for(0, n, threads, [&](std::int64_t c) {
    for (int64_t r = 0; r < m; ++r) {
      double val = 0.0;
      if (alpha != 0.0) val += alpha * (transa ? A[c + r * lda] : A[r + c * lda]);
      if (beta != 0.0) val += beta * (transb ? B[c + r * ldb] : B[r + c * ldb]);
      C[r + c * ldc] = val;
    }
  });
}
