// blas64.cpp — restatement of the double-precision BLAS the reference calls.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// The reference's cublasD* entry points (libraries/blas/src/cublas_level1.mm:658-979,
// cublas_level2.mm:135-200, cublas_level3.mm:714-819) synchronise the stream and
// call the host CBLAS (cblas_daxpy ... cblas_dgemm, column-major) of Apple's
// Accelerate framework, a closed third-party library that is not part of the
// reference tree and has no version pin beyond the macOS SDK.  What those calls
// compute is the published reference-BLAS definition (netlib BLAS, as shipped with
// LAPACK 3.12), restated here:
//   element i of (x, n, inc): x[inc >= 0 ? i*inc : (i - n + 1)*inc] (inc 0: x[0]);
//   daxpy   y(i) = y(i) + alpha*x(i) in element order, nothing when alpha == 0;
//   dscal   x(i) = alpha*x(i) (incx > 0);  dcopy, dswap in element order;
//   ddot    sum of x(i)*y(i);  dasum sum of |x(i)|;  dnrm2 sqrt(sum x(i)^2);
//   idamax  1-based index of the first |x(i)| greater than every earlier one,
//           starting from |x(1)| (so a NaN first element gives 1);
//   dgemv   y = alpha*op(A)*x + beta*y;  dgemm C = alpha*op(A)*op(B) + beta*C,
//           beta == 0 replacing y / C without reading it, alpha == 0 leaving out the
//           product.
// The reductions and products are returned together with an extended-precision
// (long double) value and the sum of term magnitudes, so that tests can bound the
// error of any summation order; the element-wise routines are exact restatements
// (built with -ffp-contract=off, every product and sum rounded on its own).
#include <cmath>
#include <cstdint>

#include "oracle.h"
#include "parallel.h"

namespace {

inline std::int64_t ix_of(std::int64_t i, std::int64_t n, std::int64_t inc) {
  return inc >= 0 ? i * inc : (i - n + 1) * inc;
}

}  // namespace

extern "C" {

void oracle_daxpy(int n, double alpha, const double* x, int incx, double* y, int incy) {
  if (n <= 0 || alpha == 0.0) return;
  for (std::int64_t i = 0; i < n; ++i) {
    const double p = alpha * x[ix_of(i, n, incx)];
    double& yi = y[ix_of(i, n, incy)];
    yi = yi + p;
  }
}

void oracle_dcopy(int n, const double* x, int incx, double* y, int incy) {
  for (std::int64_t i = 0; i < n; ++i) y[ix_of(i, n, incy)] = x[ix_of(i, n, incx)];
}

void oracle_dscal(int n, double alpha, double* x, int incx) {
  if (n <= 0 || incx <= 0) return;
  for (std::int64_t i = 0; i < n; ++i) x[i * incx] = alpha * x[i * incx];
}

void oracle_dswap(int n, double* x, int incx, double* y, int incy) {
  for (std::int64_t i = 0; i < n; ++i) {
    double& a = x[ix_of(i, n, incx)];
    double& b = y[ix_of(i, n, incy)];
    const double t = a;
    a = b;
    b = t;
  }
}

// op 0 dot, 1 nrm2, 2 asum.  out[0] = the value in element order in double (nrm2:
// from the extended sum), out[1] = the extended-precision value, out[2] = the sum of
// term magnitudes (for nrm2: of the squares).
void oracle_dreduce(int op, int n, const double* x, int incx, const double* y, int incy,
                    double* out) {
  out[0] = out[1] = out[2] = 0.0;
  if (n <= 0 || (op != 0 && incx <= 0)) return;
  double seq = 0.0;
  long double ext = 0.0L, mag = 0.0L;
  for (std::int64_t i = 0; i < n; ++i) {
    const double u = x[ix_of(i, n, incx)];
    if (op == 0) {
      const double v = y[ix_of(i, n, incy)];
      const double p = u * v;
      seq = seq + p;
      ext += static_cast<long double>(u) * v;
      mag += std::fabs(static_cast<long double>(u) * v);
    } else if (op == 1) {
      ext += static_cast<long double>(u) * u;
      mag += static_cast<long double>(u) * u;
    } else {
      seq = seq + std::fabs(u);
      ext += std::fabs(static_cast<long double>(u));
      mag += std::fabs(static_cast<long double>(u));
    }
  }
  if (op == 1) {
    ext = std::sqrt(ext);
    seq = static_cast<double>(ext);
  }
  out[0] = seq;
  out[1] = static_cast<double>(ext);
  out[2] = static_cast<double>(mag);
}

int oracle_idamax(int n, const double* x, int incx) {
  if (n < 1 || incx <= 0) return 0;
  int best = 1;
  double dmax = std::fabs(x[0]);
  for (std::int64_t i = 1; i < n; ++i) {
    const double a = std::fabs(x[i * incx]);
    if (a > dmax) {
      best = static_cast<int>(i + 1);
      dmax = a;
    }
  }
  return best;
}

// y = alpha*op(A)*x + beta*y with the products summed in extended precision; also
// writes bound[i] = |alpha| (|op(A)| |x|)_i + |beta y_i| when bound is not null.
void oracle_dgemv(int trans, int m, int n, double alpha, const double* A, int lda, const double* x,
                  int incx, double beta, double* y, int incy, double* bound, int threads) {
  const int len = trans ? n : m, inner = trans ? m : n;
  oracle_detail::parallel_for(0, len, threads, [&](std::int64_t i) {
    long double s = 0.0L, mag = 0.0L;
    if (alpha != 0.0) {
      for (std::int64_t j = 0; j < inner; ++j) {
        const double a = trans ? A[j + i * static_cast<std::int64_t>(lda)]
                               : A[i + j * static_cast<std::int64_t>(lda)];
        const double v = x[ix_of(j, inner, incx)];
        s += static_cast<long double>(a) * v;
        mag += std::fabs(static_cast<long double>(a) * v);
      }
    }
    double& yi = y[ix_of(i, len, incy)];
    const long double prev = beta == 0.0 ? 0.0L : static_cast<long double>(beta) * yi;
    if (bound != nullptr)
      bound[i] = static_cast<double>(std::fabs(static_cast<long double>(alpha)) * mag +
                                     std::fabs(prev));
    yi = static_cast<double>(static_cast<long double>(alpha) * s + prev);
  });
}

// C = alpha*op(A)*op(B) + beta*C per batch entry, products summed in extended
// precision.  entries (ne pairs of row, batch*n + column) evaluate only those
// entries; bound (ne or m*n*batch values, in the same order) receives
// |alpha| (|op(A)| |op(B)|)_ij + |beta C_ij| when not null.
void oracle_dgemm(int transa, int transb, int m, int n, int k, double alpha, const double* A,
                  int64_t lda, int64_t sa, const double* B, int64_t ldb, int64_t sb, double beta,
                  double* C, int64_t ldc, int64_t sc, int batch, const int* rows, const int* cols,
                  int ne, double* bound, int threads) {
  const std::int64_t total = ne > 0 ? ne : static_cast<std::int64_t>(m) * n * batch;
  oracle_detail::parallel_for(0, total, threads, [&](std::int64_t t) {
    int i, j, z;
    if (ne > 0) {
      i = rows[t];
      z = cols[t] / n;
      j = cols[t] % n;
    } else {
      z = static_cast<int>(t / (static_cast<std::int64_t>(m) * n));
      const std::int64_t r = t % (static_cast<std::int64_t>(m) * n);
      j = static_cast<int>(r / m);
      i = static_cast<int>(r % m);
    }
    const double* a = A + z * sa;
    const double* b = B + z * sb;
    long double s = 0.0L, mag = 0.0L;
    if (alpha != 0.0) {
      for (std::int64_t p = 0; p < k; ++p) {
        const double av = transa ? a[p + i * lda] : a[i + p * lda];
        const double bv = transb ? b[j + p * ldb] : b[p + j * ldb];
        s += static_cast<long double>(av) * bv;
        mag += std::fabs(static_cast<long double>(av) * bv);
      }
    }
    double& c = C[z * sc + i + j * ldc];
    const long double prev = beta == 0.0 ? 0.0L : static_cast<long double>(beta) * c;
    if (bound != nullptr)
      bound[t] = static_cast<double>(std::fabs(static_cast<long double>(alpha)) * mag +
                                     std::fabs(prev));
    c = static_cast<double>(static_cast<long double>(alpha) * s + prev);
  });
}

}  // extern "C"
