// dblas.hpp — launch interface of the cuBLAS double-precision kernels.
//
// The reference serves these routines on the host through the platform CBLAS
// (libraries/blas/src/cublas_level1.mm:658-979, cublas_level2.mm:135-200,
// cublas_level3.mm:714-819), i.e. the reference-BLAS definitions: vector element i
// of (p, n, inc) lives at p[inc >= 0 ? i*inc : (i - n + 1)*inc], inc = 0 repeats
// element 0.  Here they are GPU kernels with the same element rules.  Scalars
// come from *alpha_dev / *beta_dev when those are non-null (device pointer mode,
// read by the kernel), else from alpha / beta.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

#include "blas/level12.hpp"

namespace mb200::blas {

// y = y + alpha * x, product and sum rounded separately (reference daxpy); nothing
// when alpha == 0.
cudaError_t launch_daxpy(int n, double alpha, const double* alpha_dev, const double* x, int incx,
                         double* y, int incy, cudaStream_t stream) noexcept;
cudaError_t launch_dcopy(int n, const double* x, int incx, double* y, int incy,
                         cudaStream_t stream) noexcept;
// x = alpha * x for incx > 0 (reference dscal: a plain product, so 0 * inf is nan).
cudaError_t launch_dscal(int n, double alpha, const double* alpha_dev, double* x, int incx,
                         cudaStream_t stream) noexcept;
cudaError_t launch_dswap(int n, double* x, int incx, double* y, int incy,
                         cudaStream_t stream) noexcept;

// Bytes of device scratch launch_dreduce needs (zero-filled once before first use;
// every launch leaves it zeroed again).  Its first word is the same finished-CTA
// counter as launch_reduce's scratch, so one zeroed buffer of the larger size
// serves both.
std::size_t dreduce_scratch_bytes() noexcept;

// One launch, result (double; int for kAmax) written to `out` in device memory:
// dot = sum x*y, nrm2 = sqrt(sum x^2) accumulated in Blue's three scaled sums so
// that no intermediate overflows or underflows, asum = sum |x|, amax = the 1-based
// index of the first largest |x| (0 when n <= 0 or incx <= 0; a NaN is never
// chosen, except that a NaN first element gives 1, as in the reference idamax).
// Partial sums are combined in CTA order, so results do not depend on scheduling.
cudaError_t launch_dreduce(Reduce op, int n, const double* x, int incx, const double* y, int incy,
                           void* out, void* scratch, cudaStream_t stream) noexcept;

// y = alpha * op(A) x + beta * y, A column-major m x n; beta == 0: y is not read;
// alpha == 0: A and x are not read (y = beta * y).  Needs dgemv_workspace_bytes of
// device workspace for the split form (0 when one pass fills the GPU).
std::size_t dgemv_workspace_bytes(bool trans, int m, int n) noexcept;
cudaError_t launch_dgemv(bool trans, int m, int n, double alpha, const double* alpha_dev,
                         const double* A, int lda, const double* x, int incx, double beta,
                         const double* beta_dev, double* y, int incy, void* workspace,
                         std::size_t ws_bytes, cudaStream_t stream) noexcept;

// C = alpha * op(A) op(B) + beta * C for `batch` column-major matrices; beta == 0:
// C is not read; alpha == 0: A and B are not read.
struct DgemmArgs {
  bool trans_a, trans_b;
  int m, n, k;
  const double* a;
  std::int64_t lda, stride_a;
  const double* b;
  std::int64_t ldb, stride_b;
  double* c;
  std::int64_t ldc, stride_c;
  int batch;
  double alpha, beta;
  const double* alpha_dev;
  const double* beta_dev;
};
cudaError_t launch_dgemm(const DgemmArgs& g, cudaStream_t stream) noexcept;

}  // namespace mb200::blas
