// level12.hpp — launch interface of the cuBLAS level-1 / level-2 fp32 kernels.
//
// Vector element i of (p, n, inc) lives at p[inc >= 0 ? i*inc : (i - n + 1)*inc]
// (BLAS convention, the reference's cublas_kernels.metal:19-20); inc = 0 repeats
// element 0.  Scalars come from *alpha_dev / *beta_dev when those are non-null
// (device pointer mode, read by the kernel), else from alpha / beta.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

namespace mb200::blas {

// y = fma(alpha, x, y); alpha == 0 leaves y untouched (reference cublas_level1.mm:239).
cudaError_t launch_saxpy(int n, float alpha, const float* alpha_dev, const float* x, int incx,
                         float* y, int incy, cudaStream_t stream) noexcept;
cudaError_t launch_scopy(int n, const float* x, int incx, float* y, int incy,
                         cudaStream_t stream) noexcept;
// x = (alpha == 0 ? 0 : alpha * x) for incx > 0 (reference cublas_kernels.metal:57-67).
cudaError_t launch_sscal(int n, float alpha, const float* alpha_dev, float* x, int incx,
                         cudaStream_t stream) noexcept;
cudaError_t launch_sswap(int n, float* x, int incx, float* y, int incy,
                         cudaStream_t stream) noexcept;

enum class Reduce : int { kDot = 0, kNrm2 = 1, kAsum = 2, kAmax = 3 };

// Bytes of device scratch launch_reduce needs; the scratch must be zero-filled
// once before its first use (every launch leaves it zeroed again).
std::size_t reduce_scratch_bytes() noexcept;

// One launch: dot = sum x*y (fma), nrm2 = sqrt(sum x*x), asum = sum |x|, amax = the
// 1-based index of the first largest |x| (0 when n <= 0 or incx <= 0, NaN never
// chosen).  Writes a float (int for amax) to `out` in device memory.  Each CTA
// reduces a fixed slice and the last CTA to finish adds the partials in CTA order,
// so the result does not depend on scheduling.
cudaError_t launch_reduce(Reduce op, int n, const float* x, int incx, const float* y, int incy,
                          void* out, void* scratch, cudaStream_t stream) noexcept;

// y = alpha * op(A) x + beta * y, A column-major m x n (beta == 0: y is not read).
// Needs gemv_workspace_bytes(...) of device workspace for the column-split form
// (0 when a single pass suffices).
std::size_t gemv_workspace_bytes(bool trans, int m, int n) noexcept;
cudaError_t launch_sgemv(bool trans, int m, int n, float alpha, const float* alpha_dev,
                         const float* A, int lda, const float* x, int incx, float beta,
                         const float* beta_dev, float* y, int incy, void* workspace,
                         std::size_t ws_bytes, cudaStream_t stream) noexcept;

}  // namespace mb200::blas
