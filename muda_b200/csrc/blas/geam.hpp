// geam.hpp — launch interface of the cuBLAS geam kernels (fp32 and fp64).
//
// C = alpha * op(A) + beta * op(B) with column-major m x n C.  op(X) is X
// (trans false, X is m x n with leading dimension ldx) or X^T (trans true, X is
// n x m).  Scalars come from *alpha_dev / *beta_dev when those are non-null
// (device pointer mode, read by the kernel), else from alpha / beta.  An operand
// whose scalar is zero is not read, so it may be null or hold NaNs.
#pragma once

#include <cuda_runtime_api.h>

namespace mb200::blas {

template <typename T>
cudaError_t launch_geam(bool trans_a, bool trans_b, int m, int n, T alpha, const T* alpha_dev,
                        const T* A, int lda, T beta, const T* beta_dev, const T* B, int ldb,
                        T* C, int ldc, cudaStream_t stream) noexcept;

}  // namespace mb200::blas
