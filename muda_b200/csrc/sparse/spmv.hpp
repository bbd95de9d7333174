// spmv.hpp — launch interface of the CSR SpMV kernels.
#pragma once

#include <cuda_runtime_api.h>

#include <cstdint>

namespace mb200::sparse {

struct CsrView {
  std::int64_t rows;
  std::int64_t cols;
  std::int64_t nnz;
  const std::int32_t* row_offsets;  // rows + 1 entries, index base `base`
  const std::int32_t* col_ind;      // nnz entries, index base `base`
  const float* values;              // nnz entries
  int base;                         // 0 or 1
};

// y = alpha * A * x + beta * y (beta == 0: y is not read), A in CSR.
// Malformed input cannot make the kernel read outside the arrays: row offsets
// are clamped to [0, nnz] and entries whose column is outside [0, cols) are
// skipped.
cudaError_t launch_spmv_csr(const CsrView& a, const float* x, float* y, float alpha, float beta,
                            cudaStream_t stream) noexcept;

// Threads cooperating on one row for a matrix with this shape (for tests/benchmarks).
int spmv_group_width(std::int64_t rows, std::int64_t nnz) noexcept;

}  // namespace mb200::sparse
