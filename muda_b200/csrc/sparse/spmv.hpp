// spmv.hpp — launch interface of the CSR SpMV / SpMM kernels.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

namespace mb200::sparse {

// Element type of the value arrays and dense vectors (fp32 or fp16, the two the
// reference accepts).  fp16 products accumulate in fp32.
enum class Value { kF32, kF16 };

struct CsrView {
  std::int64_t rows;
  std::int64_t cols;
  std::int64_t nnz;
  const std::int32_t* row_offsets;  // rows + 1 entries, index base `base`
  const std::int32_t* col_ind;      // nnz entries, index base `base`
  const void* values;               // nnz entries of the value type
  int base;                         // 0 or 1
};

// y = alpha * A * x + beta * y (beta == 0: y is not read), A in CSR.
// Malformed input cannot make the kernel read outside the arrays: row offsets
// are clamped to [0, nnz] and entries whose column is outside [0, cols) are
// skipped.  `scratch` must hold spmv_csr_scratch_bytes(a) bytes of device memory
// (16-byte aligned; may be null when that is 0) that no other launch uses until this
// one's kernels have run.
std::size_t spmv_csr_scratch_bytes(const CsrView& a) noexcept;
cudaError_t launch_spmv_csr(const CsrView& a, Value t, const void* x, void* y, float alpha,
                            float beta, void* scratch, cudaStream_t stream) noexcept;

// y = alpha * A^T * x + beta * y (y has a.cols entries).  fp32: y is first scaled by
// beta (beta == 0: set to 0), then every stored entry adds alpha*x[r]*value to
// y[col] atomically, zero contributions skipped.  fp16: the sums of value*x[r]
// accumulate atomically in `scratch` (a.cols floats), then y = half(alpha * sum +
// beta * y).  Summation order across rows is unspecified.
cudaError_t launch_spmv_csr_t(const CsrView& a, Value t, const void* x, void* y, float alpha,
                              float beta, float* scratch, cudaStream_t stream) noexcept;

// A dense fp32 matrix operand: element (r, c) of op(M) is
//   m[er + ec * ld] (column-major) or m[er * ld + ec] (row-major),
// with (er, ec) = (r, c), or (c, r) when trans.
struct DenseView {
  float* m;
  std::int64_t ld;
  bool col_major;
  bool trans;
};

// Device scratch of the row scheduler of the row-major SpMM: counters[2 +
// kSpmmLongBuckets] (zeroed by the launch: first-phase position, row-chunk position,
// then the long-row count of each length bucket) and long_rows[long_cap], one region
// of long_cap / kSpmmLongBuckets rows per bucket.  No other call may use it while the
// launch runs.
constexpr int kSpmmLongBuckets = 8;
struct SpmmSched {
  unsigned* counters;
  int* long_rows;
  unsigned long_cap;
};
constexpr unsigned kSpmmLongCap = 65536;
constexpr std::size_t kSpmmSchedHeader = 64;  // counters, padded
static_assert((2 + kSpmmLongBuckets) * 4 <= kSpmmSchedHeader, "counters fit the header");
constexpr std::size_t kSpmmSchedBytes = kSpmmSchedHeader + std::size_t{kSpmmLongCap} * 4;

// C = alpha * op(A) * op(B) + beta * C, fp32, C with out_rows x ncols entries
// (out_rows = a.rows, or a.cols when trans_a).  Without trans_a every output is
// sum_k fma(values[k], B(col_k, c), sum) over the row's entries in order, then
// fma(alpha, sum, beta == 0 ? 0 : beta * C): the reference's own per-output
// arithmetic.  With trans_a, C is scaled by beta and the products are added
// atomically (order unspecified).
// sched (may be null: a static row order) lets row-major B and C in 16-byte vectors
// take the scheduled kernel.
cudaError_t launch_spmm_csr(const CsrView& a, bool trans_a, const DenseView& b,
                            const DenseView& c, std::int64_t ncols, float alpha, float beta,
                            const SpmmSched* sched, cudaStream_t stream) noexcept;

// Threads cooperating on one row for a matrix with this shape (for tests/benchmarks).
int spmv_group_width(std::int64_t rows, std::int64_t nnz) noexcept;

}  // namespace mb200::sparse
