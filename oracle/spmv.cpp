// spmv.cpp — restatement of the reference's CSR SpMV arithmetic (non-transposed).
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Follows muda_cusparse_spmv_csr_f32, op_a == 0 branch
// (libraries/sparse/shaders/cusparse_kernels.metal:54-77): per row,
//   start = row_offsets[r] - base, end = row_offsets[r+1] - base,
//   sum = fma(values[k], x[col_ind[k] - base], sum) for k in [start, end),
//   y[r] = fma(alpha, sum, beta == 0 ? 0 : beta * y[r]).
// Optionally also returns, per row, the exact-product sum alpha * sum values[k]*x[col]
// (+ beta*y) accumulated in double, and sum |values[k]| * |x[col]| (the scale of
// the per-element error bound), also in double.
#include <cmath>
#include <cstdint>

#include "oracle.h"
#include "parallel.h"

extern "C" void oracle_spmv_csr(int64_t rows, const int32_t* row_offsets, const int32_t* col_ind,
                                const float* values, int base, const float* x, float* y,
                                float alpha, float beta, double* exact_row, double* abs_row,
                                int threads) {
  oracle_detail::parallel_for(0, rows, threads, [&](std::int64_t r) {
    const int start = row_offsets[r] - base;
    const int end = row_offsets[r + 1] - base;
    float sum = 0.0f;
    double mag = 0.0;
    double exact = 0.0;
    for (int idx = start; idx < end; ++idx) {
      const int col = col_ind[idx] - base;
      sum = std::fma(values[idx], x[col], sum);
      const double prod = static_cast<double>(values[idx]) * static_cast<double>(x[col]);
      exact += prod;
      mag += std::fabs(prod);
    }
    const float prev = (beta == 0.0f) ? 0.0f : (beta * y[r]);
    if (exact_row != nullptr)
      exact_row[r] = static_cast<double>(alpha) * exact +
                     (beta == 0.0f ? 0.0 : static_cast<double>(beta) * y[r]);
    y[r] = std::fma(alpha, sum, prev);
    if (abs_row != nullptr) abs_row[r] = mag;
  });
}
