// spmv.cpp — restatement of the reference's CSR SpMV and SpMM arithmetic.
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
#include <utility>
#include <vector>

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

// Transposed product y = alpha * A^T * x + beta * y (y has `cols` entries).
// generic == 0 follows the fp32 fast path (cusparse_ops.mm:166-191 and
// cusparse_kernels.metal:21-52): y = (beta == 0 ? 0 : beta * y), then for rows r in
// order, ax = alpha * x[r] (rows with ax == 0 skipped), contrib = ax * values[k],
// nonzero contributions added to y[col] (the reference adds them atomically, in
// an unspecified order; here in row order).  generic == 1 follows the generic
// kernel's op_a == 1 branch (:79-92, and the fp16 kernel :116-132): per column,
// sum = fma(values[k], x[r], sum) over rows in order, then
// y = fma(alpha, sum, beta == 0 ? 0 : beta * y).  exact_col / abs_col (optional)
// receive alpha * sum values*x + beta*y0 and sum |values * x| in double.
extern "C" void oracle_spmv_csr_t(int64_t rows, int64_t cols, const int32_t* row_offsets,
                                  const int32_t* col_ind, const float* values, int base,
                                  const float* x, float* y, float alpha, float beta, int generic,
                                  double* exact_col, double* abs_col) {
  std::vector<double> exact(static_cast<std::size_t>(cols), 0.0), mag(exact);
  std::vector<float> sums(static_cast<std::size_t>(cols), 0.0f);
  std::vector<float> y0(y, y + cols);
  if (!generic)
    for (int64_t c = 0; c < cols; ++c) y[c] = (beta == 0.0f) ? 0.0f : beta * y[c];
  for (int64_t r = 0; r < rows; ++r) {
    const int start = row_offsets[r] - base;
    const int end = row_offsets[r + 1] - base;
    const float ax = alpha * x[r];
    for (int idx = start; idx < end; ++idx) {
      const int col = col_ind[idx] - base;
      const double prod = static_cast<double>(values[idx]) * static_cast<double>(x[r]);
      exact[static_cast<std::size_t>(col)] += prod;
      mag[static_cast<std::size_t>(col)] += std::fabs(prod);
      if (generic) {
        sums[static_cast<std::size_t>(col)] =
            std::fma(values[idx], x[r], sums[static_cast<std::size_t>(col)]);
      } else if (ax != 0.0f) {
        const float contrib = ax * values[idx];
        if (contrib != 0.0f) y[col] += contrib;
      }
    }
  }
  for (int64_t c = 0; c < cols; ++c) {
    const std::size_t i = static_cast<std::size_t>(c);
    if (generic) {
      const float prev = (beta == 0.0f) ? 0.0f : beta * y0[i];
      y[c] = std::fma(alpha, sums[i], prev);
    }
    if (exact_col != nullptr)
      exact_col[c] = static_cast<double>(alpha) * exact[i] +
                     (beta == 0.0f ? 0.0 : static_cast<double>(beta) * y0[i]);
    if (abs_col != nullptr) abs_col[c] = mag[i];
  }
}

namespace {

// load_dense_f32 (cusparse_kernels.metal:195-199): order 1 = column-major.
inline float dense_at(const float* m, int64_t r, int64_t c, int64_t ld, int order, int op) {
  const int64_t er = (op == 0) ? r : c;
  const int64_t ec = (op == 0) ? c : r;
  return (order == 1) ? m[er + ec * ld] : m[er * ld + ec];
}

}  // namespace

// C = alpha * op(A) * op(B) + beta * C following muda_cusparse_spmm_csr_f32
// (cusparse_kernels.metal:201-247): per output (row, col), sum = fma(values[k],
// B_eff(k, col), sum) over the row's entries in order (op_a == 0) or over the
// entries of column `row` of A taken row by row in order (op_a == 1), then
// C = fma(alpha, sum, beta == 0 ? 0 : beta * C); order 1 = column-major.  exact and
// mag (optional, out_rows x ncols row-major) receive alpha * sum + beta * C0 in
// double and sum |values * B|.
extern "C" void oracle_spmm_csr(int64_t a_rows, int64_t a_cols, const int32_t* row_offsets,
                                const int32_t* col_ind, const float* values, int base, int op_a,
                                const float* B, int64_t ldb, int order_b, int op_b, float* C,
                                int64_t ldc, int order_c, int64_t ncols, float alpha, float beta,
                                double* exact, double* mag, int threads) {
  const int64_t out_rows = (op_a == 0) ? a_rows : a_cols;
  // entries of each output row, in the order the reference visits them
  std::vector<std::vector<std::pair<int64_t, int>>> lists;  // (B row, entry)
  if (op_a != 0) {
    lists.resize(static_cast<std::size_t>(a_cols));
    for (int64_t r = 0; r < a_rows; ++r)
      for (int idx = row_offsets[r] - base; idx < row_offsets[r + 1] - base; ++idx) {
        const int64_t j = col_ind[idx] - base;
        if (j >= 0 && j < a_cols) lists[static_cast<std::size_t>(j)].push_back({r, idx});
      }
  }
  oracle_detail::parallel_for(0, out_rows, threads, [&](std::int64_t row) {
    for (int64_t col = 0; col < ncols; ++col) {
      float sum = 0.0f;
      double ex = 0.0, mg = 0.0;
      auto term = [&](int idx, int64_t brow) {
        const float b = dense_at(B, brow, col, ldb, order_b, op_b);
        sum = std::fma(values[idx], b, sum);
        const double p = static_cast<double>(values[idx]) * static_cast<double>(b);
        ex += p;
        mg += std::fabs(p);
      };
      if (op_a == 0) {
        for (int idx = row_offsets[row] - base; idx < row_offsets[row + 1] - base; ++idx)
          term(idx, col_ind[idx] - base);
      } else {
        for (const auto& e : lists[static_cast<std::size_t>(row)]) term(e.second, e.first);
      }
      const int64_t ci = (order_c == 1) ? (row + col * ldc) : (row * ldc + col);
      const float prev = (beta == 0.0f) ? 0.0f : beta * C[ci];
      if (exact != nullptr)
        exact[row * ncols + col] = static_cast<double>(alpha) * ex +
                                   (beta == 0.0f ? 0.0 : static_cast<double>(beta) * C[ci]);
      if (mag != nullptr) mag[row * ncols + col] = mg;
      C[ci] = std::fma(alpha, sum, prev);
    }
  });
}
