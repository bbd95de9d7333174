/*
 * oracle.h — CPU restatements of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  The product (muda_b200/, include/) never links,
 * loads or calls anything here.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use this library, and only as
 * the checker or the timed CPU baseline.
 *
 * Each function names the reference file:line it restates.  The reference
 * (AshitomW/MUDA) is Objective-C++ plus Metal and its build runs only on macOS
 * (CMakeLists.txt:14-15).  Its host Philox generator is plain C++, though:
 * oracle/ref/build.py compiles that file (libraries/rand/src/curand_context.mm)
 * unmodified into oracle/_ref/, and tests/test_oracle_ref.py holds the Philox
 * restatement below to it bit for bit.  The other oracles restate Metal kernel
 * arithmetic and are pinned against every known-answer test the reference's own
 * test suite holds for the path (tests/curand_test.cpp, cublas_test.cpp,
 * cufft_test.cpp, cusparse_test.cpp, cudnn_test.cpp), restated in
 * tests/test_oracle_pins.py.
 *
 * Built with -ffp-contract=off so that every float operation rounds separately,
 * as written in the restated source.
 */
#ifndef MUDA_B200_ORACLE_H_
#define MUDA_B200_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Philox4x32-10 (libraries/rand/src/curand_context.mm:42-185) ---- */
void oracle_philox_block(uint64_t ctr, uint64_t seed, uint32_t out[4]);
void oracle_philox_block4(uint64_t ctr, uint32_t c2, uint64_t seed, uint32_t out[4]);
uint64_t oracle_generate_lognormal(uint64_t seed, uint64_t offset, float* out, size_t n,
                                   float mean, float stddev, int threads);
/* kind 0 uniform, 1 normal, 2 log-normal */
uint64_t oracle_generate_double(uint64_t seed, uint64_t offset, double* out, size_t n, int kind,
                                double mean, double stddev, int threads);
/* mode 0: device-kernel definition (this library); mode 1: the reference's host path */
uint64_t oracle_generate_poisson(uint64_t seed, uint64_t offset, uint32_t* out, size_t n,
                                 double lambda, float exp_neg_lambda, int mode, int threads);
/* Writes n words of the stream that starts at generator offset `offset`;
 * returns the generator offset after the call (offset + 4*ceil(n/4)). */
uint64_t oracle_generate_uint(uint64_t seed, uint64_t offset, uint32_t* out, size_t n,
                              int threads);
uint64_t oracle_generate_uniform(uint64_t seed, uint64_t offset, float* out, size_t n,
                                 int threads);
uint64_t oracle_generate_normal(uint64_t seed, uint64_t offset, float* out, size_t n, float mean,
                                float stddev, int threads);
/* Blocks at arbitrary counters: out[4i..4i+3] = Philox(ctrs[i], seed). */
void oracle_philox_gather(const uint64_t* ctrs, size_t m, uint64_t seed, uint32_t* out,
                          int threads);

/* ---- convolution / softmax (libraries/dnn/shaders/cudnn_kernels.metal) ---- */
/* Geometry of one convolution; field meaning as in libraries/dnn/src/cudnn_kernel_params.h:8-37
 * (element strides; w_format 0 = KCRS, 1 = KRSC; conv_mode 0 = CONVOLUTION, 1 = CROSS_CORRELATION). */
typedef struct {
  int n, c_in, h_in, w_in;
  int64_t x_ns, x_cs, x_hs, x_ws;
  int c_out, h_out, w_out, groups;
  int64_t y_ns, y_cs, y_hs, y_ws;
  int kh, kw, pad_h, pad_w, stride_h, stride_w, dil_h, dil_w;
  int w_format, conv_mode;
  float alpha, beta;
} OracleConvParams;

typedef struct {
  int n, c, h, w;
  int64_t ns, cs, hs, ws;
} OracleTensor4;

float oracle_bf16_round(float v);
/* bf16 != 0: x, w, y are bf16 (widened exactly, result rounded to nearest even).
 * accum_f64 != 0: accumulate in double (ground truth) instead of the sequential fp32 fma. */
void oracle_conv2d_fwd(const void* x, const void* w, void* y, const OracleConvParams* p, int bf16,
                       int accum_f64, int threads);
/* ---- convolution backward, AddTensor, activation, pooling, batch norm
 * (cudnn_kernels.metal:194-714); accum_f64 != 0: sums in double.  For the backward
 * calls p describes the forward convolution: x / c_in is the input (dx for backward
 * data), y / c_out the output (dy). */
void oracle_conv_bwd_data(const float* w, const float* dy, float* dx, const OracleConvParams* p,
                          int accum_f64, int threads);
void oracle_conv_bwd_filter(const float* x, const float* dy, float* dw, const OracleConvParams* p,
                            int accum_f64, double* mag, int threads);
void oracle_conv_bwd_bias(const float* dy, const OracleTensor4* v, float* db, float alpha,
                          float beta, int accum_f64, double* mag);
void oracle_add_tensor(const float* a, const OracleTensor4* av, float* c, const OracleTensor4* cv,
                       float alpha, float beta);
void oracle_activation(const float* x, const OracleTensor4* xv, float* y, const OracleTensor4* yv,
                       int mode, float coef, float alpha, float beta);
void oracle_pooling(const float* x, const OracleTensor4* xv, float* y, const OracleTensor4* yv,
                    int win_h, int win_w, int pad_h, int pad_w, int stride_h, int stride_w,
                    int mode, float alpha, float beta);
void oracle_bn_inference(const float* x, const OracleTensor4* xv, float* y,
                         const OracleTensor4* yv, const float* scale, const float* bias,
                         const float* mean, const float* var, int per_activation, float eps,
                         float alpha, float beta);
void oracle_bn_training(const float* x, const OracleTensor4* xv, float* y, const OracleTensor4* yv,
                        const float* scale, const float* bias, float* running_mean,
                        float* running_var, float* save_mean, float* save_inv_var, float factor,
                        float eps, float alpha, float beta, int accum_f64);

/* ---- GEMM (libraries/blas/shaders/cublas_kernels.metal:969-1045) ---- */
/* type 0 fp32, 1 fp16, 2 bf16 (A, B, C all of that type); column-major.
 * rows/cols (optional, n_entries long): evaluate only entries (rows[t], cols[t] % n)
 * of batch cols[t] / n. */
float oracle_half_round(float v);
void oracle_gemm(int type, int transa, int transb, int m, int n, int k, float alpha,
                 const void* A, int64_t lda, int64_t stride_a, const void* B, int64_t ldb,
                 int64_t stride_b, float beta, void* C, int64_t ldc, int64_t stride_c, int batch,
                 int accum_f64, const int32_t* rows, const int32_t* cols, int64_t n_entries,
                 int threads);

/* ---- cuBLAS level 1 / 2, fp32 (libraries/blas/shaders/cublas_kernels.metal:11-524) ---- */
void oracle_saxpy(int n, float alpha, const float* x, int incx, float* y, int incy);
void oracle_scopy(int n, const float* x, int incx, float* y, int incy);
void oracle_sscal(int n, float alpha, float* x, int incx);
void oracle_sswap(int n, float* x, int incx, float* y, int incy);
/* op 0 dot, 1 nrm2, 2 asum */
void oracle_sreduce(int op, int n, const float* x, int incx, const float* y, int incy,
                    float* out_f32, double* out_f64, double* out_abs);
int oracle_isamax(int n, const float* x, int incx);
void oracle_sgeam(int transa, int transb, int m, int n, float alpha, const float* A,
                  int64_t lda, float beta, const float* B, int64_t ldb, float* C, int64_t ldc,
                  int threads);
void oracle_dgeam(int transa, int transb, int m, int n, double alpha, const double* A,
                  int64_t lda, double beta, const double* B, int64_t ldb, double* C,
                  int64_t ldc, int threads);
/* ---- fp64 BLAS: the reference-BLAS definitions behind the reference's host CBLAS
   calls (libraries/blas/src/cublas_level1.mm:658-979, cublas_level2.mm:135-200,
   cublas_level3.mm:714-819); oracle/blas64.cpp ---- */
void oracle_daxpy(int n, double alpha, const double* x, int incx, double* y, int incy);
void oracle_dcopy(int n, const double* x, int incx, double* y, int incy);
void oracle_dscal(int n, double alpha, double* x, int incx);
void oracle_dswap(int n, double* x, int incx, double* y, int incy);
/* op 0 dot, 1 nrm2, 2 asum: out = {double value, extended value, sum of magnitudes} */
void oracle_dreduce(int op, int n, const double* x, int incx, const double* y, int incy,
                    double* out);
int oracle_idamax(int n, const double* x, int incx);
void oracle_dgemv(int trans, int m, int n, double alpha, const double* A, int lda, const double* x,
                  int incx, double beta, double* y, int incy, double* bound, int threads);
void oracle_dgemm(int transa, int transb, int m, int n, int k, double alpha, const double* A,
                  int64_t lda, int64_t sa, const double* B, int64_t ldb, int64_t sb, double beta,
                  double* C, int64_t ldc, int64_t sc, int batch, const int* rows, const int* cols,
                  int ne, double* bound, int threads);
void oracle_sgemv(int trans, int m, int n, float alpha, const float* A, int64_t lda,
                  const float* x, int incx, float beta, float* y, int incy, double* exact,
                  double* absv, int threads);

/* ---- C2C FFT (libraries/fft/src/cufft_exec.mm:101-211) ---- */
/* in/out: interleaved complex64 with element strides; use_double != 0 writes the
 * double-precision result to out_f64 (same layout) instead of out. */
void oracle_fft_c2c(const float* in, float* out, int rank, const int* dims, int64_t batch,
                    int64_t istride, int64_t idist, int64_t ostride, int64_t odist, int sign,
                    int use_double, double* out_f64, int threads);

/* ---- CSR SpMV (libraries/sparse/shaders/cusparse_kernels.metal:54-77) ---- */
/* exact_row (optional): alpha * sum a_k x_col + beta * y in double;
 * abs_row (optional): per-row sum |a_k * x_col| in double. */
void oracle_spmv_csr(int64_t rows, const int32_t* row_offsets, const int32_t* col_ind,
                     const float* values, int base, const float* x, float* y, float alpha,
                     float beta, double* exact_row, double* abs_row, int threads);

/* Transposed CSR SpMV (cusparse_ops.mm:166-191 fast path, generic = 0;
 * cusparse_kernels.metal:79-92 / 116-132 generic branch, generic = 1). */
void oracle_spmv_csr_t(int64_t rows, int64_t cols, const int32_t* row_offsets,
                       const int32_t* col_ind, const float* values, int base, const float* x,
                       float* y, float alpha, float beta, int generic, double* exact_col,
                       double* abs_col);

/* CSR SpMM (cusparse_kernels.metal:201-247); order 1 = column-major, 2 = row-major. */
void oracle_spmm_csr(int64_t a_rows, int64_t a_cols, const int32_t* row_offsets,
                     const int32_t* col_ind, const float* values, int base, int op_a,
                     const float* B, int64_t ldb, int order_b, int op_b, float* C, int64_t ldc,
                     int order_c, int64_t ncols, float alpha, float beta, double* exact,
                     double* mag, int threads);

/* algo 0 FAST, 1 ACCURATE, 2 LOG; mode_channel 0 INSTANCE, 1 CHANNEL. */
void oracle_softmax_fwd(const float* x, float* y, const OracleTensor4* xd, const OracleTensor4* yd,
                        int algo, int mode_channel, float alpha, float beta, int threads);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_ORACLE_H_ */
