/*
 * cublas_v2.h — C ABI of the B200-native GEMM layer.
 *
 * Drop-in for the MUDA cuBLAS shim's level-3 hot path: names, argument lists and
 * numeric enum values follow libraries/blas/include/cublas_v2.h of the reference
 * (enums cublas_v2.h:20-97, declarations cublas_v2.h:100-201, macro aliases
 * cublas_v2.h:203-229).  Enums are int-width C enums (the reference uses 8-bit
 * enums); cudaDataType_t comes from the CUDA toolkit's library_types.h, whose
 * values are the reference's (CUDA_R_32F=0, CUDA_R_16F=2) plus CUDA_R_16BF=14,
 * which this library accepts as an extension the reference lacks.
 *
 * Matrices are column-major.  Every call is asynchronous on the handle's stream.
 */
#ifndef MUDA_B200_CUBLAS_V2_H_
#define MUDA_B200_CUBLAS_V2_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>
#include <library_types.h>

#ifdef __cplusplus
#include <cuda_fp16.h>
extern "C" {
#else
typedef struct { unsigned short x; } __half;
#endif

/* reference cublas_v2.h:20-30 */
typedef enum {
  CUBLAS_STATUS_SUCCESS = 0,
  CUBLAS_STATUS_NOT_INITIALIZED = 1,
  CUBLAS_STATUS_ALLOC_FAILED = 3,
  CUBLAS_STATUS_INVALID_VALUE = 7,
  CUBLAS_STATUS_ARCH_MISMATCH = 8,
  CUBLAS_STATUS_MAPPING_ERROR = 11,
  CUBLAS_STATUS_EXECUTION_FAILED = 13,
  CUBLAS_STATUS_INTERNAL_ERROR = 14,
  CUBLAS_STATUS_NOT_SUPPORTED = 15
} cublasStatus_t;

/* reference cublas_v2.h:35 */
typedef enum { CUBLAS_OP_N = 0, CUBLAS_OP_T = 1, CUBLAS_OP_C = 2 } cublasOperation_t;

/* reference cublas_v2.h:40-43 */
typedef enum { CUBLAS_POINTER_MODE_HOST = 0, CUBLAS_POINTER_MODE_DEVICE = 1 } cublasPointerMode_t;

/* reference cublas_v2.h:48-53 */
typedef enum {
  CUBLAS_DEFAULT_MATH = 0,
  CUBLAS_TENSOR_OP_MATH = 1,
  CUBLAS_PEDANTIC_MATH = 2,
  CUBLAS_TF32_TENSOR_OP_MATH = 3
} cublasMath_t;

/* reference cublas_v2.h:58-62 */
typedef enum {
  CUBLAS_GEMM_DFALT = -1,
  CUBLAS_GEMM_DEFAULT = -1,
  CUBLAS_GEMM_DEFAULT_TENSOR_OP = 99
} cublasGemmAlgo_t;

/* reference cublas_v2.h:67-74 */
typedef enum {
  CUBLAS_COMPUTE_16F = 64,
  CUBLAS_COMPUTE_16F_PEDANTIC = 65,
  CUBLAS_COMPUTE_32F = 68,
  CUBLAS_COMPUTE_32F_PEDANTIC = 69,
  CUBLAS_COMPUTE_32F_FAST_16F = 74,
  CUBLAS_COMPUTE_32F_FAST_TF32 = 77
} cublasComputeType_t;

struct cublasContext;
typedef struct cublasContext* cublasHandle_t;

/* Handle lifecycle and configuration — reference cublas_context.mm:154-303 */
cublasStatus_t cublasCreate_v2(cublasHandle_t* handle);
cublasStatus_t cublasDestroy_v2(cublasHandle_t handle);
cublasStatus_t cublasGetVersion_v2(cublasHandle_t handle, int* version);
cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, cudaStream_t streamId);
cublasStatus_t cublasGetStream_v2(cublasHandle_t handle, cudaStream_t* streamId);
cublasStatus_t cublasSetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t mode);
cublasStatus_t cublasGetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t* mode);
cublasStatus_t cublasSetMathMode(cublasHandle_t handle, cublasMath_t mode);
cublasStatus_t cublasGetMathMode(cublasHandle_t handle, cublasMath_t* mode);
const char* cublasGetStatusName(cublasStatus_t status);
const char* cublasGetStatusString(cublasStatus_t status);

/* Level-1 (fp32) — reference cublas_level1.mm:221-656 (kernels cublas_kernels.metal:11-495).
   Increments follow BLAS: a negative inc walks the vector from its far end; inc = 0
   repeats element 0.  Reductions write *result on the host (the call then waits for
   the stream) or, in CUBLAS_POINTER_MODE_DEVICE, to device memory asynchronously. */
cublasStatus_t cublasSaxpy_v2(cublasHandle_t handle, int n, const float* alpha, const float* x,
                              int incx, float* y, int incy);      /* cublas_level1.mm:221 */
cublasStatus_t cublasScopy_v2(cublasHandle_t handle, int n, const float* x, int incx, float* y,
                              int incy);                          /* cublas_level1.mm:289 */
cublasStatus_t cublasSscal_v2(cublasHandle_t handle, int n, const float* alpha, float* x,
                              int incx);                          /* cublas_level1.mm:344 */
cublasStatus_t cublasSswap_v2(cublasHandle_t handle, int n, float* x, int incx, float* y,
                              int incy);                          /* cublas_level1.mm:407 */
cublasStatus_t cublasSdot_v2(cublasHandle_t handle, int n, const float* x, int incx,
                             const float* y, int incy, float* result); /* cublas_level1.mm:446 */
cublasStatus_t cublasSnrm2_v2(cublasHandle_t handle, int n, const float* x, int incx,
                              float* result);                     /* cublas_level1.mm:488 */
cublasStatus_t cublasSasum_v2(cublasHandle_t handle, int n, const float* x, int incx,
                              float* result);                     /* cublas_level1.mm:527 */
cublasStatus_t cublasIsamax_v2(cublasHandle_t handle, int n, const float* x, int incx,
                               int* result);                      /* cublas_level1.mm:566 */

/* Level-2 (fp32) — reference cublas_level2.mm:38-133 (kernels cublas_kernels.metal:497-592) */
cublasStatus_t cublasSgemv_v2(cublasHandle_t handle, cublasOperation_t trans, int m, int n,
                              const float* alpha, const float* A, int lda, const float* x,
                              int incx, const float* beta, float* y, int incy);

/* Level-1 / level-2 (fp64) — reference cublas_level1.mm:658-979, cublas_level2.mm:135-200,
   which call the host CBLAS; here GPU kernels (blas/dblas_kernels.cu) with the
   reference-BLAS element rules above.  Reductions deliver *result as for fp32. */
cublasStatus_t cublasDaxpy_v2(cublasHandle_t handle, int n, const double* alpha,
                              const double* x, int incx, double* y,
                              int incy);                          /* cublas_level1.mm:658 */
cublasStatus_t cublasDcopy_v2(cublasHandle_t handle, int n, const double* x, int incx, double* y,
                              int incy);                          /* cublas_level1.mm:705 */
cublasStatus_t cublasDscal_v2(cublasHandle_t handle, int n, const double* alpha, double* x,
                              int incx);                          /* cublas_level1.mm:744 */
cublasStatus_t cublasDswap_v2(cublasHandle_t handle, int n, double* x, int incx, double* y,
                              int incy);                          /* cublas_level1.mm:784 */
cublasStatus_t cublasDdot_v2(cublasHandle_t handle, int n, const double* x, int incx,
                             const double* y, int incy,
                             double* result);                     /* cublas_level1.mm:823 */
cublasStatus_t cublasDnrm2_v2(cublasHandle_t handle, int n, const double* x, int incx,
                              double* result);                    /* cublas_level1.mm:865 */
cublasStatus_t cublasDasum_v2(cublasHandle_t handle, int n, const double* x, int incx,
                              double* result);                    /* cublas_level1.mm:903 */
cublasStatus_t cublasIdamax_v2(cublasHandle_t handle, int n, const double* x, int incx,
                               int* result);                      /* cublas_level1.mm:941 */
cublasStatus_t cublasDgemv_v2(cublasHandle_t handle, cublasOperation_t trans, int m, int n,
                              const double* alpha, const double* A, int lda, const double* x,
                              int incx, const double* beta, double* y,
                              int incy);                          /* cublas_level2.mm:135 */

/* Level-3 — reference cublas_level3.mm:474-617 */
/* C = alpha * op(A) + beta * op(B), column-major m x n; an operand whose scalar is 0
 * is not read.  Reference: libraries/blas/include/cublas_v2.h:194-201 (implemented
 * at libraries/blas/src/cublas_level3.mm:619-712 and :821-927). */
cublasStatus_t cublasSgeam(cublasHandle_t handle, cublasOperation_t transa,
                           cublasOperation_t transb, int m, int n, const float* alpha,
                           const float* A, int lda, const float* beta, const float* B, int ldb,
                           float* C, int ldc);
cublasStatus_t cublasDgeam(cublasHandle_t handle, cublasOperation_t transa,
                           cublasOperation_t transb, int m, int n, const double* alpha,
                           const double* A, int lda, const double* beta, const double* B,
                           int ldb, double* C, int ldc);
cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, cublasOperation_t transa,
                              cublasOperation_t transb, int m, int n, int k, const float* alpha,
                              const float* A, int lda, const float* B, int ldb, const float* beta,
                              float* C, int ldc);

cublasStatus_t cublasHgemm(cublasHandle_t handle, cublasOperation_t transa,
                           cublasOperation_t transb, int m, int n, int k, const __half* alpha,
                           const __half* A, int lda, const __half* B, int ldb, const __half* beta,
                           __half* C, int ldc);

cublasStatus_t cublasGemmEx(cublasHandle_t handle, cublasOperation_t transa,
                            cublasOperation_t transb, int m, int n, int k, const void* alpha,
                            const void* A, cudaDataType Atype, int lda, const void* B,
                            cudaDataType Btype, int ldb, const void* beta, void* C,
                            cudaDataType Ctype, int ldc, int computeType, cublasGemmAlgo_t algo);

cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t handle, cublasOperation_t transa,
                                         cublasOperation_t transb, int m, int n, int k,
                                         const float* alpha, const float* A, int lda,
                                         long long int strideA, const float* B, int ldb,
                                         long long int strideB, const float* beta, float* C,
                                         int ldc, long long int strideC, int batchCount);

/* fp64 GEMM — reference cublas_level3.mm:714-819 (host CBLAS dgemm per batch entry);
   here the register-blocked DFMA kernel of blas/dblas_kernels.cu. */
cublasStatus_t cublasDgemm_v2(cublasHandle_t handle, cublasOperation_t transa,
                              cublasOperation_t transb, int m, int n, int k, const double* alpha,
                              const double* A, int lda, const double* B, int ldb,
                              const double* beta, double* C, int ldc); /* cublas_level3.mm:714 */
cublasStatus_t cublasDgemmStridedBatched(cublasHandle_t handle, cublasOperation_t transa,
                                         cublasOperation_t transb, int m, int n, int k,
                                         const double* alpha, const double* A, int lda,
                                         long long int strideA, const double* B, int ldb,
                                         long long int strideB, const double* beta, double* C,
                                         int ldc, long long int strideC,
                                         int batchCount);         /* cublas_level3.mm:722 */

cublasStatus_t cublasGemmStridedBatchedEx(cublasHandle_t handle, cublasOperation_t transa,
                                          cublasOperation_t transb, int m, int n, int k,
                                          const void* alpha, const void* A, cudaDataType Atype,
                                          int lda, long long int strideA, const void* B,
                                          cudaDataType Btype, int ldb, long long int strideB,
                                          const void* beta, void* C, cudaDataType Ctype, int ldc,
                                          long long int strideC, int batchCount, int computeType,
                                          cublasGemmAlgo_t algo);

#define cublasCreate cublasCreate_v2
#define cublasDestroy cublasDestroy_v2
#define cublasGetVersion cublasGetVersion_v2
#define cublasSetStream cublasSetStream_v2
#define cublasGetStream cublasGetStream_v2
#define cublasSetPointerMode cublasSetPointerMode_v2
#define cublasGetPointerMode cublasGetPointerMode_v2
#define cublasSgemm cublasSgemm_v2
#define cublasSaxpy cublasSaxpy_v2
#define cublasScopy cublasScopy_v2
#define cublasSscal cublasSscal_v2
#define cublasSswap cublasSswap_v2
#define cublasSdot cublasSdot_v2
#define cublasSnrm2 cublasSnrm2_v2
#define cublasSasum cublasSasum_v2
#define cublasIsamax cublasIsamax_v2
#define cublasSgemv cublasSgemv_v2
#define cublasDaxpy cublasDaxpy_v2
#define cublasDcopy cublasDcopy_v2
#define cublasDscal cublasDscal_v2
#define cublasDswap cublasDswap_v2
#define cublasDdot cublasDdot_v2
#define cublasDnrm2 cublasDnrm2_v2
#define cublasDasum cublasDasum_v2
#define cublasIdamax cublasIdamax_v2
#define cublasDgemv cublasDgemv_v2
#define cublasDgemm cublasDgemm_v2

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_CUBLAS_V2_H_ */
