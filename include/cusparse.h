/*
 * cusparse.h — C ABI of the B200-native CSR SpMV and SpMM.
 *
 * Drop-in for the MUDA cuSPARSE shim's hot path: names, argument lists and
 * numeric enum values follow libraries/sparse/include/cusparse.h of the
 * reference (enums cusparse.h:20-81, declarations cusparse.h:108-156).  Enums
 * are int-width; cudaDataType_t comes from the CUDA toolkit's library_types.h
 * (same values as the reference's private copy).
 *
 * Conventions kept from the reference (libraries/sparse/src/cusparse_ops.mm):
 *   - alpha and beta are always read as host float* (cusparse_ops.mm:136-137);
 *   - beta == 0 means y is not read (kernel prev = 0);
 *   - CSR indices are int32 only (cusparse_descriptors.mm:143-145), base 0 or 1;
 *   - cusparseSpMV_bufferSize reports 0 bytes (cusparse_ops.mm:67).
 */
#ifndef MUDA_B200_CUSPARSE_H_
#define MUDA_B200_CUSPARSE_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>
#include <library_types.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  CUSPARSE_STATUS_SUCCESS = 0,
  CUSPARSE_STATUS_NOT_INITIALIZED = 1,
  CUSPARSE_STATUS_ALLOC_FAILED = 2,
  CUSPARSE_STATUS_INVALID_VALUE = 3,
  CUSPARSE_STATUS_ARCH_MISMATCH = 4,
  CUSPARSE_STATUS_MAPPING_ERROR = 5,
  CUSPARSE_STATUS_EXECUTION_FAILED = 6,
  CUSPARSE_STATUS_INTERNAL_ERROR = 7,
  CUSPARSE_STATUS_MATRIX_TYPE_NOT_SUPPORTED = 8,
  CUSPARSE_STATUS_ZERO_PIVOT = 9,
  CUSPARSE_STATUS_NOT_SUPPORTED = 10,
  CUSPARSE_STATUS_INSUFFICIENT_RESOURCES = 11
} cusparseStatus_t;

typedef enum {
  CUSPARSE_OPERATION_NON_TRANSPOSE = 0,
  CUSPARSE_OPERATION_TRANSPOSE = 1,
  CUSPARSE_OPERATION_CONJUGATE_TRANSPOSE = 2
} cusparseOperation_t;

typedef enum {
  CUSPARSE_INDEX_16U = 1,
  CUSPARSE_INDEX_32I = 2,
  CUSPARSE_INDEX_64I = 3
} cusparseIndexType_t;

typedef enum { CUSPARSE_INDEX_BASE_ZERO = 0, CUSPARSE_INDEX_BASE_ONE = 1 } cusparseIndexBase_t;

typedef enum {
  CUSPARSE_SPMV_ALG_DEFAULT = 0,
  CUSPARSE_SPMV_CSR_ALG1 = 2,
  CUSPARSE_SPMV_CSR_ALG2 = 3
} cusparseSpMVAlg_t;

/* reference cusparse.h:64 and :78-82 */
typedef enum { CUSPARSE_ORDER_COL = 1, CUSPARSE_ORDER_ROW = 2 } cusparseOrder_t;

typedef enum {
  CUSPARSE_SPMM_ALG_DEFAULT = 0,
  CUSPARSE_SPMM_CSR_ALG1 = 1,
  CUSPARSE_SPMM_CSR_ALG2 = 2
} cusparseSpMMAlg_t;

struct cusparseContext;
struct cusparseSpMatDescr;
struct cusparseDnVecDescr;
struct cusparseDnMatDescr;
typedef struct cusparseContext* cusparseHandle_t;
typedef struct cusparseSpMatDescr* cusparseSpMatDescr_t;
typedef struct cusparseDnVecDescr* cusparseDnVecDescr_t;
typedef struct cusparseDnMatDescr* cusparseDnMatDescr_t;

/* Context — reference cusparse_descriptors.mm:46-130 */
cusparseStatus_t cusparseCreate(cusparseHandle_t* handle);
cusparseStatus_t cusparseDestroy(cusparseHandle_t handle);
cusparseStatus_t cusparseGetVersion(cusparseHandle_t handle, int* version);
cusparseStatus_t cusparseSetStream(cusparseHandle_t handle, cudaStream_t streamId);
cusparseStatus_t cusparseGetStream(cusparseHandle_t handle, cudaStream_t* streamId);
const char* cusparseGetErrorName(cusparseStatus_t status);
const char* cusparseGetErrorString(cusparseStatus_t status);

/* Descriptors — reference cusparse_descriptors.mm:134-194 */
cusparseStatus_t cusparseCreateCsr(cusparseSpMatDescr_t* spMatDescr, int64_t rows, int64_t cols,
                                   int64_t nnz, void* csrRowOffsets, void* csrColInd,
                                   void* csrValues, cusparseIndexType_t csrRowOffsetsType,
                                   cusparseIndexType_t csrColIndType, cusparseIndexBase_t idxBase,
                                   cudaDataType valueType);
cusparseStatus_t cusparseDestroySpMat(cusparseSpMatDescr_t spMatDescr);
cusparseStatus_t cusparseCreateDnVec(cusparseDnVecDescr_t* dnVecDescr, int64_t size, void* values,
                                     cudaDataType valueType);
cusparseStatus_t cusparseDestroyDnVec(cusparseDnVecDescr_t dnVecDescr);
/* Dense matrices — reference cusparse_descriptors.mm:196-228: ld >= rows (column
 * order) or >= cols (row order), at least 1. */
cusparseStatus_t cusparseCreateDnMat(cusparseDnMatDescr_t* dnMatDescr, int64_t rows, int64_t cols,
                                     int64_t ld, void* values, cudaDataType valueType,
                                     cusparseOrder_t order);
cusparseStatus_t cusparseDestroyDnMat(cusparseDnMatDescr_t dnMatDescr);

/* SpMV — reference cusparse_ops.mm:44-211.  opA TRANSPOSE computes
 * alpha * A^T * x + beta * y by atomic accumulation (summation order unspecified,
 * as in the reference's own fp32 path); fp16 values and vectors accumulate in fp32. */
cusparseStatus_t cusparseSpMV_bufferSize(cusparseHandle_t handle, cusparseOperation_t opA,
                                         const void* alpha, cusparseSpMatDescr_t matA,
                                         cusparseDnVecDescr_t vecX, const void* beta,
                                         cusparseDnVecDescr_t vecY, cudaDataType computeType,
                                         cusparseSpMVAlg_t alg, size_t* bufferSize);
cusparseStatus_t cusparseSpMV(cusparseHandle_t handle, cusparseOperation_t opA, const void* alpha,
                              cusparseSpMatDescr_t matA, cusparseDnVecDescr_t vecX,
                              const void* beta, cusparseDnVecDescr_t vecY, cudaDataType computeType,
                              cusparseSpMVAlg_t alg, void* externalBuffer);

/* SpMM — reference cusparse_ops.mm:213-372: C = alpha * op(A) * op(B) + beta * C,
 * fp32 only, buffer size 0.  opA NON_TRANSPOSE reproduces the reference's
 * per-output arithmetic exactly; opA TRANSPOSE accumulates atomically. */
cusparseStatus_t cusparseSpMM_bufferSize(cusparseHandle_t handle, cusparseOperation_t opA,
                                         cusparseOperation_t opB, const void* alpha,
                                         cusparseSpMatDescr_t matA, cusparseDnMatDescr_t matB,
                                         const void* beta, cusparseDnMatDescr_t matC,
                                         cudaDataType computeType, cusparseSpMMAlg_t alg,
                                         size_t* bufferSize);
cusparseStatus_t cusparseSpMM(cusparseHandle_t handle, cusparseOperation_t opA,
                              cusparseOperation_t opB, const void* alpha, cusparseSpMatDescr_t matA,
                              cusparseDnMatDescr_t matB, const void* beta,
                              cusparseDnMatDescr_t matC, cudaDataType computeType,
                              cusparseSpMMAlg_t alg, void* externalBuffer);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_CUSPARSE_H_ */
