// cusparse_api.cpp — cuSPARSE C ABI: handle, CSR / dense-vector descriptors, SpMV.
//
// Mirrors libraries/sparse/src/cusparse_descriptors.mm and cusparse_ops.mm of the
// reference: same entry points, validation order and status codes; alpha and
// beta are host floats (cusparse_ops.mm:136-137); the buffer size is 0
// (cusparse_ops.mm:67).  Every array span is checked against its allocation
// before the kernel is launched.
#pragma GCC visibility push(default)
#include "cusparse.h"
#pragma GCC visibility pop

#include <cuda_runtime_api.h>

#include <cstdint>
#include <memory>
#include <mutex>

#include "common/device.hpp"
#include "common/registry.hpp"
#include "sparse/spmv.hpp"

namespace {

using mb200::ObjKind;
using mb200::Registry;

constexpr int kCusparseVersion = 12000;

struct SparseContext {
  std::mutex mu;
  cudaStream_t stream = nullptr;
};

struct CsrDesc {
  std::int64_t rows = 0, cols = 0, nnz = 0;
  void* row_offsets = nullptr;
  void* col_ind = nullptr;
  void* values = nullptr;
  cusparseIndexBase_t base = CUSPARSE_INDEX_BASE_ZERO;
  cudaDataType value_type = CUDA_R_32F;
};

struct DnVecDesc {
  std::int64_t size = 0;
  void* values = nullptr;
  cudaDataType value_type = CUDA_R_32F;
};

Registry<SparseContext, ObjKind::kSparseHandle>& handles() {
  static Registry<SparseContext, ObjKind::kSparseHandle> r;
  return r;
}
Registry<CsrDesc, ObjKind::kSparseCsr>& mats() {
  static Registry<CsrDesc, ObjKind::kSparseCsr> r;
  return r;
}
Registry<DnVecDesc, ObjKind::kSparseDnVec>& vecs() {
  static Registry<DnVecDesc, ObjKind::kSparseDnVec> r;
  return r;
}

// The reference accepts fp32 and fp16 value arrays (cusparse_descriptors.mm:13-15).
bool supported_value_type(cudaDataType t) { return t == CUDA_R_32F || t == CUDA_R_16F; }

struct Operands {
  std::shared_ptr<SparseContext> ctx;
  std::shared_ptr<CsrDesc> a;
  std::shared_ptr<DnVecDesc> x, y;
};

// Shared checks of cusparseSpMV_bufferSize / cusparseSpMV (cusparse_ops.mm:44-97).
cusparseStatus_t resolve(cusparseHandle_t handle, cusparseOperation_t op, cusparseSpMatDescr_t matA,
                         cusparseDnVecDescr_t vecX, cusparseDnVecDescr_t vecY, Operands* o) {
  o->ctx = handles().get(handle);
  if (!o->ctx) return CUSPARSE_STATUS_NOT_INITIALIZED;
  o->a = mats().get(matA);
  o->x = vecs().get(vecX);
  o->y = vecs().get(vecY);
  if (!o->a || !o->x || !o->y) return CUSPARSE_STATUS_INVALID_VALUE;
  const bool n = (op == CUSPARSE_OPERATION_NON_TRANSPOSE);
  const std::int64_t ex = n ? o->a->cols : o->a->rows;
  const std::int64_t ey = n ? o->a->rows : o->a->cols;
  if (o->x->size != ex || o->y->size != ey) return CUSPARSE_STATUS_INVALID_VALUE;
  return CUSPARSE_STATUS_SUCCESS;
}

}  // namespace

extern "C" {

cusparseStatus_t cusparseCreate(cusparseHandle_t* handle) {
  if (handle == nullptr) return CUSPARSE_STATUS_INVALID_VALUE;
  auto h = handles().add<cusparseHandle_t>(std::make_shared<SparseContext>());
  if (h == nullptr) return CUSPARSE_STATUS_ALLOC_FAILED;
  *handle = h;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseDestroy(cusparseHandle_t handle) {
  return handles().take(handle) ? CUSPARSE_STATUS_SUCCESS : CUSPARSE_STATUS_NOT_INITIALIZED;
}

cusparseStatus_t cusparseGetVersion(cusparseHandle_t handle, int* version) {
  if (version == nullptr) return CUSPARSE_STATUS_INVALID_VALUE;
  if (handle != nullptr && !handles().get(handle)) return CUSPARSE_STATUS_NOT_INITIALIZED;
  *version = kCusparseVersion;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseSetStream(cusparseHandle_t handle, cudaStream_t streamId) {
  auto h = handles().get(handle);
  if (!h) return CUSPARSE_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> g(h->mu);
  h->stream = streamId;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseGetStream(cusparseHandle_t handle, cudaStream_t* streamId) {
  if (streamId == nullptr) return CUSPARSE_STATUS_INVALID_VALUE;
  auto h = handles().get(handle);
  if (!h) return CUSPARSE_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> g(h->mu);
  *streamId = h->stream;
  return CUSPARSE_STATUS_SUCCESS;
}

const char* cusparseGetErrorName(cusparseStatus_t status) {
  switch (status) {
    case CUSPARSE_STATUS_SUCCESS: return "CUSPARSE_STATUS_SUCCESS";
    case CUSPARSE_STATUS_NOT_INITIALIZED: return "CUSPARSE_STATUS_NOT_INITIALIZED";
    case CUSPARSE_STATUS_ALLOC_FAILED: return "CUSPARSE_STATUS_ALLOC_FAILED";
    case CUSPARSE_STATUS_INVALID_VALUE: return "CUSPARSE_STATUS_INVALID_VALUE";
    case CUSPARSE_STATUS_ARCH_MISMATCH: return "CUSPARSE_STATUS_ARCH_MISMATCH";
    case CUSPARSE_STATUS_MAPPING_ERROR: return "CUSPARSE_STATUS_MAPPING_ERROR";
    case CUSPARSE_STATUS_EXECUTION_FAILED: return "CUSPARSE_STATUS_EXECUTION_FAILED";
    case CUSPARSE_STATUS_INTERNAL_ERROR: return "CUSPARSE_STATUS_INTERNAL_ERROR";
    case CUSPARSE_STATUS_MATRIX_TYPE_NOT_SUPPORTED:
      return "CUSPARSE_STATUS_MATRIX_TYPE_NOT_SUPPORTED";
    case CUSPARSE_STATUS_ZERO_PIVOT: return "CUSPARSE_STATUS_ZERO_PIVOT";
    case CUSPARSE_STATUS_NOT_SUPPORTED: return "CUSPARSE_STATUS_NOT_SUPPORTED";
    case CUSPARSE_STATUS_INSUFFICIENT_RESOURCES: return "CUSPARSE_STATUS_INSUFFICIENT_RESOURCES";
  }
  return "CUSPARSE_STATUS_UNKNOWN";
}

const char* cusparseGetErrorString(cusparseStatus_t status) { return cusparseGetErrorName(status); }

cusparseStatus_t cusparseCreateCsr(cusparseSpMatDescr_t* spMatDescr, int64_t rows, int64_t cols,
                                   int64_t nnz, void* csrRowOffsets, void* csrColInd,
                                   void* csrValues, cusparseIndexType_t csrRowOffsetsType,
                                   cusparseIndexType_t csrColIndType, cusparseIndexBase_t idxBase,
                                   cudaDataType valueType) {
  if (spMatDescr == nullptr || rows < 0 || cols < 0 || nnz < 0 || csrRowOffsets == nullptr ||
      (nnz > 0 && (csrColInd == nullptr || csrValues == nullptr)))
    return CUSPARSE_STATUS_INVALID_VALUE;
  if (csrRowOffsetsType != CUSPARSE_INDEX_32I || csrColIndType != CUSPARSE_INDEX_32I)
    return CUSPARSE_STATUS_NOT_SUPPORTED;
  if (idxBase != CUSPARSE_INDEX_BASE_ZERO && idxBase != CUSPARSE_INDEX_BASE_ONE)
    return CUSPARSE_STATUS_INVALID_VALUE;
  if (!supported_value_type(valueType)) return CUSPARSE_STATUS_NOT_SUPPORTED;
  // int32 offsets address at most 2^31 - 1 stored entries
  if (nnz > INT32_MAX || rows >= INT32_MAX || cols > INT32_MAX)
    return CUSPARSE_STATUS_INVALID_VALUE;
  auto d = std::make_shared<CsrDesc>();
  d->rows = rows;
  d->cols = cols;
  d->nnz = nnz;
  d->row_offsets = csrRowOffsets;
  d->col_ind = csrColInd;
  d->values = csrValues;
  d->base = idxBase;
  d->value_type = valueType;
  auto h = mats().add<cusparseSpMatDescr_t>(std::move(d));
  if (h == nullptr) return CUSPARSE_STATUS_ALLOC_FAILED;
  *spMatDescr = h;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseDestroySpMat(cusparseSpMatDescr_t spMatDescr) {
  return mats().take(spMatDescr) ? CUSPARSE_STATUS_SUCCESS : CUSPARSE_STATUS_INVALID_VALUE;
}

cusparseStatus_t cusparseCreateDnVec(cusparseDnVecDescr_t* dnVecDescr, int64_t size, void* values,
                                     cudaDataType valueType) {
  if (dnVecDescr == nullptr || size < 0 || (size > 0 && values == nullptr))
    return CUSPARSE_STATUS_INVALID_VALUE;
  if (!supported_value_type(valueType)) return CUSPARSE_STATUS_NOT_SUPPORTED;
  auto d = std::make_shared<DnVecDesc>();
  d->size = size;
  d->values = values;
  d->value_type = valueType;
  auto h = vecs().add<cusparseDnVecDescr_t>(std::move(d));
  if (h == nullptr) return CUSPARSE_STATUS_ALLOC_FAILED;
  *dnVecDescr = h;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseDestroyDnVec(cusparseDnVecDescr_t dnVecDescr) {
  return vecs().take(dnVecDescr) ? CUSPARSE_STATUS_SUCCESS : CUSPARSE_STATUS_INVALID_VALUE;
}

cusparseStatus_t cusparseSpMV_bufferSize(cusparseHandle_t handle, cusparseOperation_t opA,
                                         const void* alpha, cusparseSpMatDescr_t matA,
                                         cusparseDnVecDescr_t vecX, const void* beta,
                                         cusparseDnVecDescr_t vecY, cudaDataType computeType,
                                         cusparseSpMVAlg_t alg, size_t* bufferSize) {
  (void)computeType;
  (void)alg;
  if (bufferSize == nullptr || alpha == nullptr || beta == nullptr)
    return CUSPARSE_STATUS_INVALID_VALUE;
  Operands o;
  const cusparseStatus_t st = resolve(handle, opA, matA, vecX, vecY, &o);
  if (st != CUSPARSE_STATUS_SUCCESS) return st;
  *bufferSize = 0;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseSpMV(cusparseHandle_t handle, cusparseOperation_t opA, const void* alpha,
                              cusparseSpMatDescr_t matA, cusparseDnVecDescr_t vecX,
                              const void* beta, cusparseDnVecDescr_t vecY, cudaDataType computeType,
                              cusparseSpMVAlg_t alg, void* externalBuffer) {
  (void)computeType;
  (void)alg;
  (void)externalBuffer;
  if (alpha == nullptr || beta == nullptr) return CUSPARSE_STATUS_INVALID_VALUE;
  Operands o;
  cusparseStatus_t st = resolve(handle, opA, matA, vecX, vecY, &o);
  if (st != CUSPARSE_STATUS_SUCCESS) return st;
  if (o.a->value_type != o.x->value_type || o.a->value_type != o.y->value_type)
    return CUSPARSE_STATUS_NOT_SUPPORTED;
  const std::int64_t ey = (opA == CUSPARSE_OPERATION_NON_TRANSPOSE) ? o.a->rows : o.a->cols;
  if (ey == 0) return CUSPARSE_STATUS_SUCCESS;
  // The B200 path covers the non-transposed fp32 product named by the hot path;
  // transposed and fp16 products are not implemented.
  if (opA != CUSPARSE_OPERATION_NON_TRANSPOSE) return CUSPARSE_STATUS_NOT_SUPPORTED;
  if (o.a->value_type != CUDA_R_32F) return CUSPARSE_STATUS_NOT_SUPPORTED;
  const auto rows = static_cast<std::size_t>(o.a->rows);
  const auto nnz = static_cast<std::size_t>(o.a->nnz);
  if (!mb200::device_span_ok(o.a->row_offsets, (rows + 1) * 4) ||
      !mb200::device_span_ok(o.a->col_ind, nnz * 4) ||
      !mb200::device_span_ok(o.a->values, nnz * 4) ||
      !mb200::device_span_ok(o.x->values, static_cast<std::size_t>(o.x->size) * 4) ||
      !mb200::device_span_ok(o.y->values, static_cast<std::size_t>(o.y->size) * 4))
    return CUSPARSE_STATUS_INVALID_VALUE;
  if (!mb200::aligned_to(o.a->row_offsets, 4) || !mb200::aligned_to(o.a->col_ind, 4) ||
      !mb200::aligned_to(o.a->values, 4) || !mb200::aligned_to(o.x->values, 4) ||
      !mb200::aligned_to(o.y->values, 4))
    return CUSPARSE_STATUS_INVALID_VALUE;
  mb200::sparse::CsrView a{o.a->rows,
                           o.a->cols,
                           o.a->nnz,
                           static_cast<const std::int32_t*>(o.a->row_offsets),
                           static_cast<const std::int32_t*>(o.a->col_ind),
                           static_cast<const float*>(o.a->values),
                           o.a->base == CUSPARSE_INDEX_BASE_ONE ? 1 : 0};
  const float al = *static_cast<const float*>(alpha);
  const float be = *static_cast<const float*>(beta);
  cudaStream_t stream;
  {
    std::lock_guard<std::mutex> g(o.ctx->mu);
    stream = o.ctx->stream;
  }
  const cudaError_t e = mb200::sparse::launch_spmv_csr(
      a, static_cast<const float*>(o.x->values), static_cast<float*>(o.y->values), al, be, stream);
  return e == cudaSuccess ? CUSPARSE_STATUS_SUCCESS : CUSPARSE_STATUS_EXECUTION_FAILED;
}

}  // extern "C"
