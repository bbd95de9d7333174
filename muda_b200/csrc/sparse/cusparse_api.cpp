// cusparse_api.cpp — cuSPARSE C ABI: handle, CSR / dense descriptors, SpMV, SpMM.
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
#include "common/lru.hpp"
#include "common/registry.hpp"
#include "sparse/spmv.hpp"

namespace {

using mb200::ObjKind;
using mb200::Registry;

constexpr int kCusparseVersion = 12000;

struct SparseContext {
  std::mutex mu;
  cudaStream_t stream = nullptr;
  // device scratch (fp32 sums of the fp16 transposed product, the SpMM row
  // scheduler): held under ws_mu for the call, reuse ordered after the previous
  // call's last use by ws_done
  std::mutex ws_mu;
  std::shared_ptr<mb200::DeviceBuffer> ws;
  cudaEvent_t ws_done = nullptr;
  ~SparseContext() {
    if (ws_done != nullptr) (void)cudaEventDestroy(ws_done);
  }
};

// Runs launch(scratch pointer) with at least `need` bytes of the handle's scratch,
// after the previous user of the scratch in stream order (outside stream capture;
// a captured call orders by the capture itself).
template <class Launch>
cudaError_t with_scratch(SparseContext& ctx, cudaStream_t stream, std::size_t need,
                         Launch&& launch) {
  std::lock_guard<std::mutex> g(ctx.ws_mu);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) cap = cudaStreamCaptureStatusNone;
  const bool ordered = cap == cudaStreamCaptureStatusNone;
  if (ordered && ctx.ws_done != nullptr) {
    const cudaError_t w = cudaStreamWaitEvent(stream, ctx.ws_done, 0);
    if (w != cudaSuccess) return w;
  }
  if (!ctx.ws || ctx.ws->bytes < need || ctx.ws->device != mb200::current_device()) {
    ctx.ws.reset();
    ctx.ws = mb200::DeviceBuffer::make(need);
    if (!ctx.ws) return cudaErrorMemoryAllocation;
  }
  cudaError_t e = launch(ctx.ws->ptr);
  if (e == cudaSuccess && ordered) {
    if (ctx.ws_done == nullptr &&
        cudaEventCreateWithFlags(&ctx.ws_done, cudaEventDisableTiming) != cudaSuccess) {
      ctx.ws_done = nullptr;
      return cudaErrorUnknown;
    }
    e = cudaEventRecord(ctx.ws_done, stream);
  }
  return e;
}

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

struct DnMatDesc {
  std::int64_t rows = 0, cols = 0, ld = 1;
  void* values = nullptr;
  cudaDataType value_type = CUDA_R_32F;
  cusparseOrder_t order = CUSPARSE_ORDER_COL;
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
Registry<DnMatDesc, ObjKind::kSparseDnMat>& dmats() {
  static Registry<DnMatDesc, ObjKind::kSparseDnMat> r;
  return r;
}

// Elements a dense matrix spans in memory (cusparse_ops.mm:24-34).
std::size_t dense_span(const DnMatDesc& m) {
  if (m.rows <= 0 || m.cols <= 0) return 0;
  return (m.order == CUSPARSE_ORDER_COL)
             ? static_cast<std::size_t>(m.ld) * static_cast<std::size_t>(m.cols - 1) +
                   static_cast<std::size_t>(m.rows)
             : static_cast<std::size_t>(m.ld) * static_cast<std::size_t>(m.rows - 1) +
                   static_cast<std::size_t>(m.cols);
}

std::size_t value_bytes(cudaDataType t) { return t == CUDA_R_16F ? 2 : 4; }

// The CSR arrays of `a` lie in device allocations and are aligned to their types.
bool csr_arrays_ok(const CsrDesc& a) {
  const auto rows = static_cast<std::size_t>(a.rows);
  const auto nnz = static_cast<std::size_t>(a.nnz);
  const std::size_t vb = value_bytes(a.value_type);
  if (!mb200::device_span_ok(a.row_offsets, (rows + 1) * 4) ||
      !mb200::aligned_to(a.row_offsets, 4))
    return false;
  if (nnz == 0) return true;
  return mb200::device_span_ok(a.col_ind, nnz * 4) && mb200::device_span_ok(a.values, nnz * vb) &&
         mb200::aligned_to(a.col_ind, 4) && mb200::aligned_to(a.values, vb);
}

mb200::sparse::CsrView view_of(const CsrDesc& a) {
  return mb200::sparse::CsrView{a.rows,
                                a.cols,
                                a.nnz,
                                static_cast<const std::int32_t*>(a.row_offsets),
                                static_cast<const std::int32_t*>(a.col_ind),
                                a.values,
                                a.base == CUSPARSE_INDEX_BASE_ONE ? 1 : 0};
}

cudaStream_t stream_of(SparseContext& ctx) {
  std::lock_guard<std::mutex> g(ctx.mu);
  return ctx.stream;
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
  const bool trans = opA != CUSPARSE_OPERATION_NON_TRANSPOSE;
  const std::int64_t ey = trans ? o.a->cols : o.a->rows;
  if (ey == 0) return CUSPARSE_STATUS_SUCCESS;
  const std::size_t vb = value_bytes(o.a->value_type);
  if (!csr_arrays_ok(*o.a) ||
      !mb200::device_span_ok(o.x->values, static_cast<std::size_t>(o.x->size) * vb) ||
      !mb200::device_span_ok(o.y->values, static_cast<std::size_t>(o.y->size) * vb) ||
      !mb200::aligned_to(o.x->values, vb) || !mb200::aligned_to(o.y->values, vb))
    return CUSPARSE_STATUS_INVALID_VALUE;
  const auto a = view_of(*o.a);
  const auto vt = o.a->value_type == CUDA_R_16F ? mb200::sparse::Value::kF16
                                                : mb200::sparse::Value::kF32;
  const float al = *static_cast<const float*>(alpha);
  const float be = *static_cast<const float*>(beta);
  const cudaStream_t stream = stream_of(*o.ctx);
  cudaError_t e = cudaSuccess;
  if (!trans) {
    // the entry-range kernel's per-range partial sums live in the handle's scratch
    const std::size_t need = mb200::sparse::spmv_csr_scratch_bytes(a);
    if (need == 0) {
      e = mb200::sparse::launch_spmv_csr(a, vt, o.x->values, o.y->values, al, be, nullptr,
                                         stream);
    } else {
      e = with_scratch(*o.ctx, stream, need, [&](void* ws) {
        return mb200::sparse::launch_spmv_csr(a, vt, o.x->values, o.y->values, al, be, ws,
                                              stream);
      });
      if (e == cudaErrorMemoryAllocation) return CUSPARSE_STATUS_ALLOC_FAILED;
    }
  } else if (vt == mb200::sparse::Value::kF32) {
    e = mb200::sparse::launch_spmv_csr_t(a, vt, o.x->values, o.y->values, al, be, nullptr,
                                         stream);
  } else {
    // fp16: fp32 sums in the handle's scratch, reused in stream order across calls
    const std::size_t need = static_cast<std::size_t>(o.a->cols) * sizeof(float);
    e = with_scratch(*o.ctx, stream, need, [&](void* ws) {
      return mb200::sparse::launch_spmv_csr_t(a, vt, o.x->values, o.y->values, al, be,
                                              static_cast<float*>(ws), stream);
    });
    if (e == cudaErrorMemoryAllocation) return CUSPARSE_STATUS_ALLOC_FAILED;
  }
  return e == cudaSuccess ? CUSPARSE_STATUS_SUCCESS : CUSPARSE_STATUS_EXECUTION_FAILED;
}

// cusparse_descriptors.mm:196-223
cusparseStatus_t cusparseCreateDnMat(cusparseDnMatDescr_t* dnMatDescr, int64_t rows, int64_t cols,
                                     int64_t ld, void* values, cudaDataType valueType,
                                     cusparseOrder_t order) {
  if (dnMatDescr == nullptr || rows < 0 || cols < 0 || (rows > 0 && cols > 0 && values == nullptr))
    return CUSPARSE_STATUS_INVALID_VALUE;
  if (order != CUSPARSE_ORDER_COL && order != CUSPARSE_ORDER_ROW)
    return CUSPARSE_STATUS_INVALID_VALUE;
  const std::int64_t min_ld =
      (order == CUSPARSE_ORDER_COL) ? (rows > 1 ? rows : 1) : (cols > 1 ? cols : 1);
  if (ld < min_ld) return CUSPARSE_STATUS_INVALID_VALUE;
  if (!supported_value_type(valueType)) return CUSPARSE_STATUS_NOT_SUPPORTED;
  auto d = std::make_shared<DnMatDesc>();
  d->rows = rows;
  d->cols = cols;
  d->ld = ld;
  d->values = values;
  d->value_type = valueType;
  d->order = order;
  auto h = dmats().add<cusparseDnMatDescr_t>(std::move(d));
  if (h == nullptr) return CUSPARSE_STATUS_ALLOC_FAILED;
  *dnMatDescr = h;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseDestroyDnMat(cusparseDnMatDescr_t dnMatDescr) {
  return dmats().take(dnMatDescr) ? CUSPARSE_STATUS_SUCCESS : CUSPARSE_STATUS_INVALID_VALUE;
}

}  // extern "C"

namespace {

struct MmOperands {
  std::shared_ptr<SparseContext> ctx;
  std::shared_ptr<CsrDesc> a;
  std::shared_ptr<DnMatDesc> b, c;
  std::int64_t out_rows = 0, ncols = 0;
};

// Shared checks of cusparseSpMM_bufferSize / cusparseSpMM (cusparse_ops.mm:213-273):
// the handle, the descriptors, then op(A) (m x k) * op(B) (k x n) against C (m x n).
cusparseStatus_t resolve_mm(cusparseHandle_t handle, cusparseOperation_t opA,
                            cusparseOperation_t opB, cusparseSpMatDescr_t matA,
                            cusparseDnMatDescr_t matB, cusparseDnMatDescr_t matC,
                            bool check_types, MmOperands* o) {
  o->ctx = handles().get(handle);
  if (!o->ctx) return CUSPARSE_STATUS_NOT_INITIALIZED;
  o->a = mats().get(matA);
  o->b = dmats().get(matB);
  o->c = dmats().get(matC);
  if (!o->a || !o->b || !o->c) return CUSPARSE_STATUS_INVALID_VALUE;
  if (check_types && (o->a->value_type != CUDA_R_32F || o->b->value_type != CUDA_R_32F ||
                      o->c->value_type != CUDA_R_32F))
    return CUSPARSE_STATUS_NOT_SUPPORTED;
  const bool ta = opA != CUSPARSE_OPERATION_NON_TRANSPOSE;
  const bool tb = opB != CUSPARSE_OPERATION_NON_TRANSPOSE;
  const std::int64_t ar = ta ? o->a->cols : o->a->rows, ac = ta ? o->a->rows : o->a->cols;
  const std::int64_t br = tb ? o->b->cols : o->b->rows, bc = tb ? o->b->rows : o->b->cols;
  if (ac != br || o->c->rows != ar || o->c->cols != bc) return CUSPARSE_STATUS_INVALID_VALUE;
  o->out_rows = ar;
  o->ncols = bc;
  return CUSPARSE_STATUS_SUCCESS;
}

}  // namespace

extern "C" {

cusparseStatus_t cusparseSpMM_bufferSize(cusparseHandle_t handle, cusparseOperation_t opA,
                                         cusparseOperation_t opB, const void* alpha,
                                         cusparseSpMatDescr_t matA, cusparseDnMatDescr_t matB,
                                         const void* beta, cusparseDnMatDescr_t matC,
                                         cudaDataType computeType, cusparseSpMMAlg_t alg,
                                         size_t* bufferSize) {
  (void)computeType;
  (void)alg;
  if (bufferSize == nullptr || alpha == nullptr || beta == nullptr)
    return CUSPARSE_STATUS_INVALID_VALUE;
  MmOperands o;
  const cusparseStatus_t st = resolve_mm(handle, opA, opB, matA, matB, matC, false, &o);
  if (st != CUSPARSE_STATUS_SUCCESS) return st;
  *bufferSize = 0;
  return CUSPARSE_STATUS_SUCCESS;
}

cusparseStatus_t cusparseSpMM(cusparseHandle_t handle, cusparseOperation_t opA,
                              cusparseOperation_t opB, const void* alpha, cusparseSpMatDescr_t matA,
                              cusparseDnMatDescr_t matB, const void* beta,
                              cusparseDnMatDescr_t matC, cudaDataType computeType,
                              cusparseSpMMAlg_t alg, void* externalBuffer) {
  (void)computeType;
  (void)alg;
  (void)externalBuffer;
  if (alpha == nullptr || beta == nullptr) return CUSPARSE_STATUS_INVALID_VALUE;
  MmOperands o;
  const cusparseStatus_t st = resolve_mm(handle, opA, opB, matA, matB, matC, true, &o);
  if (st != CUSPARSE_STATUS_SUCCESS) return st;
  if (o.out_rows == 0 || o.ncols == 0) return CUSPARSE_STATUS_SUCCESS;
  if (!csr_arrays_ok(*o.a) ||
      !mb200::device_span_ok(o.b->values, dense_span(*o.b) * sizeof(float)) ||
      !mb200::device_span_ok(o.c->values, dense_span(*o.c) * sizeof(float)) ||
      !mb200::aligned_to(o.b->values, 4) || !mb200::aligned_to(o.c->values, 4))
    return CUSPARSE_STATUS_INVALID_VALUE;
  const mb200::sparse::DenseView b{static_cast<float*>(o.b->values), o.b->ld,
                                   o.b->order == CUSPARSE_ORDER_COL,
                                   opB != CUSPARSE_OPERATION_NON_TRANSPOSE};
  const mb200::sparse::DenseView c{static_cast<float*>(o.c->values), o.c->ld,
                                   o.c->order == CUSPARSE_ORDER_COL, false};
  const cudaStream_t stream = stream_of(*o.ctx);
  const cudaError_t e = with_scratch(*o.ctx, stream, mb200::sparse::kSpmmSchedBytes, [&](void* ws) {
    const mb200::sparse::SpmmSched sc{static_cast<unsigned*>(ws),
                                      reinterpret_cast<int*>(static_cast<char*>(ws) +
                                                           mb200::sparse::kSpmmSchedHeader),
                                      mb200::sparse::kSpmmLongCap};
    return mb200::sparse::launch_spmm_csr(
        view_of(*o.a), opA != CUSPARSE_OPERATION_NON_TRANSPOSE, b, c, o.ncols,
        *static_cast<const float*>(alpha), *static_cast<const float*>(beta), &sc, stream);
  });
  if (e == cudaErrorMemoryAllocation) return CUSPARSE_STATUS_ALLOC_FAILED;
  return e == cudaSuccess ? CUSPARSE_STATUS_SUCCESS : CUSPARSE_STATUS_EXECUTION_FAILED;
}

}  // extern "C"
