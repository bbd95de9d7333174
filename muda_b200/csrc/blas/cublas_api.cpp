// cublas_api.cpp — cuBLAS C ABI: handle state and the level-3 GEMM entry points.
//
// Mirrors libraries/blas/src/cublas_context.mm and cublas_level3.mm of the
// reference: the same entry points, argument checks (op, sizes, leading
// dimensions, null scalars) and status codes, column-major semantics, and the
// same GemmEx dispatch (fp32 / fp16 operands, the scalar type chosen by the
// compute type, cublas_level3.mm:544-608).  bf16 operands (CUDA_R_16BF) are an
// extension the reference lacks.  In device pointer mode the scalars are read
// by the kernel on the stream instead of synchronising the host
// (cublas_context.mm:72-75 synchronises).
//
// fp32 GEMMs run on the tensor cores in split-tf32 form (fp32-class accuracy,
// within 1.5 * 2^-20 relative per product) unless the math mode is
// CUBLAS_PEDANTIC_MATH, which keeps the FFMA kernel; the split operands live in
// a device workspace the handle owns and reuses (grown on demand, ordered after
// the previous call that used it by an event, so a cublasSetStream between calls
// stays safe).
#pragma GCC visibility push(default)
#include "cublas_v2.h"
#pragma GCC visibility pop

#include <cuda_runtime_api.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>

#include "blas/geam.hpp"
#include "blas/dblas.hpp"
#include "blas/gemm.hpp"
#include "blas/level12.hpp"
#include "common/device.hpp"
#include "common/lru.hpp"
#include "common/registry.hpp"

namespace {

using mb200::blas::Elem;
using mb200::blas::GemmArgs;

constexpr int kCublasVersion = 12000;

struct BlasContext {
  std::mutex mu;
  cudaStream_t stream = nullptr;
  cublasPointerMode_t pointer_mode = CUBLAS_POINTER_MODE_HOST;
  cublasMath_t math_mode = CUBLAS_DEFAULT_MATH;
  // split-tf32 workspace: held under ws_mu for the whole call that uses it
  std::mutex ws_mu;
  std::shared_ptr<mb200::DeviceBuffer> ws;   // split-tf32 planes, gemv partial sums
  std::shared_ptr<mb200::DeviceBuffer> red;  // reduction scratch + result slot (zeroed once)
  cudaEvent_t ws_done = nullptr;  // recorded after the last call that used ws or red

  ~BlasContext() {
    if (ws_done != nullptr) (void)cudaEventDestroy(ws_done);
  }
};

// One call's use of the handle's device buffers: holds ws_mu for the call, orders
// the stream after the previous such call (an event, skipped while the stream is
// being captured into a graph) and records this call in done().
class BufferUse {
 public:
  BufferUse(BlasContext& ctx, cudaStream_t stream) : lk_(ctx.ws_mu), ctx_(ctx), stream_(stream) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) cap = cudaStreamCaptureStatusNone;
    ordered_ = cap == cudaStreamCaptureStatusNone;
    if (ordered_ && ctx.ws_done != nullptr)
      ok_ = cudaStreamWaitEvent(stream, ctx.ws_done, 0) == cudaSuccess;
  }
  BufferUse(const BufferUse&) = delete;
  BufferUse& operator=(const BufferUse&) = delete;

  bool ok() const { return ok_; }

  // The workspace, grown to `need` bytes (null when it cannot be had).
  void* workspace(std::size_t need) {
    const int dev = mb200::current_device();
    if (!ctx_.ws || ctx_.ws->bytes < need || ctx_.ws->device != dev) {
      ctx_.ws.reset();
      ctx_.ws = mb200::DeviceBuffer::make(need);
    }
    return ctx_.ws ? ctx_.ws->ptr : nullptr;
  }
  std::size_t workspace_bytes() const { return ctx_.ws ? ctx_.ws->bytes : 0; }

  // The reduction scratch (zero-filled on the stream when first allocated) and the
  // 16-byte result slot after it.
  void* reduction_scratch() {
    const int dev = mb200::current_device();
    if (!ctx_.red || ctx_.red->device != dev) {
      ctx_.red = mb200::DeviceBuffer::make(kSlot + 16);
      if (!ctx_.red) return nullptr;
      if (cudaMemsetAsync(ctx_.red->ptr, 0, kSlot + 16, stream_) != cudaSuccess) {
        ctx_.red.reset();
        return nullptr;
      }
    }
    return ctx_.red->ptr;
  }
  void* result_slot() { return static_cast<char*>(reduction_scratch()) + kSlot; }

  cudaError_t done() {
    if (!ordered_) return cudaSuccess;
    if (ctx_.ws_done == nullptr &&
        cudaEventCreateWithFlags(&ctx_.ws_done, cudaEventDisableTiming) != cudaSuccess) {
      ctx_.ws_done = nullptr;
      return cudaErrorUnknown;
    }
    return cudaEventRecord(ctx_.ws_done, stream_);
  }

 private:
  // one scratch serves the fp32 and the fp64 reductions (same counter word first)
  static std::size_t slot_offset() {
    const std::size_t a = mb200::blas::reduce_scratch_bytes();
    const std::size_t b = mb200::blas::dreduce_scratch_bytes();
    return ((a > b ? a : b) + 255) / 256 * 256;
  }
  const std::size_t kSlot = slot_offset();
  std::lock_guard<std::mutex> lk_;
  BlasContext& ctx_;
  cudaStream_t stream_;
  bool ordered_ = true;
  bool ok_ = true;
};

// fp32 GEMM on the tensor cores with the handle's workspace; cudaErrorNotSupported
// when the shape does not qualify or the workspace cannot be had.
cudaError_t run_tf32x3(BlasContext& ctx, const GemmArgs& g, cudaStream_t stream) {
  const std::size_t need = mb200::blas::gemm_tf32x3_workspace(g);
  if (need == 0) return cudaErrorNotSupported;
  BufferUse use(ctx, stream);
  if (!use.ok()) return cudaErrorUnknown;
  void* ws = use.workspace(need);
  if (ws == nullptr) return cudaErrorNotSupported;
  const cudaError_t e = mb200::blas::launch_gemm_tf32x3(g, ws, use.workspace_bytes(), stream);
  if (e != cudaSuccess) return e;
  return use.done();
}

using HandleTable = mb200::Registry<BlasContext, mb200::ObjKind::kBlasHandle>;
HandleTable& handles() {
  static HandleTable t;
  return t;
}

bool valid_op(cublasOperation_t op) {
  return op == CUBLAS_OP_N || op == CUBLAS_OP_T || op == CUBLAS_OP_C;
}

float half_bits_to_float(std::uint16_t h) {
  const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
  std::uint32_t exp = (h >> 10) & 0x1Fu;
  std::uint32_t man = h & 0x3FFu;
  std::uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      exp = 127 - 15 + 1;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --exp;
      }
      man &= 0x3FFu;
      bits = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// Elements from the first to the last addressed element of a rows x cols
// column-major matrix (cublas_level3.mm:233-240).
std::size_t span(int rows, int cols, std::int64_t ld) {
  if (rows <= 0 || cols <= 0) return 0;
  return static_cast<std::size_t>(ld) * static_cast<std::size_t>(cols - 1) +
         static_cast<std::size_t>(rows);
}

std::size_t batch_span(int rows, int cols, std::int64_t ld, std::int64_t stride, int batch) {
  const std::size_t one = span(rows, cols, ld);
  if (one == 0 || batch <= 0) return 0;
  const std::int64_t s = stride < 0 ? -stride : stride;
  return one + static_cast<std::size_t>(s) * static_cast<std::size_t>(batch - 1);
}

struct Scalars {
  bool device = false;
  float alpha = 0.0f, beta = 0.0f;
  const void* alpha_ptr = nullptr;
  const void* beta_ptr = nullptr;
};

// Validation shared by every GEMM entry point (cublas_level3.mm:515-531).
cublasStatus_t check_args(cublasOperation_t ta, cublasOperation_t tb, int m, int n, int k,
                          int lda, int ldb, int ldc, int batch, const void* alpha,
                          const void* beta) {
  if (!valid_op(ta) || !valid_op(tb) || m < 0 || n < 0 || k < 0 || batch < 0 ||
      alpha == nullptr || beta == nullptr)
    return CUBLAS_STATUS_INVALID_VALUE;
  const int min_lda = (ta == CUBLAS_OP_N) ? (m > 1 ? m : 1) : (k > 1 ? k : 1);
  const int min_ldb = (tb == CUBLAS_OP_N) ? (k > 1 ? k : 1) : (n > 1 ? n : 1);
  const int min_ldc = m > 1 ? m : 1;
  if (lda < min_lda || ldb < min_ldb || ldc < min_ldc) return CUBLAS_STATUS_INVALID_VALUE;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t run_gemm(BlasContext& ctx, Elem type, cublasOperation_t ta, cublasOperation_t tb,
                        int m, int n, int k, const void* alpha, bool half_scalars, const void* A,
                        int lda, long long sa, const void* B, int ldb, long long sb,
                        const void* beta, void* C, int ldc, long long sc, int batch) {
  cudaStream_t stream;
  cublasPointerMode_t mode;
  cublasMath_t math;
  {
    std::lock_guard<std::mutex> g(ctx.mu);
    stream = ctx.stream;
    mode = ctx.pointer_mode;
    math = ctx.math_mode;
  }
  if (m == 0 || n == 0 || batch == 0) return CUBLAS_STATUS_SUCCESS;
  GemmArgs g{};
  g.type = type;
  g.trans_a = (ta != CUBLAS_OP_N);
  g.trans_b = (tb != CUBLAS_OP_N);
  g.m = m;
  g.n = n;
  g.k = k;
  g.a = A;
  g.lda = lda;
  g.stride_a = sa;
  g.b = B;
  g.ldb = ldb;
  g.stride_b = sb;
  g.c = C;
  g.ldc = ldc;
  g.stride_c = sc;
  g.batch = batch;
  if (mode == CUBLAS_POINTER_MODE_DEVICE) {
    // 16-bit device scalars would need a conversion kernel; the kernels read fp32.
    if (half_scalars) return CUBLAS_STATUS_NOT_SUPPORTED;
    if (!mb200::device_span_ok(alpha, 4) || !mb200::device_span_ok(beta, 4))
      return CUBLAS_STATUS_INVALID_VALUE;
    g.alpha_dev = static_cast<const float*>(alpha);
    g.beta_dev = static_cast<const float*>(beta);
  } else if (half_scalars) {
    std::uint16_t ha, hb;
    std::memcpy(&ha, alpha, 2);
    std::memcpy(&hb, beta, 2);
    g.alpha = half_bits_to_float(ha);
    g.beta = half_bits_to_float(hb);
  } else {
    g.alpha = *static_cast<const float*>(alpha);
    g.beta = *static_cast<const float*>(beta);
  }
  const int es = (type == Elem::kF32) ? 4 : 2;
  const int a_rows = g.trans_a ? k : m, a_cols = g.trans_a ? m : k;
  const int b_rows = g.trans_b ? n : k, b_cols = g.trans_b ? k : n;
  if (k > 0 && (!mb200::device_span_ok(A, batch_span(a_rows, a_cols, lda, sa, batch) * es) ||
                !mb200::device_span_ok(B, batch_span(b_rows, b_cols, ldb, sb, batch) * es)))
    return CUBLAS_STATUS_INVALID_VALUE;
  if (!mb200::device_span_ok(C, batch_span(m, n, ldc, sc, batch) * es))
    return CUBLAS_STATUS_INVALID_VALUE;
  if (!mb200::aligned_to(A, es) || !mb200::aligned_to(B, es) || !mb200::aligned_to(C, es))
    return CUBLAS_STATUS_INVALID_VALUE;
  cudaError_t e = cudaErrorNotSupported;
  if (type != Elem::kF32)
    e = mb200::blas::launch_gemm_tc(g, stream);
  else if (math != CUBLAS_PEDANTIC_MATH)
    e = run_tf32x3(ctx, g, stream);
  if (e == cudaErrorNotSupported) {
    (void)cudaGetLastError();
    const std::size_t need = mb200::blas::gemm_simt_workspace(g);
    if (need == 0) {
      e = mb200::blas::launch_gemm_simt(g, stream);
    } else {
      // K split across CTAs, partial sums in the handle's workspace
      BufferUse use(ctx, stream);
      if (!use.ok()) return CUBLAS_STATUS_EXECUTION_FAILED;
      void* ws = use.workspace(need);
      e = mb200::blas::launch_gemm_simt_split(g, ws, ws ? use.workspace_bytes() : 0, stream);
      if (e == cudaSuccess) e = use.done();
    }
  }
  return e == cudaSuccess ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

// Elements a vector of n entries with increment inc spans (reference
// cublas_level1.mm:48-54): inc = 0 touches one element.
std::size_t span_elems(int n, int inc) {
  if (n <= 0) return 0;
  const std::size_t a = inc == 0 ? 1u : static_cast<std::size_t>(inc > 0 ? inc : -inc);
  return 1u + static_cast<std::size_t>(n - 1) * a;
}

template <typename T>
bool vec_ok(const T* p, int n, int inc) {
  return mb200::device_span_ok(p, span_elems(n, inc) * sizeof(T)) &&
         mb200::aligned_to(p, sizeof(T));
}

// The handle's stream and pointer mode.
void snapshot(BlasContext& ctx, cudaStream_t* stream, cublasPointerMode_t* mode) {
  std::lock_guard<std::mutex> g(ctx.mu);
  *stream = ctx.stream;
  *mode = ctx.pointer_mode;
}

// A scalar argument: its host value, or (device pointer mode) a checked device
// pointer the kernel reads.
template <typename T>
bool scalar(cublasPointerMode_t mode, const T* p, T* host, const T** dev) {
  if (mode == CUBLAS_POINTER_MODE_DEVICE) {
    if (!mb200::device_span_ok(p, sizeof(T))) return false;
    *dev = p;
    *host = T(0);
  } else {
    *host = *p;
    *dev = nullptr;
  }
  return true;
}

// One geam call (cublas_level3.mm:619-712 for fp32, :821-927 for fp64): the
// reference's argument checks and status codes, then the kernel.  In host pointer
// mode an operand whose scalar is zero is not checked (nor read); in device
// pointer mode the scalars are unknown here, so both operands must be valid.
// True when the element spans of two column-major matrices share any byte.
template <typename T>
bool spans_overlap(const T* p, int rows, int cols, int ld, const T* c, int m, int n, int ldc) {
  const auto a0 = reinterpret_cast<std::uintptr_t>(p);
  const auto a1 = a0 + (static_cast<std::uintptr_t>(ld) * (cols - 1) + rows) * sizeof(T);
  const auto c0 = reinterpret_cast<std::uintptr_t>(c);
  const auto c1 = c0 + (static_cast<std::uintptr_t>(ldc) * (n - 1) + m) * sizeof(T);
  return a0 < c1 && c0 < a1;
}

// In-place geam: C may be the operand itself when that operand is not transposed and
// has C's leading dimension, since each element is then read and written by the same
// thread.  Any other overlap between C and an operand that is read would let one tile
// overwrite values that another tile has still to read (the tiles run in parallel,
// where the reference's host loop runs in order), so it is refused.
template <typename T>
bool bad_alias(bool trans, const T* X, int rows, int cols, int ld, const T* C, int m, int n,
               int ldc) {
  if (!spans_overlap(X, rows, cols, ld, C, m, n, ldc)) return false;
  return trans || X != C || ld != ldc;
}

template <typename T>
cublasStatus_t run_geam(cublasHandle_t handle, cublasOperation_t transa,
                        cublasOperation_t transb, int m, int n, const T* alpha, const T* A,
                        int lda, const T* beta, const T* B, int ldb, T* C, int ldc,
                        bool c_null_is_invalid);

cublasStatus_t status_of(cudaError_t e) {
  return e == cudaSuccess ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

// Runs a reduction and delivers its result: in device pointer mode the kernel
// writes `result` (device memory) directly; in host mode it writes the handle's
// result slot, copied to `result` after the stream finishes (the reference
// synchronises the same way, cublas_level1.mm:119-126).
template <typename E>
struct NoDeduce {
  using type = E;
};

template <typename T, typename E = float>
cublasStatus_t run_reduction(BlasContext& ctx, mb200::blas::Reduce op, int n, const E* x,
                             int incx, const typename NoDeduce<E>::type* y, int incy, T* result) {
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(ctx, &stream, &mode);
  if (mode == CUBLAS_POINTER_MODE_DEVICE && !mb200::device_span_ok(result, sizeof(T)))
    return CUBLAS_STATUS_INVALID_VALUE;
  const bool empty = n <= 0 || (op != mb200::blas::Reduce::kDot && incx <= 0);
  if (empty && mode == CUBLAS_POINTER_MODE_HOST) {
    *result = T{};
    return CUBLAS_STATUS_SUCCESS;
  }
  if (!empty && (!vec_ok(x, n, incx) || (op == mb200::blas::Reduce::kDot && !vec_ok(y, n, incy))))
    return CUBLAS_STATUS_INVALID_VALUE;
  BufferUse use(ctx, stream);
  if (!use.ok()) return CUBLAS_STATUS_EXECUTION_FAILED;
  void* scratch = use.reduction_scratch();
  if (scratch == nullptr) return CUBLAS_STATUS_ALLOC_FAILED;
  void* out = mode == CUBLAS_POINTER_MODE_DEVICE ? static_cast<void*>(result) : use.result_slot();
  cudaError_t e;
  if constexpr (sizeof(E) == 8)
    e = mb200::blas::launch_dreduce(op, n, x, incx, y, incy, out, scratch, stream);
  else
    e = mb200::blas::launch_reduce(op, n, x, incx, y, incy, out, scratch, stream);
  if (e == cudaSuccess && mode == CUBLAS_POINTER_MODE_HOST)
    e = cudaMemcpyAsync(result, out, sizeof(T), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = use.done();
  if (e == cudaSuccess && mode == CUBLAS_POINTER_MODE_HOST) e = cudaStreamSynchronize(stream);
  return status_of(e);
}

}  // namespace

extern "C" {

cublasStatus_t cublasCreate_v2(cublasHandle_t* handle) {
  if (handle == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  auto h = handles().add<cublasHandle_t>(std::make_shared<BlasContext>());
  if (h == nullptr) return CUBLAS_STATUS_ALLOC_FAILED;
  *handle = h;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasDestroy_v2(cublasHandle_t handle) {
  return handles().take(handle) ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_NOT_INITIALIZED;
}

cublasStatus_t cublasGetVersion_v2(cublasHandle_t handle, int* version) {
  if (version == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  if (handle != nullptr && !handles().get(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  *version = kCublasVersion;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, cudaStream_t streamId) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> g(h->mu);
  h->stream = streamId;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetStream_v2(cublasHandle_t handle, cudaStream_t* streamId) {
  if (streamId == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> g(h->mu);
  *streamId = h->stream;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t mode) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (mode != CUBLAS_POINTER_MODE_HOST && mode != CUBLAS_POINTER_MODE_DEVICE)
    return CUBLAS_STATUS_INVALID_VALUE;
  std::lock_guard<std::mutex> g(h->mu);
  h->pointer_mode = mode;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t* mode) {
  if (mode == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> g(h->mu);
  *mode = h->pointer_mode;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetMathMode(cublasHandle_t handle, cublasMath_t mode) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (mode < CUBLAS_DEFAULT_MATH || mode > CUBLAS_TF32_TENSOR_OP_MATH)
    return CUBLAS_STATUS_INVALID_VALUE;
  std::lock_guard<std::mutex> g(h->mu);
  h->math_mode = mode;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetMathMode(cublasHandle_t handle, cublasMath_t* mode) {
  if (mode == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> g(h->mu);
  *mode = h->math_mode;
  return CUBLAS_STATUS_SUCCESS;
}

const char* cublasGetStatusName(cublasStatus_t status) {
  switch (status) {
    case CUBLAS_STATUS_SUCCESS: return "CUBLAS_STATUS_SUCCESS";
    case CUBLAS_STATUS_NOT_INITIALIZED: return "CUBLAS_STATUS_NOT_INITIALIZED";
    case CUBLAS_STATUS_ALLOC_FAILED: return "CUBLAS_STATUS_ALLOC_FAILED";
    case CUBLAS_STATUS_INVALID_VALUE: return "CUBLAS_STATUS_INVALID_VALUE";
    case CUBLAS_STATUS_ARCH_MISMATCH: return "CUBLAS_STATUS_ARCH_MISMATCH";
    case CUBLAS_STATUS_MAPPING_ERROR: return "CUBLAS_STATUS_MAPPING_ERROR";
    case CUBLAS_STATUS_EXECUTION_FAILED: return "CUBLAS_STATUS_EXECUTION_FAILED";
    case CUBLAS_STATUS_INTERNAL_ERROR: return "CUBLAS_STATUS_INTERNAL_ERROR";
    case CUBLAS_STATUS_NOT_SUPPORTED: return "CUBLAS_STATUS_NOT_SUPPORTED";
  }
  return "CUBLAS_STATUS_UNKNOWN";
}

const char* cublasGetStatusString(cublasStatus_t status) { return cublasGetStatusName(status); }

cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t handle, cublasOperation_t transa,
                                         cublasOperation_t transb, int m, int n, int k,
                                         const float* alpha, const float* A, int lda,
                                         long long int strideA, const float* B, int ldb,
                                         long long int strideB, const float* beta, float* C,
                                         int ldc, long long int strideC, int batchCount) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  const cublasStatus_t st =
      check_args(transa, transb, m, n, k, lda, ldb, ldc, batchCount, alpha, beta);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  return run_gemm(*h, Elem::kF32, transa, transb, m, n, k, alpha, false, A, lda, strideA, B, ldb,
                  strideB, beta, C, ldc, strideC, batchCount);
}

cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, cublasOperation_t transa,
                              cublasOperation_t transb, int m, int n, int k, const float* alpha,
                              const float* A, int lda, const float* B, int ldb, const float* beta,
                              float* C, int ldc) {
  return cublasSgemmStridedBatched(handle, transa, transb, m, n, k, alpha, A, lda, 0, B, ldb, 0,
                                   beta, C, ldc, 0, 1);
}

cublasStatus_t cublasHgemm(cublasHandle_t handle, cublasOperation_t transa,
                           cublasOperation_t transb, int m, int n, int k, const __half* alpha,
                           const __half* A, int lda, const __half* B, int ldb, const __half* beta,
                           __half* C, int ldc) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  const cublasStatus_t st = check_args(transa, transb, m, n, k, lda, ldb, ldc, 1, alpha, beta);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  return run_gemm(*h, Elem::kF16, transa, transb, m, n, k, alpha, true, A, lda, 0, B, ldb, 0, beta,
                  C, ldc, 0, 1);
}

cublasStatus_t cublasGemmStridedBatchedEx(cublasHandle_t handle, cublasOperation_t transa,
                                          cublasOperation_t transb, int m, int n, int k,
                                          const void* alpha, const void* A, cudaDataType Atype,
                                          int lda, long long int strideA, const void* B,
                                          cudaDataType Btype, int ldb, long long int strideB,
                                          const void* beta, void* C, cudaDataType Ctype, int ldc,
                                          long long int strideC, int batchCount, int computeType,
                                          cublasGemmAlgo_t algo) {
  (void)algo;
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  const cublasStatus_t st =
      check_args(transa, transb, m, n, k, lda, ldb, ldc, batchCount, alpha, beta);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if (Atype == CUDA_R_32F && Btype == CUDA_R_32F && Ctype == CUDA_R_32F)
    return run_gemm(*h, Elem::kF32, transa, transb, m, n, k, alpha, false, A, lda, strideA, B,
                    ldb, strideB, beta, C, ldc, strideC, batchCount);
  Elem e;
  if (Atype == CUDA_R_16F && Btype == CUDA_R_16F && Ctype == CUDA_R_16F) {
    e = Elem::kF16;
  } else if (Atype == CUDA_R_16BF && Btype == CUDA_R_16BF && Ctype == CUDA_R_16BF) {
    e = Elem::kBF16;
  } else {
    return CUBLAS_STATUS_NOT_SUPPORTED;
  }
  // Scalar type follows the compute type (cublas_level3.mm:583-602).
  const bool half_scalars =
      (computeType == CUBLAS_COMPUTE_16F || computeType == CUBLAS_COMPUTE_16F_PEDANTIC ||
       computeType == static_cast<int>(CUDA_R_16F));
  return run_gemm(*h, e, transa, transb, m, n, k, alpha, half_scalars, A, lda, strideA, B, ldb,
                  strideB, beta, C, ldc, strideC, batchCount);
}

cublasStatus_t cublasGemmEx(cublasHandle_t handle, cublasOperation_t transa,
                            cublasOperation_t transb, int m, int n, int k, const void* alpha,
                            const void* A, cudaDataType Atype, int lda, const void* B,
                            cudaDataType Btype, int ldb, const void* beta, void* C,
                            cudaDataType Ctype, int ldc, int computeType, cublasGemmAlgo_t algo) {
  return cublasGemmStridedBatchedEx(handle, transa, transb, m, n, k, alpha, A, Atype, lda, 0, B,
                                    Btype, ldb, 0, beta, C, Ctype, ldc, 0, 1, computeType, algo);
}

// ---------------------------------------------------------------- level 1
cublasStatus_t cublasSaxpy_v2(cublasHandle_t handle, int n, const float* alpha, const float* x,
                              int incx, float* y, int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (alpha == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  if (n <= 0) return CUBLAS_STATUS_SUCCESS;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  float a;
  const float* a_dev;
  if (!scalar(mode, alpha, &a, &a_dev)) return CUBLAS_STATUS_INVALID_VALUE;
  if (a_dev == nullptr && a == 0.0f) return CUBLAS_STATUS_SUCCESS;
  if (!vec_ok(x, n, incx) || !vec_ok(y, n, incy)) return CUBLAS_STATUS_INVALID_VALUE;
  return status_of(mb200::blas::launch_saxpy(n, a, a_dev, x, incx, y, incy, stream));
}

cublasStatus_t cublasScopy_v2(cublasHandle_t handle, int n, const float* x, int incx, float* y,
                              int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (n <= 0) return CUBLAS_STATUS_SUCCESS;
  if (!vec_ok(x, n, incx) || !vec_ok(y, n, incy)) return CUBLAS_STATUS_INVALID_VALUE;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  return status_of(mb200::blas::launch_scopy(n, x, incx, y, incy, stream));
}

cublasStatus_t cublasSscal_v2(cublasHandle_t handle, int n, const float* alpha, float* x,
                              int incx) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (alpha == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  if (n <= 0 || incx <= 0) return CUBLAS_STATUS_SUCCESS;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  float a;
  const float* a_dev;
  if (!scalar(mode, alpha, &a, &a_dev)) return CUBLAS_STATUS_INVALID_VALUE;
  if (!vec_ok(x, n, incx)) return CUBLAS_STATUS_INVALID_VALUE;
  return status_of(mb200::blas::launch_sscal(n, a, a_dev, x, incx, stream));
}

cublasStatus_t cublasSswap_v2(cublasHandle_t handle, int n, float* x, int incx, float* y,
                              int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (n <= 0) return CUBLAS_STATUS_SUCCESS;
  if (!vec_ok(x, n, incx) || !vec_ok(y, n, incy)) return CUBLAS_STATUS_INVALID_VALUE;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  return status_of(mb200::blas::launch_sswap(n, x, incx, y, incy, stream));
}

cublasStatus_t cublasSdot_v2(cublasHandle_t handle, int n, const float* x, int incx,
                             const float* y, int incy, float* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction(*h, mb200::blas::Reduce::kDot, n, x, incx, y, incy, result);
}

cublasStatus_t cublasSnrm2_v2(cublasHandle_t handle, int n, const float* x, int incx,
                              float* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction(*h, mb200::blas::Reduce::kNrm2, n, x, incx, nullptr, 0, result);
}

cublasStatus_t cublasSasum_v2(cublasHandle_t handle, int n, const float* x, int incx,
                              float* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction(*h, mb200::blas::Reduce::kAsum, n, x, incx, nullptr, 0, result);
}

cublasStatus_t cublasIsamax_v2(cublasHandle_t handle, int n, const float* x, int incx,
                               int* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction(*h, mb200::blas::Reduce::kAmax, n, x, incx, nullptr, 0, result);
}

// ---------------------------------------------------------------- level 2
cublasStatus_t cublasSgemv_v2(cublasHandle_t handle, cublasOperation_t trans, int m, int n,
                              const float* alpha, const float* A, int lda, const float* x,
                              int incx, const float* beta, float* y, int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  // cublas_level2.mm:45-48
  if (!valid_op(trans) || m < 0 || n < 0 || lda < (m > 1 ? m : 1) || incx == 0 || incy == 0 ||
      alpha == nullptr || beta == nullptr)
    return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0) return CUBLAS_STATUS_SUCCESS;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  float a, b;
  const float *a_dev, *b_dev;
  if (!scalar(mode, alpha, &a, &a_dev) || !scalar(mode, beta, &b, &b_dev))
    return CUBLAS_STATUS_INVALID_VALUE;
  const bool t = trans != CUBLAS_OP_N;
  const int x_len = t ? m : n, y_len = t ? n : m;
  const std::size_t a_elems = static_cast<std::size_t>(lda) * (n - 1) + m;
  if (!mb200::device_span_ok(A, a_elems * sizeof(float)) || !mb200::aligned_to(A, 4) ||
      !vec_ok(x, x_len, incx) || !vec_ok(y, y_len, incy))
    return CUBLAS_STATUS_INVALID_VALUE;
  const std::size_t need = mb200::blas::gemv_workspace_bytes(t, m, n);
  if (need == 0)
    return status_of(mb200::blas::launch_sgemv(t, m, n, a, a_dev, A, lda, x, incx, b, b_dev, y,
                                                incy, nullptr, 0, stream));
  BufferUse use(*h, stream);
  if (!use.ok()) return CUBLAS_STATUS_EXECUTION_FAILED;
  void* ws = use.workspace(need);
  cudaError_t e = mb200::blas::launch_sgemv(t, m, n, a, a_dev, A, lda, x, incx, b, b_dev, y, incy,
                                            ws, ws ? use.workspace_bytes() : 0, stream);
  if (e == cudaSuccess) e = use.done();
  return status_of(e);
}

// ---------------------------------------------------------------- fp64
// Argument checks and status codes of the reference's host-BLAS wrappers
// (cublas_level1.mm:658-979, cublas_level2.mm:135-200, cublas_level3.mm:714-819),
// in their order; the arithmetic is blas/dblas_kernels.cu.
cublasStatus_t cublasDaxpy_v2(cublasHandle_t handle, int n, const double* alpha, const double* x,
                              int incx, double* y, int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (n <= 0) return CUBLAS_STATUS_SUCCESS;
  if (alpha == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  double a;
  const double* a_dev;
  if (!scalar(mode, alpha, &a, &a_dev)) return CUBLAS_STATUS_INVALID_VALUE;
  if (a_dev == nullptr && a == 0.0) return CUBLAS_STATUS_SUCCESS;
  if (!vec_ok(x, n, incx) || !vec_ok(y, n, incy)) return CUBLAS_STATUS_INVALID_VALUE;
  return status_of(mb200::blas::launch_daxpy(n, a, a_dev, x, incx, y, incy, stream));
}

cublasStatus_t cublasDcopy_v2(cublasHandle_t handle, int n, const double* x, int incx, double* y,
                              int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (n <= 0) return CUBLAS_STATUS_SUCCESS;
  if (!vec_ok(x, n, incx) || !vec_ok(y, n, incy)) return CUBLAS_STATUS_INVALID_VALUE;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  return status_of(mb200::blas::launch_dcopy(n, x, incx, y, incy, stream));
}

cublasStatus_t cublasDscal_v2(cublasHandle_t handle, int n, const double* alpha, double* x,
                              int incx) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (n <= 0 || incx <= 0) return CUBLAS_STATUS_SUCCESS;
  if (alpha == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  double a;
  const double* a_dev;
  if (!scalar(mode, alpha, &a, &a_dev)) return CUBLAS_STATUS_INVALID_VALUE;
  if (!vec_ok(x, n, incx)) return CUBLAS_STATUS_INVALID_VALUE;
  return status_of(mb200::blas::launch_dscal(n, a, a_dev, x, incx, stream));
}

cublasStatus_t cublasDswap_v2(cublasHandle_t handle, int n, double* x, int incx, double* y,
                              int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (n <= 0) return CUBLAS_STATUS_SUCCESS;
  if (!vec_ok(x, n, incx) || !vec_ok(y, n, incy)) return CUBLAS_STATUS_INVALID_VALUE;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  return status_of(mb200::blas::launch_dswap(n, x, incx, y, incy, stream));
}

cublasStatus_t cublasDdot_v2(cublasHandle_t handle, int n, const double* x, int incx,
                             const double* y, int incy, double* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction(*h, mb200::blas::Reduce::kDot, n, x, incx, y, incy, result);
}

cublasStatus_t cublasDnrm2_v2(cublasHandle_t handle, int n, const double* x, int incx,
                              double* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction<double, double>(*h, mb200::blas::Reduce::kNrm2, n, x, incx, nullptr, 0,
                                       result);
}

cublasStatus_t cublasDasum_v2(cublasHandle_t handle, int n, const double* x, int incx,
                              double* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction<double, double>(*h, mb200::blas::Reduce::kAsum, n, x, incx, nullptr, 0,
                                       result);
}

cublasStatus_t cublasIdamax_v2(cublasHandle_t handle, int n, const double* x, int incx,
                               int* result) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (result == nullptr) return CUBLAS_STATUS_INVALID_VALUE;
  return run_reduction<int, double>(*h, mb200::blas::Reduce::kAmax, n, x, incx, nullptr, 0,
                                    result);
}

cublasStatus_t cublasDgemv_v2(cublasHandle_t handle, cublasOperation_t trans, int m, int n,
                              const double* alpha, const double* A, int lda, const double* x,
                              int incx, const double* beta, double* y, int incy) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  // cublas_level2.mm:142-145
  if (!valid_op(trans) || m < 0 || n < 0 || lda < (m > 1 ? m : 1) || incx == 0 || incy == 0 ||
      alpha == nullptr || beta == nullptr)
    return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0) return CUBLAS_STATUS_SUCCESS;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  double a, b;
  const double *a_dev, *b_dev;
  if (!scalar(mode, alpha, &a, &a_dev) || !scalar(mode, beta, &b, &b_dev))
    return CUBLAS_STATUS_INVALID_VALUE;
  const bool t = trans != CUBLAS_OP_N;
  const int x_len = t ? m : n, y_len = t ? n : m;
  const std::size_t a_elems = static_cast<std::size_t>(lda) * (n - 1) + m;
  if (!mb200::device_span_ok(A, a_elems * sizeof(double)) || !mb200::aligned_to(A, 8) ||
      !vec_ok(x, x_len, incx) || !vec_ok(y, y_len, incy))
    return CUBLAS_STATUS_INVALID_VALUE;
  const std::size_t need = mb200::blas::dgemv_workspace_bytes(t, m, n);
  if (need == 0)
    return status_of(mb200::blas::launch_dgemv(t, m, n, a, a_dev, A, lda, x, incx, b, b_dev, y,
                                                incy, nullptr, 0, stream));
  BufferUse use(*h, stream);
  if (!use.ok()) return CUBLAS_STATUS_EXECUTION_FAILED;
  void* ws = use.workspace(need);
  cudaError_t e = mb200::blas::launch_dgemv(t, m, n, a, a_dev, A, lda, x, incx, b, b_dev, y, incy,
                                            ws, ws ? use.workspace_bytes() : 0, stream);
  if (e == cudaSuccess) e = use.done();
  return status_of(e);
}

cublasStatus_t cublasDgemmStridedBatched(cublasHandle_t handle, cublasOperation_t transa,
                                         cublasOperation_t transb, int m, int n, int k,
                                         const double* alpha, const double* A, int lda,
                                         long long int strideA, const double* B, int ldb,
                                         long long int strideB, const double* beta, double* C,
                                         int ldc, long long int strideC, int batchCount) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  const cublasStatus_t st =
      check_args(transa, transb, m, n, k, lda, ldb, ldc, batchCount, alpha, beta);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if (m == 0 || n == 0 || batchCount == 0) return CUBLAS_STATUS_SUCCESS;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  mb200::blas::DgemmArgs g{};
  if (!scalar(mode, alpha, &g.alpha, &g.alpha_dev) || !scalar(mode, beta, &g.beta, &g.beta_dev))
    return CUBLAS_STATUS_INVALID_VALUE;
  g.trans_a = transa != CUBLAS_OP_N;
  g.trans_b = transb != CUBLAS_OP_N;
  g.m = m;
  g.n = n;
  g.k = k;
  g.a = A;
  g.lda = lda;
  g.stride_a = strideA;
  g.b = B;
  g.ldb = ldb;
  g.stride_b = strideB;
  g.c = C;
  g.ldc = ldc;
  g.stride_c = strideC;
  g.batch = batchCount;
  // the buffers of A, B and C are resolved as in cublas_level3.mm:753-778
  const int a_rows = g.trans_a ? k : m, a_cols = g.trans_a ? m : k;
  const int b_rows = g.trans_b ? n : k, b_cols = g.trans_b ? k : n;
  if (k > 0 &&
      (!mb200::device_span_ok(A, batch_span(a_rows, a_cols, lda, strideA, batchCount) * 8) ||
       !mb200::device_span_ok(B, batch_span(b_rows, b_cols, ldb, strideB, batchCount) * 8)))
    return CUBLAS_STATUS_INVALID_VALUE;
  if (!mb200::device_span_ok(C, batch_span(m, n, ldc, strideC, batchCount) * 8))
    return CUBLAS_STATUS_INVALID_VALUE;
  if (!mb200::aligned_to(A, 8) || !mb200::aligned_to(B, 8) || !mb200::aligned_to(C, 8))
    return CUBLAS_STATUS_INVALID_VALUE;
  return status_of(mb200::blas::launch_dgemm(g, stream));
}

cublasStatus_t cublasDgemm_v2(cublasHandle_t handle, cublasOperation_t transa,
                              cublasOperation_t transb, int m, int n, int k, const double* alpha,
                              const double* A, int lda, const double* B, int ldb,
                              const double* beta, double* C, int ldc) {
  return cublasDgemmStridedBatched(handle, transa, transb, m, n, k, alpha, A, lda, 0, B, ldb, 0,
                                   beta, C, ldc, 0, 1);
}

cublasStatus_t cublasSgeam(cublasHandle_t handle, cublasOperation_t transa,
                           cublasOperation_t transb, int m, int n, const float* alpha,
                           const float* A, int lda, const float* beta, const float* B, int ldb,
                           float* C, int ldc) {
  return run_geam(handle, transa, transb, m, n, alpha, A, lda, beta, B, ldb, C, ldc, false);
}

cublasStatus_t cublasDgeam(cublasHandle_t handle, cublasOperation_t transa,
                           cublasOperation_t transb, int m, int n, const double* alpha,
                           const double* A, int lda, const double* beta, const double* B,
                           int ldb, double* C, int ldc) {
  // The reference's fp64 path also rejects a null C up front (cublas_level3.mm:829-831).
  return run_geam(handle, transa, transb, m, n, alpha, A, lda, beta, B, ldb, C, ldc, true);
}

}  // extern "C"

namespace {

template <typename T>
bool scalar_of(cublasPointerMode_t mode, const T* p, T* host, const T** dev) {
  if (mode == CUBLAS_POINTER_MODE_DEVICE) {
    if (!mb200::device_span_ok(p, sizeof(T))) return false;
    *dev = p;
    *host = T(0);
  } else {
    *host = *p;
    *dev = nullptr;
  }
  return true;
}

template <typename T>
bool matrix_ok(const T* p, int rows, int cols, int ld) {
  const std::size_t elems = static_cast<std::size_t>(ld) * (cols - 1) + rows;
  return mb200::device_span_ok(p, elems * sizeof(T)) && mb200::aligned_to(p, sizeof(T));
}

template <typename T>
cublasStatus_t run_geam(cublasHandle_t handle, cublasOperation_t transa,
                        cublasOperation_t transb, int m, int n, const T* alpha, const T* A,
                        int lda, const T* beta, const T* B, int ldb, T* C, int ldc,
                        bool c_null_is_invalid) {
  auto h = handles().get(handle);
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (!valid_op(transa) || !valid_op(transb) || m < 0 || n < 0 || alpha == nullptr ||
      beta == nullptr || (c_null_is_invalid && C == nullptr))
    return CUBLAS_STATUS_INVALID_VALUE;
  const bool ta = transa != CUBLAS_OP_N, tb = transb != CUBLAS_OP_N;
  const int m1 = m > 1 ? m : 1, n1 = n > 1 ? n : 1;
  if (lda < (ta ? n1 : m1) || ldb < (tb ? n1 : m1) || ldc < m1)
    return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0) return CUBLAS_STATUS_SUCCESS;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  snapshot(*h, &stream, &mode);
  T a, b;
  const T *a_dev, *b_dev;
  if (!scalar_of(mode, alpha, &a, &a_dev) || !scalar_of(mode, beta, &b, &b_dev))
    return CUBLAS_STATUS_INVALID_VALUE;
  const bool device_mode = mode == CUBLAS_POINTER_MODE_DEVICE;
  if (!matrix_ok(C, m, n, ldc)) return CUBLAS_STATUS_INVALID_VALUE;
  if ((device_mode || a != T(0)) && !matrix_ok(A, ta ? n : m, ta ? m : n, lda))
    return CUBLAS_STATUS_INVALID_VALUE;
  if ((device_mode || b != T(0)) && !matrix_ok(B, tb ? n : m, tb ? m : n, ldb))
    return CUBLAS_STATUS_INVALID_VALUE;
  if ((device_mode || a != T(0)) && bad_alias(ta, A, ta ? n : m, ta ? m : n, lda, C, m, n, ldc))
    return CUBLAS_STATUS_INVALID_VALUE;
  if ((device_mode || b != T(0)) && bad_alias(tb, B, tb ? n : m, tb ? m : n, ldb, C, m, n, ldc))
    return CUBLAS_STATUS_INVALID_VALUE;
  return status_of(mb200::blas::launch_geam<T>(ta, tb, m, n, a, a_dev, A, lda, b, b_dev, B, ldb,
                                               C, ldc, stream));
}

}  // namespace
