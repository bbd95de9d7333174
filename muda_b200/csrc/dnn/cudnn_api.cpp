// cudnn_api.cpp — cuDNN C ABI: handles, descriptors, convolution forward, softmax forward.
//
// Mirrors libraries/dnn/src/cudnn_descriptors.mm and cudnn_ops.mm of the
// reference: same entry points, validation order and status codes.  Every
// buffer span is checked against its allocation before a kernel is launched.
//
// fp32 convolutions that the split-tf32 tensor-core kernel covers need a device
// workspace for the hi/lo planes of x and w.  cudnnGetConvolutionForwardWorkspaceSize
// reports 0 as the reference does (cudnn_ops.mm:112), so the handle owns a
// workspace (grown on demand, ordered after its previous use by an event); a
// caller-supplied workSpace that is large enough is used instead.
#pragma GCC visibility push(default)
#include "cudnn.h"
#pragma GCC visibility pop

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cstdint>
#include <initializer_list>
#include <memory>
#include <mutex>
#include <utility>

#include "common/device.hpp"
#include "common/lru.hpp"
#include "common/registry.hpp"
#include "dnn/dnn.hpp"

namespace {

using mb200::ObjKind;
using mb200::Registry;
using mb200::dnn::View4;

struct DnnContext {
  std::mutex mu;
  cudaStream_t stream = nullptr;
  // split-tf32 workspace: held under ws_mu for the whole call that uses it
  std::mutex ws_mu;
  std::shared_ptr<mb200::DeviceBuffer> ws;
  cudaEvent_t ws_done = nullptr;  // recorded after the last call that used ws

  ~DnnContext() {
    if (ws_done != nullptr) (void)cudaEventDestroy(ws_done);
  }
};

struct TensorDesc {
  std::mutex mu;
  bool configured = false;
  cudnnTensorFormat_t format = CUDNN_TENSOR_NCHW;
  cudnnDataType_t dtype = CUDNN_DATA_FLOAT;
  int n = 0, c = 0, h = 0, w = 0;
  int ns = 0, cs = 0, hs = 0, ws = 0;
};

struct FilterDesc {
  std::mutex mu;
  bool configured = false;
  cudnnDataType_t dtype = CUDNN_DATA_FLOAT;
  cudnnTensorFormat_t format = CUDNN_TENSOR_NCHW;
  int k = 0, c = 0, h = 0, w = 0;
};

struct ConvDesc {
  std::mutex mu;
  bool configured = false;
  int pad_h = 0, pad_w = 0, stride_h = 1, stride_w = 1, dil_h = 1, dil_w = 1;
  int groups = 1;
  cudnnConvolutionMode_t mode = CUDNN_CROSS_CORRELATION;
  cudnnDataType_t compute = CUDNN_DATA_FLOAT;
};

struct ActivationDesc {
  std::mutex mu;
  bool configured = false;
  cudnnActivationMode_t mode = CUDNN_ACTIVATION_RELU;
  cudnnNanPropagation_t nan_opt = CUDNN_NOT_PROPAGATE_NAN;
  double coef = 0.0;
};

struct PoolingDesc {
  std::mutex mu;
  bool configured = false;
  cudnnPoolingMode_t mode = CUDNN_POOLING_MAX;
  cudnnNanPropagation_t nan_opt = CUDNN_NOT_PROPAGATE_NAN;
  int win_h = 0, win_w = 0, pad_h = 0, pad_w = 0, stride_h = 1, stride_w = 1;
};

Registry<ActivationDesc, ObjKind::kDnnActivation>& activations() {
  static Registry<ActivationDesc, ObjKind::kDnnActivation> r;
  return r;
}
Registry<PoolingDesc, ObjKind::kDnnPooling>& poolings() {
  static Registry<PoolingDesc, ObjKind::kDnnPooling> r;
  return r;
}

Registry<DnnContext, ObjKind::kDnnHandle>& handles() {
  static Registry<DnnContext, ObjKind::kDnnHandle> r;
  return r;
}
Registry<TensorDesc, ObjKind::kDnnTensor>& tensors() {
  static Registry<TensorDesc, ObjKind::kDnnTensor> r;
  return r;
}
Registry<FilterDesc, ObjKind::kDnnFilter>& filters() {
  static Registry<FilterDesc, ObjKind::kDnnFilter> r;
  return r;
}
Registry<ConvDesc, ObjKind::kDnnConv>& convs() {
  static Registry<ConvDesc, ObjKind::kDnnConv> r;
  return r;
}

// The reference accepts FLOAT and HALF descriptors (cudnn_descriptors.mm:13-15);
// BFLOAT16 is this library's extension.
bool supported_dtype(cudnnDataType_t t) {
  return t == CUDNN_DATA_FLOAT || t == CUDNN_DATA_HALF || t == CUDNN_DATA_BFLOAT16;
}

int elem_size(cudnnDataType_t t) { return t == CUDNN_DATA_FLOAT ? 4 : 2; }

// Snapshot of a tensor descriptor taken under its lock.
struct TensorSnap {
  bool configured;
  cudnnDataType_t dtype;
  View4 v;
};

TensorSnap snap(TensorDesc& d) {
  std::lock_guard<std::mutex> g(d.mu);
  return {d.configured, d.dtype, View4{d.n, d.c, d.h, d.w, d.ns, d.cs, d.hs, d.ws}};
}

// Elements from the first to the last addressed element, inclusive.
std::size_t span_elems(const View4& v) {
  if (v.n <= 0 || v.c <= 0 || v.h <= 0 || v.w <= 0) return 0;
  return 1 + static_cast<std::size_t>(v.n - 1) * v.ns + static_cast<std::size_t>(v.c - 1) * v.cs +
         static_cast<std::size_t>(v.h - 1) * v.hs + static_cast<std::size_t>(v.w - 1) * v.ws;
}

bool packed_nchw(const View4& v) {
  return v.ws == 1 && v.hs == v.w && v.cs == static_cast<std::int64_t>(v.h) * v.w &&
         v.ns == static_cast<std::int64_t>(v.c) * v.h * v.w;
}

bool packed_nhwc(const View4& v) {
  return v.cs == 1 && v.ws == v.c && v.hs == static_cast<std::int64_t>(v.w) * v.c &&
         v.ns == static_cast<std::int64_t>(v.h) * v.w * v.c;
}

struct ConvPlan {
  mb200::dnn::ConvShape shape;
  cudnnDataType_t dtype;
  std::size_t x_bytes, w_bytes, y_bytes;
};

// Validation of BuildConvParams (libraries/dnn/src/cudnn_ops.mm:26-83).
bool build_conv(TensorDesc& xd, FilterDesc& wd, ConvDesc& cd, TensorDesc& yd, ConvPlan* out) {
  const TensorSnap xs = snap(xd), ys = snap(yd);
  FilterDesc f;
  {
    std::lock_guard<std::mutex> g(wd.mu);
    f.configured = wd.configured;
    f.dtype = wd.dtype;
    f.format = wd.format;
    f.k = wd.k;
    f.c = wd.c;
    f.h = wd.h;
    f.w = wd.w;
  }
  ConvDesc c;
  {
    std::lock_guard<std::mutex> g(cd.mu);
    c.configured = cd.configured;
    c.pad_h = cd.pad_h;
    c.pad_w = cd.pad_w;
    c.stride_h = cd.stride_h;
    c.stride_w = cd.stride_w;
    c.dil_h = cd.dil_h;
    c.dil_w = cd.dil_w;
    c.groups = cd.groups;
    c.mode = cd.mode;
  }
  if (!xs.configured || !f.configured || !c.configured || !ys.configured) return false;
  if (xs.v.n != ys.v.n || ys.v.c != f.k) return false;
  if (c.groups <= 0 || xs.v.c % c.groups != 0 || f.k % c.groups != 0) return false;
  if (f.c != xs.v.c / c.groups) return false;
  const int eff_kh = 1 + (f.h - 1) * c.dil_h;
  const int eff_kw = 1 + (f.w - 1) * c.dil_w;
  const int oh = 1 + (xs.v.h + 2 * c.pad_h - eff_kh) / c.stride_h;
  const int ow = 1 + (xs.v.w + 2 * c.pad_w - eff_kw) / c.stride_w;
  if (ys.v.h != oh || ys.v.w != ow) return false;
  out->shape.x = xs.v;
  out->shape.y = ys.v;
  out->shape.kh = f.h;
  out->shape.kw = f.w;
  out->shape.pad_h = c.pad_h;
  out->shape.pad_w = c.pad_w;
  out->shape.stride_h = c.stride_h;
  out->shape.stride_w = c.stride_w;
  out->shape.dil_h = c.dil_h;
  out->shape.dil_w = c.dil_w;
  out->shape.groups = c.groups;
  out->shape.filter_krsc = (f.format == CUDNN_TENSOR_NHWC);
  out->shape.convolution = (c.mode == CUDNN_CONVOLUTION);
  out->dtype = xs.dtype;
  const int es = elem_size(xs.dtype);
  out->x_bytes = span_elems(xs.v) * es;
  out->y_bytes = span_elems(ys.v) * es;
  out->w_bytes = static_cast<std::size_t>(f.k) * f.c * f.h * f.w * es;
  if (xs.dtype != ys.dtype || f.dtype != xs.dtype) out->dtype = CUDNN_DATA_DOUBLE;  // mixed: reject
  return true;
}

cudaStream_t stream_of(DnnContext& h) {
  std::lock_guard<std::mutex> g(h.mu);
  return h.stream;
}

}  // namespace

extern "C" {

size_t cudnnGetVersion(void) { return CUDNN_VERSION; }

const char* cudnnGetErrorString(cudnnStatus_t status) {
  switch (status) {
    case CUDNN_STATUS_SUCCESS: return "CUDNN_STATUS_SUCCESS";
    case CUDNN_STATUS_NOT_INITIALIZED: return "CUDNN_STATUS_NOT_INITIALIZED";
    case CUDNN_STATUS_ALLOC_FAILED: return "CUDNN_STATUS_ALLOC_FAILED";
    case CUDNN_STATUS_BAD_PARAM: return "CUDNN_STATUS_BAD_PARAM";
    case CUDNN_STATUS_INTERNAL_ERROR: return "CUDNN_STATUS_INTERNAL_ERROR";
    case CUDNN_STATUS_INVALID_VALUE: return "CUDNN_STATUS_INVALID_VALUE";
    case CUDNN_STATUS_ARCH_MISMATCH: return "CUDNN_STATUS_ARCH_MISMATCH";
    case CUDNN_STATUS_MAPPING_ERROR: return "CUDNN_STATUS_MAPPING_ERROR";
    case CUDNN_STATUS_EXECUTION_FAILED: return "CUDNN_STATUS_EXECUTION_FAILED";
    case CUDNN_STATUS_NOT_SUPPORTED: return "CUDNN_STATUS_NOT_SUPPORTED";
  }
  return "CUDNN_STATUS_UNKNOWN";
}

cudnnStatus_t cudnnCreate(cudnnHandle_t* handle) {
  if (handle == nullptr) return CUDNN_STATUS_BAD_PARAM;
  cudnnHandle_t h = handles().add<cudnnHandle_t>(std::make_shared<DnnContext>());
  if (h == nullptr) return CUDNN_STATUS_ALLOC_FAILED;
  *handle = h;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroy(cudnnHandle_t handle) {
  return handles().take(handle) ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_BAD_PARAM;
}

cudnnStatus_t cudnnSetStream(cudnnHandle_t handle, cudaStream_t streamId) {
  auto h = handles().get(handle);
  if (!h) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(h->mu);
  h->stream = streamId;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetStream(cudnnHandle_t handle, cudaStream_t* streamId) {
  if (streamId == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  if (!h) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(h->mu);
  *streamId = h->stream;
  return CUDNN_STATUS_SUCCESS;
}

// ---------------------------------------------------------------- tensors --
cudnnStatus_t cudnnCreateTensorDescriptor(cudnnTensorDescriptor_t* tensorDesc) {
  if (tensorDesc == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto h = tensors().add<cudnnTensorDescriptor_t>(std::make_shared<TensorDesc>());
  if (h == nullptr) return CUDNN_STATUS_ALLOC_FAILED;
  *tensorDesc = h;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetTensor4dDescriptor(cudnnTensorDescriptor_t tensorDesc,
                                         cudnnTensorFormat_t format, cudnnDataType_t dataType,
                                         int n, int c, int h, int w) {
  auto d = tensors().get(tensorDesc);
  if (!d || n <= 0 || c <= 0 || h <= 0 || w <= 0) return CUDNN_STATUS_BAD_PARAM;
  if (format != CUDNN_TENSOR_NCHW && format != CUDNN_TENSOR_NHWC) return CUDNN_STATUS_BAD_PARAM;
  if (dataType == CUDNN_DATA_DOUBLE) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!supported_dtype(dataType)) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  d->configured = true;
  d->format = format;
  d->dtype = dataType;
  d->n = n;
  d->c = c;
  d->h = h;
  d->w = w;
  if (format == CUDNN_TENSOR_NCHW) {
    d->ws = 1;
    d->hs = w;
    d->cs = h * w;
    d->ns = c * h * w;
  } else {
    d->cs = 1;
    d->ws = c;
    d->hs = w * c;
    d->ns = h * w * c;
  }
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetTensor4dDescriptorEx(cudnnTensorDescriptor_t tensorDesc,
                                           cudnnDataType_t dataType, int n, int c, int h, int w,
                                           int nStride, int cStride, int hStride, int wStride) {
  auto d = tensors().get(tensorDesc);
  if (!d || n <= 0 || c <= 0 || h <= 0 || w <= 0 || nStride <= 0 || cStride <= 0 ||
      hStride <= 0 || wStride <= 0)
    return CUDNN_STATUS_BAD_PARAM;
  if (dataType == CUDNN_DATA_DOUBLE) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!supported_dtype(dataType)) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  d->configured = true;
  d->format = (cStride == 1 && wStride >= c) ? CUDNN_TENSOR_NHWC : CUDNN_TENSOR_NCHW;
  d->dtype = dataType;
  d->n = n;
  d->c = c;
  d->h = h;
  d->w = w;
  d->ns = nStride;
  d->cs = cStride;
  d->hs = hStride;
  d->ws = wStride;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetTensor4dDescriptor(cudnnTensorDescriptor_t tensorDesc,
                                         cudnnDataType_t* dataType, int* n, int* c, int* h, int* w,
                                         int* nStride, int* cStride, int* hStride, int* wStride) {
  auto d = tensors().get(tensorDesc);
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  if (!d->configured) return CUDNN_STATUS_BAD_PARAM;
  if (dataType) *dataType = d->dtype;
  if (n) *n = d->n;
  if (c) *c = d->c;
  if (h) *h = d->h;
  if (w) *w = d->w;
  if (nStride) *nStride = d->ns;
  if (cStride) *cStride = d->cs;
  if (hStride) *hStride = d->hs;
  if (wStride) *wStride = d->ws;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyTensorDescriptor(cudnnTensorDescriptor_t tensorDesc) {
  return tensors().take(tensorDesc) ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_BAD_PARAM;
}

// ---------------------------------------------------------------- filters --
cudnnStatus_t cudnnCreateFilterDescriptor(cudnnFilterDescriptor_t* filterDesc) {
  if (filterDesc == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto h = filters().add<cudnnFilterDescriptor_t>(std::make_shared<FilterDesc>());
  if (h == nullptr) return CUDNN_STATUS_ALLOC_FAILED;
  *filterDesc = h;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetFilter4dDescriptor(cudnnFilterDescriptor_t filterDesc,
                                         cudnnDataType_t dataType, cudnnTensorFormat_t format,
                                         int k, int c, int h, int w) {
  auto d = filters().get(filterDesc);
  if (!d || k <= 0 || c <= 0 || h <= 0 || w <= 0) return CUDNN_STATUS_BAD_PARAM;
  if (format != CUDNN_TENSOR_NCHW && format != CUDNN_TENSOR_NHWC) return CUDNN_STATUS_BAD_PARAM;
  if (dataType == CUDNN_DATA_DOUBLE) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!supported_dtype(dataType)) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  d->configured = true;
  d->dtype = dataType;
  d->format = format;
  d->k = k;
  d->c = c;
  d->h = h;
  d->w = w;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetFilter4dDescriptor(cudnnFilterDescriptor_t filterDesc,
                                         cudnnDataType_t* dataType, cudnnTensorFormat_t* format,
                                         int* k, int* c, int* h, int* w) {
  auto d = filters().get(filterDesc);
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  if (!d->configured) return CUDNN_STATUS_BAD_PARAM;
  if (dataType) *dataType = d->dtype;
  if (format) *format = d->format;
  if (k) *k = d->k;
  if (c) *c = d->c;
  if (h) *h = d->h;
  if (w) *w = d->w;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyFilterDescriptor(cudnnFilterDescriptor_t filterDesc) {
  return filters().take(filterDesc) ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_BAD_PARAM;
}

// ------------------------------------------------------------ convolution --
cudnnStatus_t cudnnCreateConvolutionDescriptor(cudnnConvolutionDescriptor_t* convDesc) {
  if (convDesc == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto h = convs().add<cudnnConvolutionDescriptor_t>(std::make_shared<ConvDesc>());
  if (h == nullptr) return CUDNN_STATUS_ALLOC_FAILED;
  *convDesc = h;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetConvolution2dDescriptor(cudnnConvolutionDescriptor_t convDesc, int pad_h,
                                              int pad_w, int u, int v, int dilation_h,
                                              int dilation_w, cudnnConvolutionMode_t mode,
                                              cudnnDataType_t computeType) {
  auto d = convs().get(convDesc);
  if (!d || pad_h < 0 || pad_w < 0 || u <= 0 || v <= 0 || dilation_h <= 0 || dilation_w <= 0)
    return CUDNN_STATUS_BAD_PARAM;
  if (mode != CUDNN_CONVOLUTION && mode != CUDNN_CROSS_CORRELATION) return CUDNN_STATUS_BAD_PARAM;
  if (computeType == CUDNN_DATA_DOUBLE) return CUDNN_STATUS_NOT_SUPPORTED;
  std::lock_guard<std::mutex> g(d->mu);
  d->configured = true;
  d->pad_h = pad_h;
  d->pad_w = pad_w;
  d->stride_h = u;
  d->stride_w = v;
  d->dil_h = dilation_h;
  d->dil_w = dilation_w;
  d->mode = mode;
  d->compute = computeType;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetConvolutionGroupCount(cudnnConvolutionDescriptor_t convDesc, int groupCount) {
  auto d = convs().get(convDesc);
  if (!d || groupCount <= 0) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  d->groups = groupCount;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetConvolutionGroupCount(cudnnConvolutionDescriptor_t convDesc,
                                            int* groupCount) {
  if (groupCount == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto d = convs().get(convDesc);
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  *groupCount = d->groups;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetConvolution2dForwardOutputDim(cudnnConvolutionDescriptor_t convDesc,
                                                    cudnnTensorDescriptor_t inputTensorDesc,
                                                    cudnnFilterDescriptor_t filterDesc, int* n,
                                                    int* c, int* h, int* w) {
  auto cd = convs().get(convDesc);
  auto xd = tensors().get(inputTensorDesc);
  auto fd = filters().get(filterDesc);
  if (!cd || !xd || !fd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap xs = snap(*xd);
  int fk, fh, fw;
  bool fconf;
  {
    std::lock_guard<std::mutex> g(fd->mu);
    fconf = fd->configured;
    fk = fd->k;
    fh = fd->h;
    fw = fd->w;
  }
  int ph, pw, sh, sw, dh, dw;
  bool cconf;
  {
    std::lock_guard<std::mutex> g(cd->mu);
    cconf = cd->configured;
    ph = cd->pad_h;
    pw = cd->pad_w;
    sh = cd->stride_h;
    sw = cd->stride_w;
    dh = cd->dil_h;
    dw = cd->dil_w;
  }
  if (!cconf || !xs.configured || !fconf) return CUDNN_STATUS_BAD_PARAM;
  const int oh = 1 + (xs.v.h + 2 * ph - (1 + (fh - 1) * dh)) / sh;
  const int ow = 1 + (xs.v.w + 2 * pw - (1 + (fw - 1) * dw)) / sw;
  if (oh <= 0 || ow <= 0) return CUDNN_STATUS_BAD_PARAM;
  if (n) *n = xs.v.n;
  if (c) *c = fk;
  if (h) *h = oh;
  if (w) *w = ow;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyConvolutionDescriptor(cudnnConvolutionDescriptor_t convDesc) {
  return convs().take(convDesc) ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_BAD_PARAM;
}

cudnnStatus_t cudnnGetConvolutionForwardWorkspaceSize(
    cudnnHandle_t handle, cudnnTensorDescriptor_t xDesc, cudnnFilterDescriptor_t wDesc,
    cudnnConvolutionDescriptor_t convDesc, cudnnTensorDescriptor_t yDesc,
    cudnnConvolutionFwdAlgo_t algo, size_t* sizeInBytes) {
  (void)algo;
  if (sizeInBytes == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto xd = tensors().get(xDesc);
  auto fd = filters().get(wDesc);
  auto cd = convs().get(convDesc);
  auto yd = tensors().get(yDesc);
  if (!h || !xd || !fd || !cd || !yd) return CUDNN_STATUS_BAD_PARAM;
  ConvPlan plan{};
  if (!build_conv(*xd, *fd, *cd, *yd, &plan)) return CUDNN_STATUS_BAD_PARAM;
  *sizeInBytes = 0;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnConvolutionForward(cudnnHandle_t handle, const void* alpha,
                                      cudnnTensorDescriptor_t xDesc, const void* x,
                                      cudnnFilterDescriptor_t wDesc, const void* w,
                                      cudnnConvolutionDescriptor_t convDesc,
                                      cudnnConvolutionFwdAlgo_t algo, void* workSpace,
                                      size_t workSpaceSizeInBytes, const void* beta,
                                      cudnnTensorDescriptor_t yDesc, void* y) {
  (void)algo;
  (void)workSpace;
  (void)workSpaceSizeInBytes;
  if (alpha == nullptr || beta == nullptr || x == nullptr || w == nullptr || y == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto xd = tensors().get(xDesc);
  auto fd = filters().get(wDesc);
  auto cd = convs().get(convDesc);
  auto yd = tensors().get(yDesc);
  if (!h || !xd || !fd || !cd || !yd) return CUDNN_STATUS_BAD_PARAM;
  ConvPlan plan{};
  const float a = *static_cast<const float*>(alpha);
  const float b = *static_cast<const float*>(beta);
  if (!build_conv(*xd, *fd, *cd, *yd, &plan)) return CUDNN_STATUS_BAD_PARAM;
  mb200::dnn::ConvDtype dt;
  if (plan.dtype == CUDNN_DATA_FLOAT) {
    dt = mb200::dnn::ConvDtype::kF32;
  } else if (plan.dtype == CUDNN_DATA_BFLOAT16) {
    dt = mb200::dnn::ConvDtype::kBF16;
  } else {
    return CUDNN_STATUS_NOT_SUPPORTED;  // fp32 only in the reference (cudnn_ops.mm:134-137)
  }
  if (!mb200::device_span_ok(x, plan.x_bytes) || !mb200::device_span_ok(w, plan.w_bytes) ||
      !mb200::device_span_ok(y, plan.y_bytes))
    return CUDNN_STATUS_BAD_PARAM;
  const cudaStream_t st = stream_of(*h);
  const std::size_t need =
      dt == mb200::dnn::ConvDtype::kF32 ? mb200::dnn::conv_tf32x3_workspace(plan.shape) : 0;
  if (need == 0) {
    const cudaError_t e = mb200::dnn::launch_conv(x, w, y, plan.shape, dt, a, b, nullptr, 0, st);
    return e == cudaSuccess ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_EXECUTION_FAILED;
  }
  if (workSpace != nullptr && workSpaceSizeInBytes >= need && mb200::aligned_to(workSpace, 16) &&
      mb200::device_span_ok(workSpace, need)) {
    const cudaError_t e =
        mb200::dnn::launch_conv(x, w, y, plan.shape, dt, a, b, workSpace, need, st);
    return e == cudaSuccess ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_EXECUTION_FAILED;
  }
  std::lock_guard<std::mutex> lk(h->ws_mu);
  const int dev = mb200::current_device();
  if (!h->ws || h->ws->bytes < need || h->ws->device != dev) {
    h->ws.reset();
    h->ws = mb200::DeviceBuffer::make(need);
  }
  void* wsp = h->ws ? h->ws->ptr : nullptr;
  const std::size_t wsb = h->ws ? h->ws->bytes : 0;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) cap = cudaStreamCaptureStatusNone;
  const bool ordered = cap == cudaStreamCaptureStatusNone && wsp != nullptr;
  if (ordered && h->ws_done != nullptr && cudaStreamWaitEvent(st, h->ws_done, 0) != cudaSuccess)
    return CUDNN_STATUS_EXECUTION_FAILED;
  const cudaError_t e = mb200::dnn::launch_conv(x, w, y, plan.shape, dt, a, b, wsp, wsb, st);
  if (e != cudaSuccess) return CUDNN_STATUS_EXECUTION_FAILED;
  if (ordered) {
    if (h->ws_done == nullptr &&
        cudaEventCreateWithFlags(&h->ws_done, cudaEventDisableTiming) != cudaSuccess) {
      h->ws_done = nullptr;
      return CUDNN_STATUS_EXECUTION_FAILED;
    }
    if (cudaEventRecord(h->ws_done, st) != cudaSuccess) return CUDNN_STATUS_EXECUTION_FAILED;
  }
  return CUDNN_STATUS_SUCCESS;
}

// ---------------------------------------------------------------- softmax --
cudnnStatus_t cudnnSoftmaxForward(cudnnHandle_t handle, cudnnSoftmaxAlgorithm_t algo,
                                  cudnnSoftmaxMode_t mode, const void* alpha,
                                  cudnnTensorDescriptor_t xDesc, const void* x, const void* beta,
                                  cudnnTensorDescriptor_t yDesc, void* y) {
  if (alpha == nullptr || beta == nullptr || x == nullptr || y == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto xd = tensors().get(xDesc);
  auto yd = tensors().get(yDesc);
  if (!h || !xd || !yd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap xs = snap(*xd), ys = snap(*yd);
  if (!xs.configured || !ys.configured) return CUDNN_STATUS_BAD_PARAM;
  if (xs.v.n != ys.v.n || xs.v.c != ys.v.c || xs.v.h != ys.v.h || xs.v.w != ys.v.w)
    return CUDNN_STATUS_BAD_PARAM;
  if (algo != CUDNN_SOFTMAX_FAST && algo != CUDNN_SOFTMAX_ACCURATE && algo != CUDNN_SOFTMAX_LOG)
    return CUDNN_STATUS_BAD_PARAM;
  if (mode != CUDNN_SOFTMAX_MODE_INSTANCE && mode != CUDNN_SOFTMAX_MODE_CHANNEL)
    return CUDNN_STATUS_BAD_PARAM;
  if (xs.dtype != CUDNN_DATA_FLOAT || ys.dtype != CUDNN_DATA_FLOAT)
    return CUDNN_STATUS_NOT_SUPPORTED;
  if (!mb200::device_span_ok(x, span_elems(xs.v) * 4) ||
      !mb200::device_span_ok(y, span_elems(ys.v) * 4))
    return CUDNN_STATUS_BAD_PARAM;
  const float a = *static_cast<const float*>(alpha);
  const float b = *static_cast<const float*>(beta);
  const auto al = static_cast<mb200::dnn::SoftmaxAlgo>(algo);
  const cudaStream_t st = stream_of(*h);
  const auto* xp = static_cast<const float*>(x);
  auto* yp = static_cast<float*>(y);
  const std::int64_t hw = static_cast<std::int64_t>(xs.v.h) * xs.v.w;
  cudaError_t e;
  // Contiguous slices become rows: whole packed NCHW instances (the reference's
  // warp path, cudnn_ops.mm:656-682), or the channel vector of each pixel of a
  // packed NHWC tensor.
  if (packed_nchw(xs.v) && packed_nchw(ys.v) && (mode == CUDNN_SOFTMAX_MODE_INSTANCE || hw == 1)) {
    e = mb200::dnn::launch_softmax_rows(xp, yp, xs.v.n, xs.v.c * hw, al, a, b, st);
  } else if (mode == CUDNN_SOFTMAX_MODE_CHANNEL && packed_nhwc(xs.v) && packed_nhwc(ys.v)) {
    e = mb200::dnn::launch_softmax_rows(xp, yp, xs.v.n * hw, xs.v.c, al, a, b, st);
  } else {
    e = mb200::dnn::launch_softmax_strided(xp, xs.v, yp, ys.v, mode == CUDNN_SOFTMAX_MODE_INSTANCE,
                                           al, a, b, st);
  }
  return e == cudaSuccess ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_EXECUTION_FAILED;
}

// ------------------------------------------- activation / pooling descriptors --
// cudnn_descriptors.mm:382-484
cudnnStatus_t cudnnCreateActivationDescriptor(cudnnActivationDescriptor_t* activationDesc) {
  if (activationDesc == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto h = activations().add<cudnnActivationDescriptor_t>(std::make_shared<ActivationDesc>());
  if (h == nullptr) return CUDNN_STATUS_ALLOC_FAILED;
  *activationDesc = h;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetActivationDescriptor(cudnnActivationDescriptor_t activationDesc,
                                           cudnnActivationMode_t mode,
                                           cudnnNanPropagation_t reluNanOpt, double coef) {
  auto d = activations().get(activationDesc);
  if (!d || mode < CUDNN_ACTIVATION_SIGMOID || mode > CUDNN_ACTIVATION_SWISH)
    return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  d->configured = true;
  d->mode = mode;
  d->nan_opt = reluNanOpt;
  d->coef = coef;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetActivationDescriptor(cudnnActivationDescriptor_t activationDesc,
                                           cudnnActivationMode_t* mode,
                                           cudnnNanPropagation_t* reluNanOpt, double* coef) {
  auto d = activations().get(activationDesc);
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  if (!d->configured) return CUDNN_STATUS_BAD_PARAM;
  if (mode != nullptr) *mode = d->mode;
  if (reluNanOpt != nullptr) *reluNanOpt = d->nan_opt;
  if (coef != nullptr) *coef = d->coef;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyActivationDescriptor(cudnnActivationDescriptor_t activationDesc) {
  return activations().take(activationDesc) ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_BAD_PARAM;
}

cudnnStatus_t cudnnCreatePoolingDescriptor(cudnnPoolingDescriptor_t* poolingDesc) {
  if (poolingDesc == nullptr) return CUDNN_STATUS_BAD_PARAM;
  auto h = poolings().add<cudnnPoolingDescriptor_t>(std::make_shared<PoolingDesc>());
  if (h == nullptr) return CUDNN_STATUS_ALLOC_FAILED;
  *poolingDesc = h;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetPooling2dDescriptor(cudnnPoolingDescriptor_t poolingDesc,
                                          cudnnPoolingMode_t mode,
                                          cudnnNanPropagation_t maxpoolingNanOpt, int windowHeight,
                                          int windowWidth, int verticalPadding,
                                          int horizontalPadding, int verticalStride,
                                          int horizontalStride) {
  auto d = poolings().get(poolingDesc);
  if (!d || windowHeight <= 0 || windowWidth <= 0 || verticalPadding < 0 ||
      horizontalPadding < 0 || verticalStride <= 0 || horizontalStride <= 0)
    return CUDNN_STATUS_BAD_PARAM;
  if (mode < CUDNN_POOLING_MAX || mode > CUDNN_POOLING_MAX_DETERMINISTIC)
    return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(d->mu);
  d->configured = true;
  d->mode = mode;
  d->nan_opt = maxpoolingNanOpt;
  d->win_h = windowHeight;
  d->win_w = windowWidth;
  d->pad_h = verticalPadding;
  d->pad_w = horizontalPadding;
  d->stride_h = verticalStride;
  d->stride_w = horizontalStride;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetPooling2dForwardOutputDim(cudnnPoolingDescriptor_t poolingDesc,
                                                cudnnTensorDescriptor_t inputTensorDesc, int* n,
                                                int* c, int* h, int* w) {
  auto pd = poolings().get(poolingDesc);
  auto xd = tensors().get(inputTensorDesc);
  if (!pd || !xd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap xs = snap(*xd);
  PoolingDesc p;
  {
    std::lock_guard<std::mutex> g(pd->mu);
    p.configured = pd->configured;
    p.win_h = pd->win_h;
    p.win_w = pd->win_w;
    p.pad_h = pd->pad_h;
    p.pad_w = pd->pad_w;
    p.stride_h = pd->stride_h;
    p.stride_w = pd->stride_w;
  }
  if (!p.configured || !xs.configured) return CUDNN_STATUS_BAD_PARAM;
  const int oh = 1 + (xs.v.h + 2 * p.pad_h - p.win_h) / p.stride_h;
  const int ow = 1 + (xs.v.w + 2 * p.pad_w - p.win_w) / p.stride_w;
  if (oh <= 0 || ow <= 0) return CUDNN_STATUS_BAD_PARAM;
  if (n != nullptr) *n = xs.v.n;
  if (c != nullptr) *c = xs.v.c;
  if (h != nullptr) *h = oh;
  if (w != nullptr) *w = ow;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyPoolingDescriptor(cudnnPoolingDescriptor_t poolingDesc) {
  return poolings().take(poolingDesc) ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_BAD_PARAM;
}

// cudnn_descriptors.mm:486-500
cudnnStatus_t cudnnDeriveBNTensorDescriptor(cudnnTensorDescriptor_t derivedBnDesc,
                                            cudnnTensorDescriptor_t xDesc,
                                            cudnnBatchNormMode_t mode) {
  auto xd = tensors().get(xDesc);
  if (!xd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap xs = snap(*xd);
  if (!xs.configured) return CUDNN_STATUS_BAD_PARAM;
  const cudnnDataType_t t = xs.dtype == CUDNN_DATA_HALF ? CUDNN_DATA_FLOAT : xs.dtype;
  if (mode == CUDNN_BATCHNORM_PER_ACTIVATION)
    return cudnnSetTensor4dDescriptor(derivedBnDesc, CUDNN_TENSOR_NCHW, t, 1, xs.v.c, xs.v.h,
                                      xs.v.w);
  return cudnnSetTensor4dDescriptor(derivedBnDesc, CUDNN_TENSOR_NCHW, t, 1, xs.v.c, 1, 1);
}

}  // extern "C"

namespace {

bool all_float(std::initializer_list<cudnnDataType_t> ts) {
  for (auto t : ts)
    if (t != CUDNN_DATA_FLOAT) return false;
  return true;
}

bool spans_ok(std::initializer_list<std::pair<const void*, std::size_t>> spans) {
  for (const auto& s : spans)
    if (!mb200::device_span_ok(s.first, s.second * sizeof(float))) return false;
  return true;
}

// Runs fn(workspace) with `need` bytes of the handle's workspace, ordered after the
// previous call that used it (the same protocol as the forward convolution).
template <class Fn>
cudnnStatus_t with_workspace(DnnContext& h, std::size_t need, cudaStream_t st, Fn&& fn) {
  std::lock_guard<std::mutex> lk(h.ws_mu);
  const int dev = mb200::current_device();
  if (!h.ws || h.ws->bytes < need || h.ws->device != dev) {
    h.ws.reset();
    h.ws = mb200::DeviceBuffer::make(need);
    if (!h.ws) return CUDNN_STATUS_ALLOC_FAILED;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) cap = cudaStreamCaptureStatusNone;
  const bool ordered = cap == cudaStreamCaptureStatusNone;
  if (ordered && h.ws_done != nullptr && cudaStreamWaitEvent(st, h.ws_done, 0) != cudaSuccess)
    return CUDNN_STATUS_EXECUTION_FAILED;
  if (fn(h.ws->ptr) != cudaSuccess) return CUDNN_STATUS_EXECUTION_FAILED;
  if (ordered) {
    if (h.ws_done == nullptr &&
        cudaEventCreateWithFlags(&h.ws_done, cudaEventDisableTiming) != cudaSuccess) {
      h.ws_done = nullptr;
      return CUDNN_STATUS_EXECUTION_FAILED;
    }
    if (cudaEventRecord(h.ws_done, st) != cudaSuccess) return CUDNN_STATUS_EXECUTION_FAILED;
  }
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t status_of(cudaError_t e) {
  return e == cudaSuccess ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_EXECUTION_FAILED;
}

}  // namespace

extern "C" {

// cudnn_ops.mm:195-259
cudnnStatus_t cudnnConvolutionBackwardData(cudnnHandle_t handle, const void* alpha,
                                           cudnnFilterDescriptor_t wDesc, const void* w,
                                           cudnnTensorDescriptor_t dyDesc, const void* dy,
                                           cudnnConvolutionDescriptor_t convDesc,
                                           cudnnConvolutionBwdDataAlgo_t algo, void* workSpace,
                                           size_t workSpaceSizeInBytes, const void* beta,
                                           cudnnTensorDescriptor_t dxDesc, void* dx) {
  (void)algo;
  (void)workSpace;
  (void)workSpaceSizeInBytes;
  if (alpha == nullptr || beta == nullptr || w == nullptr || dy == nullptr || dx == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto dxd = tensors().get(dxDesc);
  auto fd = filters().get(wDesc);
  auto cd = convs().get(convDesc);
  auto dyd = tensors().get(dyDesc);
  if (!h || !dxd || !fd || !cd || !dyd) return CUDNN_STATUS_BAD_PARAM;
  ConvPlan plan{};
  if (!build_conv(*dxd, *fd, *cd, *dyd, &plan)) return CUDNN_STATUS_BAD_PARAM;
  if (plan.dtype != CUDNN_DATA_FLOAT) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!mb200::device_span_ok(w, plan.w_bytes) || !mb200::device_span_ok(dy, plan.y_bytes) ||
      !mb200::device_span_ok(dx, plan.x_bytes))
    return CUDNN_STATUS_BAD_PARAM;
  const float a = *static_cast<const float*>(alpha), b = *static_cast<const float*>(beta);
  const cudaStream_t st = stream_of(*h);
  const auto* wp = static_cast<const float*>(w);
  const auto* dyp = static_cast<const float*>(dy);
  auto* dxp = static_cast<float*>(dx);
  const std::size_t need = mb200::dnn::conv_bwd_data_tc_workspace(plan.shape);
  if (need > 0) {
    return with_workspace(*h, need, st, [&](void* ws) {
      const cudaError_t e =
          mb200::dnn::launch_conv_bwd_data_tc(wp, dyp, dxp, plan.shape, a, b, ws, need, st);
      return e == cudaErrorNotSupported
                 ? mb200::dnn::launch_conv_bwd_data(wp, dyp, dxp, plan.shape, a, b, st)
                 : e;
    });
  }
  return status_of(mb200::dnn::launch_conv_bwd_data(wp, dyp, dxp, plan.shape, a, b, st));
}

// cudnn_ops.mm:261-323
cudnnStatus_t cudnnConvolutionBackwardFilter(cudnnHandle_t handle, const void* alpha,
                                             cudnnTensorDescriptor_t xDesc, const void* x,
                                             cudnnTensorDescriptor_t dyDesc, const void* dy,
                                             cudnnConvolutionDescriptor_t convDesc,
                                             cudnnConvolutionBwdFilterAlgo_t algo, void* workSpace,
                                             size_t workSpaceSizeInBytes, const void* beta,
                                             cudnnFilterDescriptor_t dwDesc, void* dw) {
  (void)algo;
  (void)workSpace;
  (void)workSpaceSizeInBytes;
  if (alpha == nullptr || beta == nullptr || x == nullptr || dy == nullptr || dw == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto xd = tensors().get(xDesc);
  auto fd = filters().get(dwDesc);
  auto cd = convs().get(convDesc);
  auto dyd = tensors().get(dyDesc);
  if (!h || !xd || !fd || !cd || !dyd) return CUDNN_STATUS_BAD_PARAM;
  ConvPlan plan{};
  if (!build_conv(*xd, *fd, *cd, *dyd, &plan)) return CUDNN_STATUS_BAD_PARAM;
  if (plan.dtype != CUDNN_DATA_FLOAT) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!mb200::device_span_ok(x, plan.x_bytes) || !mb200::device_span_ok(dy, plan.y_bytes) ||
      !mb200::device_span_ok(dw, plan.w_bytes))
    return CUDNN_STATUS_BAD_PARAM;
  const float a = *static_cast<const float*>(alpha), b = *static_cast<const float*>(beta);
  const cudaStream_t st = stream_of(*h);
  const std::size_t tc_need = mb200::dnn::conv_bwd_filter_tc_workspace(plan.shape);
  const std::size_t simt_need = mb200::dnn::conv_bwd_filter_workspace(plan.shape);
  return with_workspace(*h, std::max(tc_need, simt_need), st, [&](void* ws) {
    const auto* xp = static_cast<const float*>(x);
    const auto* dyp = static_cast<const float*>(dy);
    auto* dwp = static_cast<float*>(dw);
    if (tc_need > 0) {
      const cudaError_t e =
          mb200::dnn::launch_conv_bwd_filter_tc(xp, dyp, dwp, plan.shape, a, b, ws, tc_need, st);
      if (e != cudaErrorNotSupported) return e;
    }
    return mb200::dnn::launch_conv_bwd_filter(xp, dyp, dwp, plan.shape, a, b,
                                              static_cast<float*>(ws), st);
  });
}

// cudnn_ops.mm:325-383
cudnnStatus_t cudnnConvolutionBackwardBias(cudnnHandle_t handle, const void* alpha,
                                           cudnnTensorDescriptor_t dyDesc, const void* dy,
                                           const void* beta, cudnnTensorDescriptor_t dbDesc,
                                           void* db) {
  if (alpha == nullptr || beta == nullptr || dy == nullptr || db == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto dyd = tensors().get(dyDesc);
  auto dbd = tensors().get(dbDesc);
  if (!h || !dyd || !dbd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap ys = snap(*dyd), bs = snap(*dbd);
  if (!ys.configured || !bs.configured) return CUDNN_STATUS_BAD_PARAM;
  if (bs.v.n != 1 || bs.v.c != ys.v.c || bs.v.h != 1 || bs.v.w != 1) return CUDNN_STATUS_BAD_PARAM;
  if (!all_float({ys.dtype, bs.dtype})) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!spans_ok({{dy, span_elems(ys.v)}, {db, static_cast<std::size_t>(bs.v.c)}}))
    return CUDNN_STATUS_BAD_PARAM;
  return status_of(mb200::dnn::launch_conv_bwd_bias(
      static_cast<const float*>(dy), ys.v, static_cast<float*>(db),
      *static_cast<const float*>(alpha), *static_cast<const float*>(beta), stream_of(*h)));
}

// cudnn_ops.mm:385-451
cudnnStatus_t cudnnAddTensor(cudnnHandle_t handle, const void* alpha, cudnnTensorDescriptor_t aDesc,
                             const void* A, const void* beta, cudnnTensorDescriptor_t cDesc,
                             void* C) {
  if (alpha == nullptr || beta == nullptr || A == nullptr || C == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto ad = tensors().get(aDesc);
  auto cdd = tensors().get(cDesc);
  if (!h || !ad || !cdd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap as = snap(*ad), cs = snap(*cdd);
  if (!as.configured || !cs.configured) return CUDNN_STATUS_BAD_PARAM;
  if ((as.v.n != 1 && as.v.n != cs.v.n) || (as.v.c != 1 && as.v.c != cs.v.c) ||
      (as.v.h != 1 && as.v.h != cs.v.h) || (as.v.w != 1 && as.v.w != cs.v.w))
    return CUDNN_STATUS_BAD_PARAM;
  if (!all_float({as.dtype, cs.dtype})) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!spans_ok({{A, span_elems(as.v)}, {C, span_elems(cs.v)}})) return CUDNN_STATUS_BAD_PARAM;
  return status_of(mb200::dnn::launch_add_tensor(
      static_cast<const float*>(A), as.v, static_cast<float*>(C), cs.v,
      *static_cast<const float*>(alpha), *static_cast<const float*>(beta), stream_of(*h)));
}

// cudnn_ops.mm:453-548
cudnnStatus_t cudnnActivationForward(cudnnHandle_t handle,
                                     cudnnActivationDescriptor_t activationDesc, const void* alpha,
                                     cudnnTensorDescriptor_t xDesc, const void* x, const void* beta,
                                     cudnnTensorDescriptor_t yDesc, void* y) {
  if (alpha == nullptr || beta == nullptr || x == nullptr || y == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto act = activations().get(activationDesc);
  auto xd = tensors().get(xDesc);
  auto yd = tensors().get(yDesc);
  if (!h || !act || !xd || !yd) return CUDNN_STATUS_BAD_PARAM;
  int mode;
  float coef;
  {
    std::lock_guard<std::mutex> g(act->mu);
    if (!act->configured) return CUDNN_STATUS_BAD_PARAM;
    mode = static_cast<int>(act->mode);
    coef = static_cast<float>(act->coef);
  }
  const TensorSnap xs = snap(*xd), ys = snap(*yd);
  if (!xs.configured || !ys.configured) return CUDNN_STATUS_BAD_PARAM;
  if (xs.v.n != ys.v.n || xs.v.c != ys.v.c || xs.v.h != ys.v.h || xs.v.w != ys.v.w)
    return CUDNN_STATUS_BAD_PARAM;
  if (!all_float({xs.dtype, ys.dtype})) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!spans_ok({{x, span_elems(xs.v)}, {y, span_elems(ys.v)}})) return CUDNN_STATUS_BAD_PARAM;
  return status_of(mb200::dnn::launch_activation(
      static_cast<const float*>(x), xs.v, static_cast<float*>(y), ys.v, mode, coef,
      *static_cast<const float*>(alpha), *static_cast<const float*>(beta), stream_of(*h)));
}

// cudnn_ops.mm:550-623
cudnnStatus_t cudnnPoolingForward(cudnnHandle_t handle, cudnnPoolingDescriptor_t poolingDesc,
                                  const void* alpha, cudnnTensorDescriptor_t xDesc, const void* x,
                                  const void* beta, cudnnTensorDescriptor_t yDesc, void* y) {
  if (alpha == nullptr || beta == nullptr || x == nullptr || y == nullptr)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto pd = poolings().get(poolingDesc);
  auto xd = tensors().get(xDesc);
  auto yd = tensors().get(yDesc);
  if (!h || !pd || !xd || !yd) return CUDNN_STATUS_BAD_PARAM;
  mb200::dnn::PoolShape p{};
  {
    std::lock_guard<std::mutex> g(pd->mu);
    if (!pd->configured) return CUDNN_STATUS_BAD_PARAM;
    p.win_h = pd->win_h;
    p.win_w = pd->win_w;
    p.pad_h = pd->pad_h;
    p.pad_w = pd->pad_w;
    p.stride_h = pd->stride_h;
    p.stride_w = pd->stride_w;
    p.mode = static_cast<int>(pd->mode);
  }
  const TensorSnap xs = snap(*xd), ys = snap(*yd);
  if (!xs.configured || !ys.configured) return CUDNN_STATUS_BAD_PARAM;
  if (xs.v.n != ys.v.n || xs.v.c != ys.v.c) return CUDNN_STATUS_BAD_PARAM;
  if (!all_float({xs.dtype, ys.dtype})) return CUDNN_STATUS_NOT_SUPPORTED;
  if (!spans_ok({{x, span_elems(xs.v)}, {y, span_elems(ys.v)}})) return CUDNN_STATUS_BAD_PARAM;
  p.x = xs.v;
  p.y = ys.v;
  return status_of(mb200::dnn::launch_pooling(
      static_cast<const float*>(x), static_cast<float*>(y), p, *static_cast<const float*>(alpha),
      *static_cast<const float*>(beta), stream_of(*h)));
}

// cudnn_ops.mm:722-802
cudnnStatus_t cudnnBatchNormalizationForwardInference(
    cudnnHandle_t handle, cudnnBatchNormMode_t mode, const void* alpha, const void* beta,
    cudnnTensorDescriptor_t xDesc, const void* x, cudnnTensorDescriptor_t yDesc, void* y,
    cudnnTensorDescriptor_t bnScaleBiasMeanVarDesc, const void* bnScale, const void* bnBias,
    const void* estimatedMean, const void* estimatedVariance, double epsilon) {
  if (alpha == nullptr || beta == nullptr || x == nullptr || y == nullptr || bnScale == nullptr ||
      bnBias == nullptr || estimatedMean == nullptr || estimatedVariance == nullptr ||
      epsilon <= 0.0)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto xd = tensors().get(xDesc);
  auto yd = tensors().get(yDesc);
  auto bd = tensors().get(bnScaleBiasMeanVarDesc);
  if (!h || !xd || !yd || !bd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap xs = snap(*xd), ys = snap(*yd), bs = snap(*bd);
  if (!xs.configured || !ys.configured || !bs.configured) return CUDNN_STATUS_BAD_PARAM;
  if (xs.v.n != ys.v.n || xs.v.c != ys.v.c || xs.v.h != ys.v.h || xs.v.w != ys.v.w)
    return CUDNN_STATUS_BAD_PARAM;
  if (!all_float({xs.dtype, ys.dtype})) return CUDNN_STATUS_NOT_SUPPORTED;
  const bool per_act = mode == CUDNN_BATCHNORM_PER_ACTIVATION;
  const std::size_t pe = per_act ? static_cast<std::size_t>(xs.v.c) * xs.v.h * xs.v.w
                                 : static_cast<std::size_t>(xs.v.c);
  if (!spans_ok({{x, span_elems(xs.v)}, {y, span_elems(ys.v)}, {bnScale, pe}, {bnBias, pe},
                 {estimatedMean, pe}, {estimatedVariance, pe}}))
    return CUDNN_STATUS_BAD_PARAM;
  return status_of(mb200::dnn::launch_bn_inference(
      static_cast<const float*>(x), xs.v, static_cast<float*>(y), ys.v,
      static_cast<const float*>(bnScale), static_cast<const float*>(bnBias),
      static_cast<const float*>(estimatedMean), static_cast<const float*>(estimatedVariance),
      per_act, static_cast<float>(epsilon), *static_cast<const float*>(alpha),
      *static_cast<const float*>(beta), stream_of(*h)));
}

// cudnn_ops.mm:804-902 (the mode argument is ignored there: statistics are always
// per channel)
cudnnStatus_t cudnnBatchNormalizationForwardTraining(
    cudnnHandle_t handle, cudnnBatchNormMode_t mode, const void* alpha, const void* beta,
    cudnnTensorDescriptor_t xDesc, const void* x, cudnnTensorDescriptor_t yDesc, void* y,
    cudnnTensorDescriptor_t bnScaleBiasMeanVarDesc, const void* bnScale, const void* bnBias,
    double exponentialAverageFactor, void* resultRunningMean, void* resultRunningVariance,
    double epsilon, void* resultSaveMean, void* resultSaveInvVariance) {
  (void)mode;
  if (alpha == nullptr || beta == nullptr || x == nullptr || y == nullptr || bnScale == nullptr ||
      bnBias == nullptr || epsilon <= 0.0)
    return CUDNN_STATUS_BAD_PARAM;
  auto h = handles().get(handle);
  auto xd = tensors().get(xDesc);
  auto yd = tensors().get(yDesc);
  auto bd = tensors().get(bnScaleBiasMeanVarDesc);
  if (!h || !xd || !yd || !bd) return CUDNN_STATUS_BAD_PARAM;
  const TensorSnap xs = snap(*xd), ys = snap(*yd), bs = snap(*bd);
  if (!xs.configured || !ys.configured || !bs.configured) return CUDNN_STATUS_BAD_PARAM;
  if (xs.v.n != ys.v.n || xs.v.c != ys.v.c || xs.v.h != ys.v.h || xs.v.w != ys.v.w)
    return CUDNN_STATUS_BAD_PARAM;
  if (!all_float({xs.dtype, ys.dtype})) return CUDNN_STATUS_NOT_SUPPORTED;
  const auto ce = static_cast<std::size_t>(xs.v.c);
  if (!spans_ok({{x, span_elems(xs.v)}, {y, span_elems(ys.v)}, {bnScale, ce}, {bnBias, ce}}))
    return CUDNN_STATUS_BAD_PARAM;
  const bool has_running = resultRunningMean != nullptr || resultRunningVariance != nullptr;
  if (has_running && (resultRunningMean == nullptr || resultRunningVariance == nullptr ||
                      !spans_ok({{resultRunningMean, ce}, {resultRunningVariance, ce}})))
    return CUDNN_STATUS_BAD_PARAM;
  const bool has_save = resultSaveMean != nullptr || resultSaveInvVariance != nullptr;
  if (has_save && (resultSaveMean == nullptr || resultSaveInvVariance == nullptr ||
                   !spans_ok({{resultSaveMean, ce}, {resultSaveInvVariance, ce}})))
    return CUDNN_STATUS_BAD_PARAM;
  const cudaStream_t st = stream_of(*h);
  auto run = [&](void* ws) {
    return mb200::dnn::launch_bn_training(
        static_cast<const float*>(x), xs.v, static_cast<float*>(y), ys.v,
        static_cast<const float*>(bnScale), static_cast<const float*>(bnBias),
        static_cast<float*>(has_running ? resultRunningMean : nullptr),
        static_cast<float*>(has_running ? resultRunningVariance : nullptr),
        static_cast<float*>(has_save ? resultSaveMean : nullptr),
        static_cast<float*>(has_save ? resultSaveInvVariance : nullptr),
        static_cast<float>(exponentialAverageFactor), static_cast<float>(epsilon),
        *static_cast<const float*>(alpha), *static_cast<const float*>(beta),
        static_cast<float*>(ws), st);
  };
  const std::size_t need = mb200::dnn::bn_training_workspace(xs.v);
  if (need == 0) return status_of(run(nullptr));
  return with_workspace(*h, need, st, run);
}

}  // extern "C"
