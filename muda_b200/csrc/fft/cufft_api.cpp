// cufft_api.cpp — cuFFT C ABI: plans and C2C execution.
//
// Mirrors libraries/fft/src/cufft_plan.mm and cufft_exec.mm of the reference:
// same entry points and status codes, the same effective-stride rules
// (inembed == NULL forces unit stride and the dense batch distance,
// cufft_plan.mm:68-83), the same transform conventions (sign, no scaling,
// in-place allowed) and the same axis order for 2-D/3-D transforms (innermost
// axis first, cufft_exec.mm:190-199).
//
// A plan owns device twiddle tables (shared between plans through an LRU keyed
// by device and length) and, for power-of-two lengths above the single-pass
// limit, a workspace for the two-pass split; cufftGetSize reports those bytes.
#pragma GCC visibility push(default)
#include "cufft.h"
#pragma GCC visibility pop

#include <cuda_runtime_api.h>

#include <algorithm>
#include <array>
#include <cstdint>
#include <memory>
#include <mutex>
#include <utility>
#include <vector>

#include "common/device.hpp"
#include "common/lru.hpp"
#include "common/registry.hpp"
#include "fft/fft.hpp"

namespace {

using mb200::DeviceBuffer;
using mb200::fft::Batch1D;

constexpr std::int64_t kMaxSplit = mb200::fft::kMaxSinglePass * mb200::fft::kMaxSinglePass;
constexpr std::size_t kSplitWorkspaceBytes = std::size_t{256} << 20;

bool is_pow2(std::int64_t n) { return n > 0 && (n & (n - 1)) == 0; }

// How one axis of length n is transformed.
enum class AxisKind { kTrivial, kSinglePass, kDirect, kSplit };

AxisKind axis_kind(std::int64_t n) {
  if (n == 1) return AxisKind::kTrivial;
  if (mb200::fft::single_pass_supported(n)) return AxisKind::kSinglePass;
  if (!is_pow2(n) && n <= mb200::fft::kMaxDirect) return AxisKind::kDirect;
  if (is_pow2(n) && n <= kMaxSplit) return AxisKind::kSplit;
  return AxisKind::kTrivial;  // unsupported; rejected by plan()
}

bool axis_supported(std::int64_t n) {
  return n == 1 || mb200::fft::single_pass_supported(n) ||
         (!is_pow2(n) && n <= mb200::fft::kMaxDirect) || (is_pow2(n) && n <= kMaxSplit);
}

// Twiddle tables exp(-2*pi*i*m/n), shared per (device, n).
mb200::LruCache<std::pair<int, std::int64_t>, DeviceBuffer>& twiddle_cache() {
  static mb200::LruCache<std::pair<int, std::int64_t>, DeviceBuffer> c(128);
  return c;
}

std::shared_ptr<DeviceBuffer> twiddles(std::int64_t n) {
  const int dev = mb200::current_device();
  auto key = std::make_pair(dev, n);
  if (auto hit = twiddle_cache().find(key)) return hit;
  auto buf = DeviceBuffer::make(static_cast<std::size_t>(n) * sizeof(float2));
  if (!buf) return nullptr;
  std::vector<float2> host(static_cast<std::size_t>(n));
  mb200::fft::host_twiddles(n, host.data());
  if (cudaMemcpy(buf->ptr, host.data(), host.size() * sizeof(float2), cudaMemcpyHostToDevice) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  twiddle_cache().put(key, buf);
  return buf;
}

struct Plan {
  std::mutex mu;
  bool configured = false;
  int rank = 1;
  std::array<std::int64_t, 3> dims{1, 1, 1};
  std::int64_t batch = 1;
  cufftType type = CUFFT_C2C;
  std::int64_t istride = 1, idist = 0, ostride = 1, odist = 0;
  cudaStream_t stream = nullptr;
  int device = -1;
  std::vector<std::shared_ptr<DeviceBuffer>> tables;  // keeps twiddles alive
  std::array<const float2*, 3> axis_tw{};              // per axis
  // two-pass split of a long power-of-two axis (rank 1 only)
  std::int64_t n1 = 0, n2 = 0;
  const float2* tw_n1 = nullptr;
  const float2* tw_n2 = nullptr;
  const float2* tw_total = nullptr;
  std::shared_ptr<DeviceBuffer> workspace;
  std::int64_t split_chunk = 0;  // transforms per workspace fill
  std::size_t work_bytes = 0;
};

using PlanTable = mb200::Registry<Plan, mb200::ObjKind::kFftPlan>;
PlanTable& plans() {
  static PlanTable t;
  return t;
}

std::int64_t elems_per_batch(const Plan& p) {
  std::int64_t e = 1;
  for (int i = 0; i < p.rank; ++i) e *= p.dims[i];
  return e;
}

// ConfigurePlanState (libraries/fft/src/cufft_plan.mm:36-137).
cufftResult configure(Plan& p, int rank, const int* n, const int* inembed, int istride, int idist,
                      const int* onembed, int ostride, int odist, cufftType type, int batch,
                      size_t* work) {
  if (n == nullptr || rank < 1 || rank > 3 || batch <= 0) return CUFFT_INVALID_VALUE;
  if (type == CUFFT_Z2Z || type == CUFFT_D2Z || type == CUFFT_Z2D) return CUFFT_NOT_SUPPORTED;
  if (type != CUFFT_C2C && type != CUFFT_R2C && type != CUFFT_C2R) return CUFFT_INVALID_TYPE;
  std::array<std::int64_t, 3> dims{1, 1, 1};
  std::int64_t total = 1;
  for (int i = 0; i < rank; ++i) {
    if (n[i] <= 0) return CUFFT_INVALID_SIZE;
    dims[i] = n[i];
    total *= n[i];
  }
  // Real-data transforms are outside this library's hot path.
  if (type != CUFFT_C2C) return CUFFT_NOT_SUPPORTED;
  for (int i = 0; i < rank; ++i) {
    if (!axis_supported(dims[i])) return CUFFT_NOT_SUPPORTED;
    if (rank > 1 && axis_kind(dims[i]) == AxisKind::kSplit) return CUFFT_NOT_SUPPORTED;
  }
  const std::int64_t eis = (inembed != nullptr) ? istride : 1;
  const std::int64_t eos = (onembed != nullptr) ? ostride : 1;
  if (eis <= 0 || eos <= 0) return CUFFT_INVALID_VALUE;
  const std::int64_t eid = (inembed != nullptr && idist > 0) ? idist : total;
  const std::int64_t eod = (onembed != nullptr && odist > 0) ? odist : total;
  if (mb200::current_device() < 0) return CUFFT_SETUP_FAILED;

  std::lock_guard<std::mutex> g(p.mu);
  p.configured = false;
  p.tables.clear();
  p.workspace.reset();
  p.rank = rank;
  p.dims = dims;
  p.batch = batch;
  p.type = type;
  p.istride = eis;
  p.idist = eid;
  p.ostride = eos;
  p.odist = eod;
  p.device = mb200::current_device();
  p.work_bytes = 0;
  auto hold = [&](std::int64_t len) -> const float2* {
    auto t = twiddles(len);
    if (!t) return nullptr;
    p.tables.push_back(t);
    p.work_bytes += t->bytes;
    return static_cast<const float2*>(t->ptr);
  };
  for (int i = 0; i < rank; ++i) {
    p.axis_tw[i] = nullptr;
    if (axis_kind(dims[i]) == AxisKind::kSinglePass || axis_kind(dims[i]) == AxisKind::kDirect) {
      p.axis_tw[i] = hold(dims[i]);
      if (p.axis_tw[i] == nullptr) return CUFFT_ALLOC_FAILED;
    }
  }
  if (rank == 1 && axis_kind(dims[0]) == AxisKind::kSplit) {
    int l = 0;
    while ((std::int64_t{1} << l) < dims[0]) ++l;
    p.n1 = std::int64_t{1} << (l / 2);
    p.n2 = dims[0] / p.n1;
    p.tw_n1 = hold(p.n1);
    p.tw_n2 = hold(p.n2);
    p.tw_total = hold(dims[0]);
    if (!p.tw_n1 || !p.tw_n2 || !p.tw_total) return CUFFT_ALLOC_FAILED;
    const std::int64_t per = dims[0] * static_cast<std::int64_t>(sizeof(float2));
    p.split_chunk = std::max<std::int64_t>(
        1, std::min<std::int64_t>(batch, static_cast<std::int64_t>(kSplitWorkspaceBytes) / per));
    p.workspace = DeviceBuffer::make(static_cast<std::size_t>(p.split_chunk * per));
    if (!p.workspace) return CUFFT_ALLOC_FAILED;
    p.work_bytes += p.workspace->bytes;
  }
  if (p.work_bytes == 0) p.work_bytes = 1;  // plans always report a non-zero size
  p.configured = true;
  if (work != nullptr) *work = p.work_bytes;
  return CUFFT_SUCCESS;
}

cudaError_t run_axis(std::int64_t n, int sign, const Batch1D& b, const float2* tw,
                     cudaStream_t st) {
  switch (axis_kind(n)) {
    case AxisKind::kSinglePass: {
      Batch1D c = b;
      c.tw = tw;
      return mb200::fft::launch_stockham(n, sign, c, st);
    }
    case AxisKind::kDirect: {
      Batch1D c = b;
      c.tw = tw;
      return mb200::fft::launch_direct_dft(n, sign, c, st);
    }
    default:
      return cudaErrorInvalidValue;
  }
}

// Length-N = n1*n2 transform in two passes through the workspace:
//   pass A, per (b, r2): length-n1 transform over t = n2*r1 + r2, output k1 scaled by
//           W_N^{r2*k1}, stored at ws[b][k1*n2 + r2];
//   pass B, per (b, k1): length-n2 transform over r2, output k2 stored at X[k1 + n1*k2].
cudaError_t run_split(const Plan& p, const float2* in, float2* out, int sign, cudaStream_t st) {
  const std::int64_t n = p.dims[0];
  auto* ws = static_cast<float2*>(p.workspace->ptr);
  for (std::int64_t b0 = 0; b0 < p.batch; b0 += p.split_chunk) {
    const std::int64_t nb = std::min(p.split_chunk, p.batch - b0);
    Batch1D a{};
    a.in = in + b0 * p.idist;
    a.out = ws;
    a.in_stride = p.n2 * p.istride;
    a.in_outer = p.idist;
    a.in_inner = p.istride;
    a.out_stride = p.n2;
    a.out_outer = n;
    a.out_inner = 1;
    a.batch = nb * p.n2;
    a.inner_count = p.n2;
    a.tw = p.tw_n1;
    a.post_tw = p.tw_total;
    a.post_n = n;
    cudaError_t e = mb200::fft::launch_stockham(p.n1, sign, a, st);
    if (e != cudaSuccess) return e;
    Batch1D c{};
    c.in = ws;
    c.out = out + b0 * p.odist;
    c.in_stride = 1;
    c.in_outer = n;
    c.in_inner = p.n2;
    c.out_stride = p.n1 * p.ostride;
    c.out_outer = p.odist;
    c.out_inner = p.ostride;
    c.batch = nb * p.n1;
    c.inner_count = p.n1;
    c.tw = p.tw_n2;
    c.post_tw = nullptr;
    c.post_n = 1;
    e = mb200::fft::launch_stockham(p.n2, sign, c, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cufftResult make_plan(cufftHandle* plan, int rank, int* n, int* inembed, int istride, int idist,
                      int* onembed, int ostride, int odist, cufftType type, int batch);

}  // namespace

extern "C" {

cufftResult cufftCreate(cufftHandle* handle) {
  if (handle == nullptr) return CUFFT_INVALID_VALUE;
  auto h = plans().add<cufftHandle>(std::make_shared<Plan>());
  if (h == nullptr) return CUFFT_ALLOC_FAILED;
  *handle = h;
  return CUFFT_SUCCESS;
}

cufftResult cufftMakePlan1d(cufftHandle plan, int nx, cufftType type, int batch,
                            size_t* workSize) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  const int dims[1] = {nx};
  return configure(*p, 1, dims, nullptr, 1, 0, nullptr, 1, 0, type, batch, workSize);
}

cufftResult cufftMakePlanMany(cufftHandle plan, int rank, int* n, int* inembed, int istride,
                              int idist, int* onembed, int ostride, int odist, cufftType type,
                              int batch, size_t* workSize) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  return configure(*p, rank, n, inembed, istride, idist, onembed, ostride, odist, type, batch,
                   workSize);
}

cufftResult cufftPlan1d(cufftHandle* plan, int nx, cufftType type, int batch) {
  int dims[1] = {nx};
  return make_plan(plan, 1, dims, nullptr, 1, 0, nullptr, 1, 0, type, batch);
}

cufftResult cufftPlanMany(cufftHandle* plan, int rank, int* n, int* inembed, int istride,
                          int idist, int* onembed, int ostride, int odist, cufftType type,
                          int batch) {
  return make_plan(plan, rank, n, inembed, istride, idist, onembed, ostride, odist, type, batch);
}

cufftResult cufftSetStream(cufftHandle plan, cudaStream_t stream) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  std::lock_guard<std::mutex> g(p->mu);
  p->stream = stream;
  return CUFFT_SUCCESS;
}

cufftResult cufftGetSize(cufftHandle handle, size_t* workSize) {
  if (workSize == nullptr) return CUFFT_INVALID_VALUE;
  auto p = plans().get(handle);
  if (!p) return CUFFT_INVALID_PLAN;
  std::lock_guard<std::mutex> g(p->mu);
  if (!p->configured) return CUFFT_INVALID_PLAN;
  *workSize = p->work_bytes;
  return CUFFT_SUCCESS;
}

cufftResult cufftDestroy(cufftHandle plan) {
  return plans().take(plan) ? CUFFT_SUCCESS : CUFFT_INVALID_PLAN;
}

cufftResult cufftExecC2C(cufftHandle plan, cufftComplex* idata, cufftComplex* odata,
                         int direction) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  std::lock_guard<std::mutex> g(p->mu);
  if (!p->configured) return CUFFT_INVALID_PLAN;
  if (idata == nullptr || odata == nullptr ||
      (direction != CUFFT_FORWARD && direction != CUFFT_INVERSE))
    return CUFFT_INVALID_VALUE;
  if (p->type != CUFFT_C2C) return CUFFT_INVALID_TYPE;
  if (mb200::current_device() != p->device) return CUFFT_INVALID_DEVICE;
  const std::int64_t epb = elems_per_batch(*p);
  const std::size_t in_span =
      static_cast<std::size_t>((p->batch - 1) * p->idist + (epb - 1) * p->istride + 1);
  const std::size_t out_span =
      static_cast<std::size_t>((p->batch - 1) * p->odist + (epb - 1) * p->ostride + 1);
  if (!mb200::device_span_ok(idata, in_span * sizeof(float2)) ||
      !mb200::device_span_ok(odata, out_span * sizeof(float2)) || !mb200::aligned_to(idata, 8) ||
      !mb200::aligned_to(odata, 8))
    return CUFFT_INVALID_VALUE;
  // In place requires the same layout on both sides: each transform is read
  // completely before it is written, but a different output layout would
  // overwrite elements of transforms that have not been read yet.
  if (idata == odata && (p->istride != p->ostride || p->idist != p->odist))
    return CUFFT_INVALID_VALUE;
  const int sign = (direction == CUFFT_FORWARD) ? -1 : 1;
  const cudaStream_t st = p->stream;
  cudaError_t e = cudaSuccess;

  if (p->rank == 1) {
    const std::int64_t n = p->dims[0];
    if (axis_kind(n) == AxisKind::kSplit) {
      e = run_split(*p, idata, odata, sign, st);
    } else if (n == 1) {
      if (idata != odata || p->istride != p->ostride || p->idist != p->odist) {
        for (std::int64_t b = 0; b < p->batch && e == cudaSuccess; ++b)
          e = cudaMemcpyAsync(odata + b * p->odist, idata + b * p->idist, sizeof(float2),
                              cudaMemcpyDeviceToDevice, st);
      }
    } else {
      Batch1D b{};
      b.in = idata;
      b.out = odata;
      b.in_stride = p->istride;
      b.in_outer = p->idist;
      b.in_inner = 0;
      b.out_stride = p->ostride;
      b.out_outer = p->odist;
      b.out_inner = 0;
      b.batch = p->batch;
      b.inner_count = 1;
      b.post_n = 1;
      e = run_axis(n, sign, b, p->axis_tw[0], st);
    }
    return e == cudaSuccess ? CUFFT_SUCCESS : CUFFT_EXEC_FAILED;
  }

  // Multi-dimensional: innermost axis reads the input, the others run in place
  // on the output.  Logical element (o, t, i) of axis a sits at
  // o*L*S + t*S + i with L = dims[a], S = product of the later dims.
  bool first = true;
  for (int a = p->rank - 1; a >= 0 && e == cudaSuccess; --a) {
    const std::int64_t L = p->dims[a];
    std::int64_t S = 1, Pr = 1;
    for (int i = a + 1; i < p->rank; ++i) S *= p->dims[i];
    for (int i = 0; i < a; ++i) Pr *= p->dims[i];
    // A length-1 axis is the identity; the next axis then reads the input.
    if (L == 1) continue;
    const float2* src = first ? idata : odata;
    const std::int64_t s_str = first ? p->istride : p->ostride;
    const std::int64_t s_dist = first ? p->idist : p->odist;
    const bool dense = (s_dist == epb * s_str) && (p->odist == epb * p->ostride);
    const std::int64_t nb_loop = (S == 1 || dense) ? 1 : p->batch;
    for (std::int64_t bl = 0; bl < nb_loop && e == cudaSuccess; ++bl) {
      Batch1D b{};
      b.in = src + bl * s_dist;
      b.out = odata + bl * p->odist;
      b.in_stride = S * s_str;
      b.out_stride = S * p->ostride;
      b.post_n = 1;
      b.inner_count = S;
      b.in_inner = s_str;
      b.out_inner = p->ostride;
      if (nb_loop == 1 && S == 1) {
        // (batch, o) -> contiguous rows of length L
        b.batch = p->batch * Pr;
        b.inner_count = Pr;
        b.in_outer = s_dist;
        b.in_inner = L * s_str;
        b.out_outer = p->odist;
        b.out_inner = L * p->ostride;
        b.in_stride = s_str;
        b.out_stride = p->ostride;
      } else if (nb_loop == 1) {
        // dense batches: (batch, o) fold into one outer index of stride L*S
        b.batch = p->batch * Pr * S;
        b.in_outer = L * S * s_str;
        b.out_outer = L * S * p->ostride;
      } else {
        b.batch = Pr * S;
        b.in_outer = L * S * s_str;
        b.out_outer = L * S * p->ostride;
      }
      e = run_axis(L, sign, b, p->axis_tw[a], st);
    }
    first = false;
  }
  if (first && e == cudaSuccess) {
    // every axis has length 1: the transform is the identity
    for (std::int64_t b = 0; b < p->batch && e == cudaSuccess && idata != odata; ++b)
      e = cudaMemcpyAsync(odata + b * p->odist, idata + b * p->idist, sizeof(float2),
                          cudaMemcpyDeviceToDevice, st);
  }
  return e == cudaSuccess ? CUFFT_SUCCESS : CUFFT_EXEC_FAILED;
}

}  // extern "C"

namespace {

cufftResult make_plan(cufftHandle* plan, int rank, int* n, int* inembed, int istride, int idist,
                      int* onembed, int ostride, int odist, cufftType type, int batch) {
  if (plan == nullptr) return CUFFT_INVALID_VALUE;
  cufftHandle h = nullptr;
  cufftResult r = cufftCreate(&h);
  if (r != CUFFT_SUCCESS) return r;
  r = cufftMakePlanMany(h, rank, n, inembed, istride, idist, onembed, ostride, odist, type, batch,
                        nullptr);
  if (r != CUFFT_SUCCESS) {
    (void)cufftDestroy(h);
    return r;
  }
  *plan = h;
  return CUFFT_SUCCESS;
}

}  // namespace
