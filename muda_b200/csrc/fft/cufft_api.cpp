// cufft_api.cpp — cuFFT C ABI: plans, C2C, R2C and C2R execution.
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
//
// Real-data plans (R2C, C2R; cufft_exec.mm:213-438): an even last axis L with
// unit-stride reals runs as a length-L/2 complex FFT of the reals read as pairs
// plus one post-pass (R2C) or pre-pass (C2R) of fft/real_kernels.cu; other
// layouts gather into complex rows, transform and scatter, as the reference does.
// Leading axes run on the half spectrum.  The plan owns the workspace.
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
enum class AxisKind {
  kTrivial, kSinglePass, kMixed, kDirect, kBluestein, kBluesteinGlobal, kSplit, kUnsupported
};

AxisKind axis_kind(std::int64_t n) {
  if (n == 1) return AxisKind::kTrivial;
  if (mb200::fft::single_pass_supported(n)) return AxisKind::kSinglePass;
  if (!is_pow2(n) && n < mb200::fft::kMinBluestein) return AxisKind::kDirect;
  if (!is_pow2(n) && mb200::fft::mixed_radix_supported(n)) return AxisKind::kMixed;
  if (!is_pow2(n) && n <= mb200::fft::kMaxBluestein) return AxisKind::kBluestein;
  if (!is_pow2(n) && n <= mb200::fft::kMaxBluesteinGlobal) return AxisKind::kBluesteinGlobal;
  if (is_pow2(n) && n <= kMaxSplit) return AxisKind::kSplit;
  return AxisKind::kUnsupported;
}

bool axis_supported(std::int64_t n) { return axis_kind(n) != AxisKind::kUnsupported; }

// True when run_axis transforms an axis of length n for any Batch1D layout (the
// power-of-two split is a rank-1 plan of its own).
bool one_pass(std::int64_t n) {
  const AxisKind k = axis_kind(n);
  return k == AxisKind::kTrivial || k == AxisKind::kSinglePass || k == AxisKind::kMixed ||
         k == AxisKind::kDirect || k == AxisKind::kBluestein || k == AxisKind::kBluesteinGlobal;
}

// Workspace per global-memory Bluestein axis (chunks of transforms).
constexpr std::size_t kBluesteinWsBytes = std::size_t{256} << 20;

// Tables the transform of one axis reads.
struct AxisTables {
  const float2* tw = nullptr;     // exp(-2*pi*i*m/n): single-pass and direct axes
  const float2* chirp = nullptr;  // Bluestein axes: chirp, FFT of the chirp filter,
  const float2* bhat = nullptr;   // and the inner length's twiddles
  const float2* tw_m = nullptr;
  mb200::fft::BluesteinGlobal glob{};  // longer Bluestein axes: tables and workspace
};

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
  if (n > mb200::fft::kMaxHostTwiddles) {
    // long tables on the device (the host loop would take seconds); ready before return
    if (mb200::fft::build_twiddles(static_cast<float2*>(buf->ptr), n, nullptr) != cudaSuccess ||
        cudaStreamSynchronize(nullptr) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    twiddle_cache().put(key, buf);
    return buf;
  }
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

// Bluestein tables of length n (chirp, then bhat at an even offset), shared per
// (device, n) in the twiddle cache under the key (device, -n).  Lengths above
// kMaxHostBluestein are built on the device with the FFT resources of `g`.
std::shared_ptr<DeviceBuffer> bluestein_tables(std::int64_t n,
                                               const mb200::fft::BluesteinGlobal* g = nullptr) {
  const int dev = mb200::current_device();
  auto key = std::make_pair(dev, -n);
  if (auto hit = twiddle_cache().find(key)) return hit;
  const std::int64_t mb = mb200::fft::bluestein_length(n);
  const std::int64_t off = (n + 1) / 2 * 2;
  auto buf = DeviceBuffer::make(static_cast<std::size_t>(off + mb) * sizeof(float2));
  if (!buf) return nullptr;
  if (n > mb200::fft::kMaxHostBluestein) {
    float2* base = static_cast<float2*>(buf->ptr);
    if (g == nullptr ||
        mb200::fft::build_bluestein_tables(n, base, base + off, *g, nullptr) != cudaSuccess ||
        cudaStreamSynchronize(nullptr) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    twiddle_cache().put(key, buf);
    return buf;
  }
  std::vector<float2> host(static_cast<std::size_t>(off + mb));
  mb200::fft::host_bluestein_tables(n, mb, host.data(), host.data() + off);
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
  std::array<AxisTables, 3> axis_tw{};                 // per axis
  // two-pass split of a long power-of-two axis (rank 1 only)
  std::int64_t n1 = 0, n2 = 0;
  const float2* tw_n1 = nullptr;
  const float2* tw_n2 = nullptr;
  const float2* tw_total = nullptr;
  std::shared_ptr<DeviceBuffer> workspace;
  std::int64_t split_chunk = 0;  // transforms per workspace fill
  std::size_t work_bytes = 0;
  // real-data plans: last axis L, half length M, half-spectrum length H = L/2 + 1
  std::int64_t L = 0, M = 0, H = 0, prefix = 1;
  bool packed = false;          // even L with unit-stride reals: length-M complex FFT
  const float2* tw_L = nullptr;  // exp(-2*pi*i*m/L)
  const float2* tw_M = nullptr;
  AxisTables ax_L, ax_M;         // transforms of length L (general path) and M (packed)
  std::shared_ptr<DeviceBuffer> real_ws;
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
  const bool real = type != CUFFT_C2C;
  const std::int64_t L = dims[rank - 1];
  const std::int64_t H = L / 2 + 1;
  const std::int64_t herm_total = total / L * H;
  if (real) {
    // every complex transform a real plan runs must take one pass (no split)
    for (int i = 0; i + 1 < rank; ++i)
      if (!one_pass(dims[i])) return CUFFT_NOT_SUPPORTED;
    const bool packed_ok = L % 2 == 0 && L >= 4 && one_pass(L / 2);
    if (!packed_ok && !one_pass(L)) return CUFFT_NOT_SUPPORTED;
  } else {
    for (int i = 0; i < rank; ++i) {
      if (!axis_supported(dims[i])) return CUFFT_NOT_SUPPORTED;
      if (rank > 1 && axis_kind(dims[i]) == AxisKind::kSplit) return CUFFT_NOT_SUPPORTED;
    }
  }
  const std::int64_t eis = (inembed != nullptr) ? istride : 1;
  const std::int64_t eos = (onembed != nullptr) ? ostride : 1;
  if (eis <= 0 || eos <= 0) return CUFFT_INVALID_VALUE;
  // default distances (cufft_plan.mm:74-79): the half spectrum is the dense complex side
  const std::int64_t def_id = type == CUFFT_C2R ? herm_total : total;
  const std::int64_t def_od = type == CUFFT_R2C ? herm_total : total;
  const std::int64_t eid = (inembed != nullptr && idist > 0) ? idist : def_id;
  const std::int64_t eod = (onembed != nullptr && odist > 0) ? odist : def_od;
  if (mb200::current_device() < 0) return CUFFT_SETUP_FAILED;

  std::lock_guard<std::mutex> g(p.mu);
  p.configured = false;
  p.tables.clear();
  p.workspace.reset();
  p.real_ws.reset();
  p.packed = false;
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
  auto keep = [&](std::shared_ptr<DeviceBuffer> t) -> const float2* {
    if (!t) return nullptr;
    p.tables.push_back(t);
    p.work_bytes += t->bytes;
    return static_cast<const float2*>(t->ptr);
  };
  auto hold = [&](std::int64_t len) { return keep(twiddles(len)); };
  // the tables (and workspace) a transform of length len over `count` rows needs
  auto axis_tables = [&](std::int64_t len, std::int64_t count, AxisTables& t) -> bool {
    t = AxisTables{};
    switch (axis_kind(len)) {
      case AxisKind::kSinglePass:
      case AxisKind::kMixed:
      case AxisKind::kDirect:
        t.tw = hold(len);
        return t.tw != nullptr;
      case AxisKind::kBluestein: {
        t.tw_m = hold(mb200::fft::bluestein_length(len));
        t.chirp = keep(bluestein_tables(len));
        t.bhat = t.chirp ? t.chirp + (len + 1) / 2 * 2 : nullptr;
        return t.tw_m != nullptr && t.chirp != nullptr;
      }
      case AxisKind::kBluesteinGlobal: {
        const std::int64_t mb = mb200::fft::bluestein_length(len);
        auto& g = t.glob;
        g.tw_m = hold(mb);
        if (g.tw_m == nullptr) return false;
        const std::int64_t row_bytes = mb * static_cast<std::int64_t>(sizeof(float2));
        g.ws_rows = std::max<std::int64_t>(
            1, std::min<std::int64_t>(count, static_cast<std::int64_t>(kBluesteinWsBytes) /
                                                 row_bytes));
        const auto bytes = static_cast<std::size_t>(g.ws_rows * row_bytes);
        g.ws = const_cast<float2*>(keep(DeviceBuffer::make(bytes)));
        if (g.ws == nullptr) return false;
        if (mb > mb200::fft::kMaxSinglePass) {
          int l = 0;
          while ((std::int64_t{1} << l) < mb) ++l;
          g.n1 = std::int64_t{1} << (l / 2);
          g.n2 = mb / g.n1;
          g.tw_n1 = hold(g.n1);
          g.tw_n2 = hold(g.n2);
          g.ws2 = const_cast<float2*>(keep(DeviceBuffer::make(bytes)));
          if (g.tw_n1 == nullptr || g.tw_n2 == nullptr || g.ws2 == nullptr) return false;
        }
        // the tables last: long ones are built with the FFT resources set up above
        g.chirp = keep(bluestein_tables(len, &g));
        if (g.chirp == nullptr) return false;
        g.bhat = g.chirp + (len + 1) / 2 * 2;
        return true;
      }
      default:
        return true;
    }
  };
  for (int i = 0; i < rank; ++i) {
    p.axis_tw[i] = AxisTables{};
    if (real && i == rank - 1) continue;  // the last axis of a real plan: below
    const std::int64_t count = batch * (real ? herm_total : total) / dims[i];
    if (!axis_tables(dims[i], count, p.axis_tw[i])) return CUFFT_ALLOC_FAILED;
  }
  if (real) {
    p.L = L;
    p.H = H;
    p.M = L / 2;
    p.prefix = total / L;
    const bool packed_ok = L % 2 == 0 && L >= 4 && one_pass(p.M);
    p.packed = packed_ok && (type == CUFFT_R2C ? (eis == 1 && eid % 2 == 0)
                                               : (eos == 1 && eod % 2 == 0));
    p.tw_L = p.tw_M = nullptr;
    p.ax_L = p.ax_M = AxisTables{};
    if (L > 1) {
      // the post-/pre-passes read exp(-2*pi*i*m/L) whatever the kind of L
      p.tw_L = hold(L);
      if (p.tw_L == nullptr) return CUFFT_ALLOC_FAILED;
      // the general path (odd L, strided or 4-byte aligned reals) transforms length L
      if (one_pass(L) && !axis_tables(L, batch * p.prefix, p.ax_L)) return CUFFT_ALLOC_FAILED;
    }
    if (packed_ok) {
      if (!axis_tables(p.M, batch * p.prefix, p.ax_M)) return CUFFT_ALLOC_FAILED;
      p.tw_M = p.ax_M.tw;  // the fused kernels' table (power-of-two M)
    }
    const std::int64_t rows = batch * p.prefix;
    const std::int64_t need =
        p.packed ? rows * (p.M + (type == CUFFT_C2R && rank > 1 ? H : 0))
                 : rows * (L + (type == CUFFT_C2R ? H : 0));
    p.real_ws = DeviceBuffer::make(static_cast<std::size_t>(need) * sizeof(float2));
    if (!p.real_ws) return CUFFT_ALLOC_FAILED;
    p.work_bytes += p.real_ws->bytes;
  }
  if (!real && rank == 1 && axis_kind(dims[0]) == AxisKind::kSplit) {
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

cudaError_t run_axis(std::int64_t n, int sign, const Batch1D& b, const AxisTables& t,
                     cudaStream_t st) {
  switch (axis_kind(n)) {
    case AxisKind::kSinglePass: {
      Batch1D c = b;
      c.tw = t.tw;
      return mb200::fft::launch_stockham(n, sign, c, st);
    }
    case AxisKind::kDirect: {
      Batch1D c = b;
      c.tw = t.tw;
      return mb200::fft::launch_direct_dft(n, sign, c, st);
    }
    case AxisKind::kMixed: {
      Batch1D c = b;
      c.tw = t.tw;
      return mb200::fft::launch_mixed_radix(n, sign, c, st);
    }
    case AxisKind::kBluestein:
      return mb200::fft::launch_bluestein(n, sign, b, t.chirp, t.bhat, t.tw_m, st);
    case AxisKind::kBluesteinGlobal:
      return mb200::fft::launch_bluestein_global(n, sign, b, t.glob, st);
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

// Transforms axes a_hi .. 0 (innermost first) of `batch` row-major arrays of
// complex elements with dims[0 .. rank) (dims[rank - 1] innermost; axes above
// a_hi are left alone).  The first axis of length > 1 reads `in` (element stride
// is, batch distance id) and writes `out` (os, od); the later ones run in place on
// `out`.  *moved reports whether any axis had length > 1.
cudaError_t run_axes(int rank, const std::array<std::int64_t, 3>& dims, int a_hi,
                     const std::array<AxisTables, 3>& tw, const float2* in, std::int64_t is,
                     std::int64_t id, float2* out, std::int64_t os, std::int64_t od,
                     std::int64_t batch, int sign, cudaStream_t st, bool* moved) {
  cudaError_t e = cudaSuccess;
  std::int64_t epb = 1;
  for (int i = 0; i < rank; ++i) epb *= dims[i];
  bool first = true;
  // The first transformed axis reads the input, the others run in place on the
  // output.  Logical element (o, t, i) of axis a sits at
  // o*L*S + t*S + i with L = dims[a], S = product of the later dims.
  for (int a = a_hi; a >= 0 && e == cudaSuccess; --a) {
    const std::int64_t L = dims[a];
    std::int64_t S = 1, Pr = 1;
    for (int i = a + 1; i < rank; ++i) S *= dims[i];
    for (int i = 0; i < a; ++i) Pr *= dims[i];
    // A length-1 axis is the identity; the next axis then reads the input.
    if (L == 1) continue;
    const float2* src = first ? in : out;
    const std::int64_t s_str = first ? is : os;
    const std::int64_t s_dist = first ? id : od;
    const bool dense = (s_dist == epb * s_str) && (od == epb * os);
    const std::int64_t nb_loop = (S == 1 || dense) ? 1 : batch;
    for (std::int64_t bl = 0; bl < nb_loop && e == cudaSuccess; ++bl) {
      Batch1D b{};
      b.in = src + bl * s_dist;
      b.out = out + bl * od;
      b.in_stride = S * s_str;
      b.out_stride = S * os;
      b.post_n = 1;
      b.inner_count = S;
      b.in_inner = s_str;
      b.out_inner = os;
      if (nb_loop == 1 && S == 1) {
        // (batch, o) -> contiguous rows of length L
        b.batch = batch * Pr;
        b.inner_count = Pr;
        b.in_outer = s_dist;
        b.in_inner = L * s_str;
        b.out_outer = od;
        b.out_inner = L * os;
        b.in_stride = s_str;
        b.out_stride = os;
      } else if (nb_loop == 1) {
        // dense batches: (batch, o) fold into one outer index of stride L*S
        b.batch = batch * Pr * S;
        b.in_outer = L * S * s_str;
        b.out_outer = L * S * os;
      } else {
        b.batch = Pr * S;
        b.in_outer = L * S * s_str;
        b.out_outer = L * S * os;
      }
      e = run_axis(L, sign, b, tw[a], st);
    }
    first = false;
  }
  *moved = !first;
  return e;
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

cufftResult cufftMakePlan2d(cufftHandle plan, int nx, int ny, cufftType type, size_t* workSize) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  const int dims[2] = {nx, ny};
  return configure(*p, 2, dims, nullptr, 1, 0, nullptr, 1, 0, type, 1, workSize);
}

cufftResult cufftMakePlan3d(cufftHandle plan, int nx, int ny, int nz, cufftType type,
                            size_t* workSize) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  const int dims[3] = {nx, ny, nz};
  return configure(*p, 3, dims, nullptr, 1, 0, nullptr, 1, 0, type, 1, workSize);
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

cufftResult cufftPlan2d(cufftHandle* plan, int nx, int ny, cufftType type) {
  int dims[2] = {nx, ny};
  return make_plan(plan, 2, dims, nullptr, 1, 0, nullptr, 1, 0, type, 1);
}

cufftResult cufftPlan3d(cufftHandle* plan, int nx, int ny, int nz, cufftType type) {
  int dims[3] = {nx, ny, nz};
  return make_plan(plan, 3, dims, nullptr, 1, 0, nullptr, 1, 0, type, 1);
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

  bool moved = false;
  e = run_axes(p->rank, p->dims, p->rank - 1, p->axis_tw, idata, p->istride, p->idist, odata,
               p->ostride, p->odist, p->batch, sign, st, &moved);
  const bool first = !moved;
  if (first && e == cudaSuccess) {
    // every axis has length 1: the transform is the identity
    for (std::int64_t b = 0; b < p->batch && e == cudaSuccess && idata != odata; ++b)
      e = cudaMemcpyAsync(odata + b * p->odist, idata + b * p->idist, sizeof(float2),
                          cudaMemcpyDeviceToDevice, st);
  }
  return e == cudaSuccess ? CUFFT_SUCCESS : CUFFT_EXEC_FAILED;
}

// Length-M complex transforms of rows r = b * prefix + p: the reals of row r seen
// as M complex pairs at base + b * dist2 + p * M (complex units), dense rows at Z.
namespace {

Batch1D pair_rows(const Plan& p, const float2* in, std::int64_t in_dist2, float2* out,
                  std::int64_t out_dist2, bool reals_in) {
  Batch1D b{};
  b.in = in;
  b.out = out;
  b.in_stride = 1;
  b.out_stride = 1;
  b.inner_count = p.prefix;
  b.batch = p.batch * p.prefix;
  b.in_outer = reals_in ? in_dist2 : p.prefix * p.M;
  b.in_inner = p.M;
  b.out_outer = reals_in ? p.prefix * p.M : out_dist2;
  b.out_inner = p.M;
  b.post_n = 1;
  return b;
}

// Dense complex rows of length len at base (rows r = b * prefix + p contiguous).
Batch1D dense_rows(const Plan& p, float2* base, std::int64_t len) {
  Batch1D b{};
  b.in = base;
  b.out = base;
  b.in_stride = b.out_stride = 1;
  b.inner_count = 1;
  b.batch = p.batch * p.prefix;
  b.in_outer = b.out_outer = len;
  b.in_inner = b.out_inner = 0;
  b.post_n = 1;
  return b;
}

// The plan's dims with the last axis replaced by `last`.
std::array<std::int64_t, 3> with_last(const Plan& p, std::int64_t last) {
  std::array<std::int64_t, 3> d = p.dims;
  d[p.rank - 1] = last;
  return d;
}

// True when the byte ranges [a, a + na) and [b, b + nb) share an address.
bool overlap(const void* a, std::size_t na, const void* b, std::size_t nb) {
  const auto x = reinterpret_cast<std::uintptr_t>(a);
  const auto y = reinterpret_cast<std::uintptr_t>(b);
  return x < y + nb && y < x + na;
}

// Grows the plan's real-data workspace to `floats2` complex elements.
float2* real_workspace(Plan& p, std::int64_t floats2) {
  const std::size_t need = static_cast<std::size_t>(floats2) * sizeof(float2);
  if (!p.real_ws || p.real_ws->bytes < need) {
    p.real_ws.reset();
    p.real_ws = DeviceBuffer::make(need);
  }
  return p.real_ws ? static_cast<float2*>(p.real_ws->ptr) : nullptr;
}

}  // namespace

cufftResult cufftExecR2C(cufftHandle plan, cufftReal* idata, cufftComplex* odata) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  std::lock_guard<std::mutex> g(p->mu);
  if (!p->configured) return CUFFT_INVALID_PLAN;
  if (idata == nullptr || odata == nullptr) return CUFFT_INVALID_VALUE;
  if (p->type != CUFFT_R2C) return CUFFT_INVALID_TYPE;
  if (mb200::current_device() != p->device) return CUFFT_INVALID_DEVICE;
  const std::int64_t epb = elems_per_batch(*p);
  const std::int64_t hpb = p->prefix * p->H;
  const std::size_t in_span =
      static_cast<std::size_t>((p->batch - 1) * p->idist + (epb - 1) * p->istride + 1);
  const std::size_t out_span =
      static_cast<std::size_t>((p->batch - 1) * p->odist + (hpb - 1) * p->ostride + 1);
  if (!mb200::device_span_ok(idata, in_span * sizeof(float)) ||
      !mb200::device_span_ok(odata, out_span * sizeof(float2)) || !mb200::aligned_to(idata, 4) ||
      !mb200::aligned_to(odata, 8))
    return CUFFT_INVALID_VALUE;
  const cudaStream_t st = p->stream;
  const std::int64_t rows = p->batch * p->prefix;
  cudaError_t e = cudaSuccess;
  const bool dense = p->istride == 1 && p->idist == epb && p->ostride == 1 && p->odist == hpb &&
                     !overlap(idata, rows * p->L * sizeof(float), odata,
                              rows * p->H * sizeof(float2));
  const std::int64_t per =
      (p->packed && dense && mb200::fft::real_bulk_aligned(true, p->M, idata, odata))
          ? mb200::fft::real_bulk_rows_per_group(p->M)
          : 0;
  if (per > 0 && rows >= per) {
    // whole groups through the fused kernel, the remaining rows as dense rows below
    const std::int64_t groups = rows / per, done = groups * per;
    e = mb200::fft::launch_real_bulk(true, p->M, idata, odata, groups, p->tw_M, p->tw_L, st);
    if (e == cudaSuccess && done < rows) {
      float2* Z = real_workspace(*p, (rows - done) * p->M);
      if (Z == nullptr) return CUFFT_ALLOC_FAILED;
      Batch1D f = dense_rows(*p, Z, p->M);
      f.in = reinterpret_cast<const float2*>(idata) + done * p->M;
      f.batch = rows - done;
      e = run_axis(p->M, -1, f, p->ax_M, st);
      const mb200::fft::RealRows rr{rows - done, 1, p->M, p->tw_L};
      if (e == cudaSuccess)
        e = mb200::fft::launch_r2c_post(rr, Z, odata + done * p->H, p->H, 1, st);
    }
  } else if (p->packed && mb200::aligned_to(idata, 8)) {
    float2* Z = real_workspace(*p, rows * p->M);
    if (Z == nullptr) return CUFFT_ALLOC_FAILED;
    Batch1D f = pair_rows(*p, reinterpret_cast<const float2*>(idata), p->idist / 2, Z, 0, true);
    e = run_axis(p->M, -1, f, p->ax_M, st);
    const mb200::fft::RealRows rr{rows, p->prefix, p->M, p->tw_L};
    if (e == cudaSuccess) e = mb200::fft::launch_r2c_post(rr, Z, odata, p->odist, p->ostride, st);
  } else {
    float2* A = real_workspace(*p, rows * p->L);
    if (A == nullptr) return CUFFT_ALLOC_FAILED;
    e = mb200::fft::launch_gather_real(rows, p->prefix, p->L, idata, p->idist, p->istride, A, st);
    if (e == cudaSuccess && p->L > 1) {
      Batch1D b = dense_rows(*p, A, p->L);
      e = run_axis(p->L, -1, b, p->ax_L, st);
    }
    if (e == cudaSuccess)
      e = mb200::fft::launch_scatter_half(rows, p->prefix, p->L, A, odata, p->odist, p->ostride,
                                          st);
  }
  // leading axes on the half spectrum, in place on the output
  if (e == cudaSuccess && p->rank > 1) {
    bool moved = false;
    e = run_axes(p->rank, with_last(*p, p->H), p->rank - 2, p->axis_tw, odata, p->ostride,
                 p->odist, odata, p->ostride, p->odist, p->batch, -1, st, &moved);
  }
  return e == cudaSuccess ? CUFFT_SUCCESS : CUFFT_EXEC_FAILED;
}

cufftResult cufftExecC2R(cufftHandle plan, cufftComplex* idata, cufftReal* odata) {
  auto p = plans().get(plan);
  if (!p) return CUFFT_INVALID_PLAN;
  std::lock_guard<std::mutex> g(p->mu);
  if (!p->configured) return CUFFT_INVALID_PLAN;
  if (idata == nullptr || odata == nullptr) return CUFFT_INVALID_VALUE;
  if (p->type != CUFFT_C2R) return CUFFT_INVALID_TYPE;
  if (mb200::current_device() != p->device) return CUFFT_INVALID_DEVICE;
  const std::int64_t epb = elems_per_batch(*p);
  const std::int64_t hpb = p->prefix * p->H;
  const std::size_t in_span =
      static_cast<std::size_t>((p->batch - 1) * p->idist + (hpb - 1) * p->istride + 1);
  const std::size_t out_span =
      static_cast<std::size_t>((p->batch - 1) * p->odist + (epb - 1) * p->ostride + 1);
  if (!mb200::device_span_ok(idata, in_span * sizeof(float2)) ||
      !mb200::device_span_ok(odata, out_span * sizeof(float)) || !mb200::aligned_to(idata, 8) ||
      !mb200::aligned_to(odata, 4))
    return CUFFT_INVALID_VALUE;
  const cudaStream_t st = p->stream;
  const std::int64_t rows = p->batch * p->prefix;
  cudaError_t e = cudaSuccess;
  if (p->packed && mb200::aligned_to(odata, 8)) {
    const bool lead = p->rank > 1;
    float2* base = real_workspace(*p, rows * (p->M + (lead ? p->H : 0)));
    if (base == nullptr) return CUFFT_ALLOC_FAILED;
    float2* W = base;                           // leading axes: dense half spectrum
    float2* Z = base + (lead ? rows * p->H : 0);  // pre-pass output
    const float2* src = idata;
    std::int64_t sdist = p->idist, sstr = p->istride;
    if (lead) {
      bool moved = false;
      e = run_axes(p->rank, with_last(*p, p->H), p->rank - 2, p->axis_tw, idata, p->istride,
                   p->idist, W, 1, hpb, p->batch, +1, st, &moved);
      if (moved) {
        src = W;
        sdist = hpb;
        sstr = 1;
      }
    }
    const bool dense = sstr == 1 && sdist == hpb && p->ostride == 1 && p->odist == epb &&
                       mb200::fft::real_bulk_aligned(false, p->M, src, odata) &&
                       !overlap(src, rows * p->H * sizeof(float2), odata,
                                rows * p->L * sizeof(float));
    const std::int64_t per = dense ? mb200::fft::real_bulk_rows_per_group(p->M) : 0;
    std::int64_t done = 0;
    if (e == cudaSuccess && per > 0 && rows >= per) {
      const std::int64_t groups = rows / per;
      done = groups * per;
      e = mb200::fft::launch_real_bulk(false, p->M, src, odata, groups, p->tw_M, p->tw_L, st);
    }
    if (e == cudaSuccess && done > 0 && done < rows) {
      // the remaining dense rows
      const mb200::fft::RealRows rr{rows - done, 1, p->M, p->tw_L};
      e = mb200::fft::launch_c2r_pre(rr, src + done * p->H, p->H, 1, Z, st);
      if (e == cudaSuccess) {
        Batch1D b = dense_rows(*p, Z, p->M);
        b.out = reinterpret_cast<float2*>(odata) + done * p->M;
        b.batch = rows - done;
        e = run_axis(p->M, +1, b, p->ax_M, st);
      }
    } else if (e == cudaSuccess && done == 0) {
      const mb200::fft::RealRows rr{rows, p->prefix, p->M, p->tw_L};
      e = mb200::fft::launch_c2r_pre(rr, src, sdist, sstr, Z, st);
      if (e == cudaSuccess) {
        Batch1D b = pair_rows(*p, Z, 0, reinterpret_cast<float2*>(odata), p->odist / 2, false);
        e = run_axis(p->M, +1, b, p->ax_M, st);
      }
    }
  } else {
    float2* A = real_workspace(*p, rows * (p->H + p->L));
    if (A == nullptr) return CUFFT_ALLOC_FAILED;
    float2* B = A + rows * p->H;
    e = mb200::fft::launch_gather_half(rows, p->prefix, p->L, idata, p->idist, p->istride, A, st);
    if (e == cudaSuccess && p->rank > 1) {
      bool moved = false;
      e = run_axes(p->rank, with_last(*p, p->H), p->rank - 2, p->axis_tw, A, 1, hpb, A, 1, hpb,
                   p->batch, +1, st, &moved);
    }
    if (e == cudaSuccess) e = mb200::fft::launch_expand_half(rows, p->L, A, B, st);
    if (e == cudaSuccess && p->L > 1) {
      Batch1D b = dense_rows(*p, B, p->L);
      e = run_axis(p->L, +1, b, p->ax_L, st);
    }
    if (e == cudaSuccess)
      e = mb200::fft::launch_scatter_real(rows, p->prefix, p->L, B, odata, p->odist, p->ostride,
                                          st);
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
