// fft_static.cu — batched power-of-two C2C FFT that allocates nothing.
//
// cufftExecC2C needs a plan, and a plan allocates device memory for its
// twiddle tables and, above 16384 points, a workspace for the two-pass split.
// Some callers cannot allocate at the point where they need a transform: code
// running inside a custom allocator or memory-pool callback (re-entering
// cudaMalloc there deadlocks or recurses), real-time paths that forbid
// allocation after start-up, and processes working under a hard device-memory
// cap.  cufftExecC2CNoAlloc serves them: its tables and workspace live in one
// fixed array of device memory that belongs to this library (kScratchBytes,
// below), reserved when the library is loaded and held until the process exits.
//
// The kernels are the same Stockham kernels the planned path uses; only the
// memory they use for tables and workspace differs.
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <mutex>

#include "common/device.hpp"
#include "fft/fft.hpp"

#pragma GCC visibility push(default)
#include "cufft.h"
#pragma GCC visibility pop

namespace mb200::fft {
namespace {

// Largest transform length served, and the layout of the fixed array:
//   [workspace: kMaxLen complex][table n: kMaxLen][table n1: kMaxPass][table n2: kMaxPass]
constexpr std::int64_t kMaxLen = std::int64_t{1} << 20;
constexpr std::int64_t kMaxPass = kMaxSinglePass;
constexpr std::int64_t kScratchElems = 2 * kMaxLen + 2 * kMaxPass;
constexpr std::size_t kScratchBytes = static_cast<std::size_t>(kScratchElems) * sizeof(float2);
static_assert(kScratchBytes <= (std::size_t{17} << 20), "the fixed scratch stays below 17 MiB");

// The fixed scratch array (about 16.3 MiB on every device that loads the library).
static __device__ __align__(256) float2 g_scratch[kScratchElems];

// tw[m] = exp(-2*pi*i*m/n), m < n, from sincospi in double (2m/n is exact for n a
// power of two), rounded once to float like the planned path's host tables.
__global__ void fill_twiddles(float2* tw, std::int64_t n) {
  for (std::int64_t m = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; m < n;
       m += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    double s, c;
    sincospi(2.0 * static_cast<double>(m) / static_cast<double>(n), &s, &c);
    tw[m] = make_float2(static_cast<float>(c), static_cast<float>(-s));
  }
}

// Device address of g_scratch, looked up once per device.  Host code may not use
// the symbol itself as a pointer: on the host it names a shadow variable, not
// device memory.
float2* scratch_address() {
  static std::mutex mu;
  static std::array<float2*, 64> addr{};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    addr[dev] = static_cast<float2*>(p);
  }
  return addr[dev];
}

cudaError_t fill(float2* tw, std::int64_t n, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
  fill_twiddles<<<grid, 256, 0, st>>>(tw, n);
  return cudaGetLastError();
}

}  // namespace
}  // namespace mb200::fft

extern "C" cufftResult cufftExecC2CNoAlloc(cufftComplex* idata, cufftComplex* odata,
                                           long long n, long long batch, int direction,
                                           cudaStream_t stream) {
  using namespace mb200::fft;
  if (idata == nullptr || odata == nullptr || batch <= 0 ||
      (direction != CUFFT_FORWARD && direction != CUFFT_INVERSE))
    return CUFFT_INVALID_VALUE;
  if (n < 2 || n > kMaxLen || (n & (n - 1)) != 0) return CUFFT_INVALID_SIZE;
  const std::size_t bytes = static_cast<std::size_t>(n) * static_cast<std::size_t>(batch) *
                            sizeof(float2);
  if (!mb200::device_span_ok(idata, bytes) || !mb200::device_span_ok(odata, bytes) ||
      !mb200::aligned_to(idata, 8) || !mb200::aligned_to(odata, 8))
    return CUFFT_INVALID_VALUE;
  float2* base = scratch_address();
  if (base == nullptr) return CUFFT_SETUP_FAILED;
  float2* ws = base;
  float2* tw_n = base + kMaxLen;
  float2* tw_n1 = tw_n + kMaxLen;
  float2* tw_n2 = tw_n1 + kMaxPass;
  const int sign = (direction == CUFFT_FORWARD) ? -1 : 1;

  if (fill(tw_n, n, stream) != cudaSuccess) return CUFFT_EXEC_FAILED;
  if (single_pass_supported(n)) {
    Batch1D b{};
    b.in = idata;
    b.out = odata;
    b.in_stride = 1;
    b.in_outer = n;
    b.out_stride = 1;
    b.out_outer = n;
    b.batch = batch;
    b.inner_count = 1;
    b.tw = tw_n;
    b.post_n = 1;
    return launch_stockham(n, sign, b, stream) == cudaSuccess ? CUFFT_SUCCESS : CUFFT_EXEC_FAILED;
  }
  // Two passes through the workspace (n = n1 * n2, both <= 16384), a chunk of
  // kMaxLen / n transforms at a time:
  //   pass A, per (b, r2): length-n1 transform over t = n2*r1 + r2, output k1 scaled
  //           by W_n^{r2*k1}, stored at ws[b][k1*n2 + r2];
  //   pass B, per (b, k1): length-n2 transform over r2, output k2 stored at X[k1 + n1*k2].
  int l = 0;
  while ((std::int64_t{1} << l) < n) ++l;
  const std::int64_t n1 = std::int64_t{1} << (l / 2);
  const std::int64_t n2 = n / n1;
  if (fill(tw_n1, n1, stream) != cudaSuccess || fill(tw_n2, n2, stream) != cudaSuccess)
    return CUFFT_EXEC_FAILED;
  const std::int64_t chunk = kMaxLen / n;
  for (std::int64_t b0 = 0; b0 < batch; b0 += chunk) {
    const std::int64_t nb = (batch - b0 < chunk) ? batch - b0 : chunk;
    Batch1D a{};
    a.in = idata + b0 * n;
    a.out = ws;
    a.in_stride = n2;
    a.in_outer = n;
    a.in_inner = 1;
    a.out_stride = n2;
    a.out_outer = n;
    a.out_inner = 1;
    a.batch = nb * n2;
    a.inner_count = n2;
    a.tw = tw_n1;
    a.post_tw = tw_n;
    a.post_n = n;
    if (launch_stockham(n1, sign, a, stream) != cudaSuccess) return CUFFT_EXEC_FAILED;
    Batch1D c{};
    c.in = ws;
    c.out = odata + b0 * n;
    c.in_stride = 1;
    c.in_outer = n;
    c.in_inner = n2;
    c.out_stride = n1;
    c.out_outer = n;
    c.out_inner = 1;
    c.batch = nb * n1;
    c.inner_count = n1;
    c.tw = tw_n2;
    c.post_n = 1;
    if (launch_stockham(n2, sign, c, stream) != cudaSuccess) return CUFFT_EXEC_FAILED;
  }
  return CUFFT_SUCCESS;
}
