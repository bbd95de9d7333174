// conv_tc_kernels.cu — NHWC implicit-GEMM convolution forward on tcgen05 (bf16, fp32).
//
// The convolution is the GEMM  Y[pixel][k] = sum_{r,s,c} X[pixel shifted by (r,s)][c] *
// W[k][r][s][c]  with the output pixels as rows (M), the output channels as columns
// (N) and (r, s, c) as the reduction, both operands contiguous in c (K-major).
// It runs on the persistent tcgen05 main loop of tc_gemm_core.cuh; only the
// loads and the epilogue are specific:
//   - the 128 rows of an output tile are a rectangle of HB x WB output pixels of one
//     image (WB = 64 for 56-pixel rows), and for reduction block (r, s, c0) the
//     producer loads the matching input rectangle, shifted by the tap, with one 4-D
//     TMA box {64 channels, WB, HB, 1} of the NHWC input: out-of-image coordinates
//     (the zero padding) come back as zeros from the TMA unit itself, no index math
//     or predication in the main loop;
//   - the weight block is a {64, 256} box of the KRSC filter viewed as a
//     (R*S*C) x K matrix; CUDNN_CONVOLUTION (flipped filter) just selects the
//     mirrored tap;
//   - the epilogue writes each pixel's 32-channel chunk as 64 contiguous bytes of
//     the NHWC output and skips the rows of the rectangle outside the image.
// Arithmetic: products accumulated in fp32, then y = fma(alpha, acc, beta == 0 ?
// 0 : beta * y) (the reference's direct kernel, cudnn_kernels.metal:20-62).  bf16
// tensors are this library's extension.  fp32 tensors (the reference's only
// type: libraries/dnn/src/cudnn_ops.mm:134-137) run in split-tf32 form: one pass
// writes x and w as hi/lo tf32 planes (x stays NHWC, a KRSC or KCRS filter becomes
// KRSC) into the handle's workspace, the input box gains a plane dimension (5-D
// TMA), k-blocks are 32 channels, and each K step issues lo*hi + hi*lo + hi*hi
// (within 1.5 * 2^-20 relative per product, fp32-class accuracy).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <mutex>

#include "blas/tc_gemm_core.cuh"
#include "blas/tf32_split.hpp"
#include "common/device.hpp"
#include "dnn/dnn.hpp"

namespace mb200::dnn {
namespace {

constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int STAGES32 = 2;  // 2 x (32 + 64) KB stages for the split-tf32 planes
constexpr std::size_t kWorkspaceCap = std::size_t{4} << 30;

__device__ unsigned int g_conv_tc_timeouts;

template <typename T, int FMT>
struct ConvProblem {
  static constexpr int KB = FMT == tc::kFmtTf32x3 ? tc::kBK32 : tc::kBK;  // channels per block
  // NHWC input: dims (c, w, h, n), box {KB, WB, HB, 1}; split tf32 adds the plane
  // dimension (c, w, h, n, plane) with a box of both planes
  CUtensorMap mx;
  CUtensorMap mw;  // KRSC filter as (R*S*C) x K (x plane): dims (rsc, k, planes), box {KB, BN, planes}
  long long tiles_total;
  int num_kb;
  int P, Q, K, C;
  int HB, WB, tiles_p, tiles_q, tiles_k;
  int cblocks, R, S;
  int pad_h, pad_w, dil_h, dil_w, flip;
  T* y;
  long long y_ns, y_hs, y_ws;
  float alpha, beta;

  __device__ void prefetch() const {
    tc::prefetch_tensormap(&mx);
    tc::prefetch_tensormap(&mw);
  }

  // (image, pixel rectangle, output-channel block); the channel block varies
  // fastest so tiles that read the same input rectangle run together.
  __device__ void coords(long long t, int (&c3)[3]) const {
    const long long per_img = static_cast<long long>(tiles_p) * tiles_q * tiles_k;
    c3[0] = static_cast<int>(t / per_img);
    const int rem = static_cast<int>(t % per_img);
    c3[1] = rem / tiles_k;
    c3[2] = rem % tiles_k;
  }

  __device__ void load(const int (&c3)[3], int kb, void* sa, void* sb, std::uint64_t* bar) const {
    const int rs = kb / cblocks;
    const int cb = kb % cblocks;
    const int r = rs / S;
    const int s = rs % S;
    const int tp = c3[1] / tiles_q;
    const int tq = c3[1] % tiles_q;
    const int fr = flip ? R - 1 - r : r;
    const int fs = flip ? S - 1 - s : s;
    const int xw = tq * WB + s * dil_w - pad_w, xh = tp * HB + r * dil_h - pad_h;
    if constexpr (FMT == tc::kFmtTf32x3)
      tc::tma_load_5d(sa, &mx, cb * KB, xw, xh, c3[0], 0, bar);
    else
      tc::tma_load_4d(sa, &mx, cb * KB, xw, xh, c3[0], bar);
    tc::tma_load_3d(sb, &mw, (fr * S + fs) * C + cb * KB, c3[2] * BN, 0, bar);
  }

  __device__ void scalars(float& a, float& b) const {
    a = alpha;
    b = beta;
  }

  __device__ void store(const int (&c3)[3], int row, int col0, const float (&v)[32], float a,
                        float b) const {
    const int tp = c3[1] / tiles_q;
    const int tq = c3[1] % tiles_q;
    const int p = tp * HB + row / WB;
    const int q = tq * WB + row % WB;
    if (p >= P || q >= Q) return;
    const int k0 = c3[2] * BN + col0;
    T* out = y + c3[0] * y_ns + p * y_hs + q * y_ws + k0;
    if (k0 + 32 <= K && b == 0.0f) {
      // 32 channels = 32 * sizeof(T) contiguous bytes, as 16-byte stores
      constexpr int E = 16 / static_cast<int>(sizeof(T));
#pragma unroll
      for (int g = 0; g < 32 / E; ++g) {
        T h[E];
#pragma unroll
        for (int j = 0; j < E; ++j) h[j] = from_float(a * v[g * E + j]);
        *reinterpret_cast<uint4*>(out + g * E) = *reinterpret_cast<const uint4*>(h);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (k0 + j < K) {
          const float prev = (b == 0.0f) ? 0.0f : b * to_float(out[j]);
          out[j] = from_float(fmaf(a, v[j], prev));
        }
      }
    }
  }

  __device__ static float to_float(T v) {
    if constexpr (std::is_same_v<T, float>) {
      return v;
    } else if constexpr (std::is_same_v<T, __half>) {
      return __half2float(v);
    } else {
      return __bfloat162float(v);
    }
  }
  __device__ static T from_float(float v) {
    if constexpr (std::is_same_v<T, float>) {
      return v;
    } else if constexpr (std::is_same_v<T, __half>) {
      return __float2half_rn(v);
    } else {
      return __float2bfloat16_rn(v);
    }
  }
};

unsigned int* timeout_counter() {
  static std::mutex mu;
  static std::array<unsigned int*, 64> addr{};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_conv_tc_timeouts) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    addr[dev] = static_cast<unsigned int*>(p);
  }
  return addr[dev];
}

bool packed_nhwc(const View4& v) {
  return v.cs == 1 && v.ws == v.c && v.hs == static_cast<std::int64_t>(v.w) * v.c &&
         v.ns == static_cast<std::int64_t>(v.h) * v.w * v.c;
}

int pow2_at_least(int v, int lo, int hi) {
  int p = lo;
  while (p < v && p < hi) p <<= 1;
  return p;
}

// Geometry shared by both formats; `x_images` is the number of images the input
// map covers (a chunk of the batch for split tf32).
template <typename T, int FMT>
void fill_geometry(ConvProblem<T, FMT>& p, const ConvShape& s, void* y, int images, float alpha,
                   float beta) {
  using P = ConvProblem<T, FMT>;
  p.P = s.y.h;
  p.Q = s.y.w;
  p.K = s.y.c;
  p.C = s.x.c;
  p.R = s.kh;
  p.S = s.kw;
  p.WB = pow2_at_least(p.Q, 8, 64);
  p.HB = tc::kBM / p.WB;
  p.tiles_p = (p.P + p.HB - 1) / p.HB;
  p.tiles_q = (p.Q + p.WB - 1) / p.WB;
  p.tiles_k = (p.K + BN - 1) / BN;
  p.cblocks = p.C / P::KB;
  p.num_kb = p.R * p.S * p.cblocks;
  p.tiles_total = static_cast<long long>(images) * p.tiles_p * p.tiles_q * p.tiles_k;
  p.pad_h = s.pad_h;
  p.pad_w = s.pad_w;
  p.dil_h = s.dil_h;
  p.dil_w = s.dil_w;
  p.flip = s.convolution ? 1 : 0;
  p.y = static_cast<T*>(y);
  p.y_ns = s.y.ns;
  p.y_hs = s.y.hs;
  p.y_ws = s.y.ws;
  p.alpha = alpha;
  p.beta = beta;
}

template <typename T, int FMT>
cudaError_t run16(const void* x, const void* w, void* y, const ConvShape& s, float alpha,
                  float beta, cudaStream_t stream) {
  ConvProblem<T, FMT> p{};
  fill_geometry(p, s, y, s.x.n, alpha, beta);
  const int N = s.x.n, H = s.x.h, W = s.x.w, C = s.x.c, K = s.y.c;
  const cuuint64_t xd[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W),
                            static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(N)};
  const cuuint64_t xs[3] = {static_cast<cuuint64_t>(s.x.ws * 2),
                            static_cast<cuuint64_t>(s.x.hs * 2),
                            static_cast<cuuint64_t>(s.x.ns * 2)};
  const cuuint32_t xb[4] = {static_cast<cuuint32_t>(tc::kBK), static_cast<cuuint32_t>(p.WB),
                            static_cast<cuuint32_t>(p.HB), 1u};
  const long long rsc = static_cast<long long>(p.R) * p.S * C;
  const cuuint64_t wd[3] = {static_cast<cuuint64_t>(rsc), static_cast<cuuint64_t>(K), 1u};
  const cuuint64_t ws[2] = {static_cast<cuuint64_t>(rsc * 2),
                            static_cast<cuuint64_t>(((rsc * K * 2 + 15) / 16) * 16)};
  const cuuint32_t wb[3] = {static_cast<cuuint32_t>(tc::kBK), static_cast<cuuint32_t>(BN), 1u};
  if (!tc::encode_tiled(&p.mx, FMT, x, 4, xd, xs, xb) ||
      !tc::encode_tiled(&p.mw, FMT, w, 3, wd, ws, wb))
    return cudaErrorNotSupported;
  unsigned int* to = timeout_counter();
  if (to == nullptr) return cudaErrorNotSupported;
  return tc::launch_tc_gemm<ConvProblem<T, FMT>, BN, STAGES, FMT>(p, sm_count(current_device()),
                                                                  to, stream);
}

// Split-tf32 workspace: filter planes, then the input planes of `chunk` images.
struct Tf32Plan {
  int chunk;
  std::size_t w_floats, x_floats;
  std::size_t bytes() const { return (w_floats + x_floats) * sizeof(float); }
};

Tf32Plan plan_tf32(const ConvShape& s) {
  Tf32Plan pl{};
  pl.w_floats = 2ull * s.y.c * s.kh * s.kw * s.x.c;
  const std::size_t per_image = 2ull * s.x.h * s.x.w * s.x.c;
  std::size_t room = kWorkspaceCap > pl.w_floats * 4 ? kWorkspaceCap - pl.w_floats * 4 : 0;
  std::size_t fit = room / (per_image * 4);
  pl.chunk = static_cast<int>(fit < static_cast<std::size_t>(s.x.n) ? fit : s.x.n);
  pl.x_floats = per_image * (pl.chunk > 0 ? pl.chunk : 0);
  return pl;
}

bool tf32_geometry_ok(const ConvShape& s) {
  if (s.groups != 1 || s.stride_h != 1 || s.stride_w != 1) return false;
  if (!packed_nhwc(s.x) || !packed_nhwc(s.y)) return false;
  if (s.x.c % tc::kBK32 != 0 || s.y.c % 4 != 0) return false;
  const long long total = static_cast<long long>(s.y.n) * s.y.h * s.y.w;
  return total * s.y.c * s.x.c * s.kh * s.kw >= (1ll << 24);  // smaller: direct kernel
}

cudaError_t run_tf32x3(const float* x, const float* w, float* y, const ConvShape& s, float alpha,
                       float beta, float* ws, const Tf32Plan& pl, cudaStream_t stream) {
  const int H = s.x.h, W = s.x.w, C = s.x.c, K = s.y.c;
  float* wp = ws;
  float* xp = ws + pl.w_floats;
  cudaError_t e = tc::launch_tf32_split_filter(w, K, C, s.kh, s.kw, s.filter_krsc, wp, stream);
  if (e != cudaSuccess) return e;
  unsigned int* to = timeout_counter();
  if (to == nullptr) return cudaErrorNotSupported;
  const int sms = sm_count(current_device());
  for (int z0 = 0; z0 < s.x.n; z0 += pl.chunk) {
    const int nb = s.x.n - z0 < pl.chunk ? s.x.n - z0 : pl.chunk;
    // pixels of the chunk as rows, channels as the contiguous k dimension
    const long long pixels = static_cast<long long>(nb) * H * W;
    e = tc::launch_tf32_split(x + z0 * s.x.ns, pixels, C, 1, C, 1, 0, xp, C, stream);
    if (e != cudaSuccess) return e;
    ConvProblem<float, tc::kFmtTf32x3> p{};
    fill_geometry(p, s, y + z0 * s.y.ns, nb, alpha, beta);
    const cuuint64_t xd[5] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W),
                              static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(nb), 2u};
    const cuuint64_t xs[4] = {static_cast<cuuint64_t>(C) * 4, static_cast<cuuint64_t>(W) * C * 4,
                              static_cast<cuuint64_t>(H) * W * C * 4,
                              static_cast<cuuint64_t>(pixels) * C * 4};
    const cuuint32_t xb[5] = {static_cast<cuuint32_t>(tc::kBK32), static_cast<cuuint32_t>(p.WB),
                              static_cast<cuuint32_t>(p.HB), 1u, 2u};
    const long long rsc = static_cast<long long>(s.kh) * s.kw * C;
    const cuuint64_t wd[3] = {static_cast<cuuint64_t>(rsc), static_cast<cuuint64_t>(K), 2u};
    const cuuint64_t wst[2] = {static_cast<cuuint64_t>(rsc * 4),
                               static_cast<cuuint64_t>(rsc * K * 4)};
    const cuuint32_t wb[3] = {static_cast<cuuint32_t>(tc::kBK32), static_cast<cuuint32_t>(BN), 2u};
    if (!tc::encode_tiled(&p.mx, 2, xp, 5, xd, xs, xb) ||
        !tc::encode_tiled(&p.mw, 2, wp, 3, wd, wst, wb))
      return cudaErrorNotSupported;
    e = tc::launch_tc_gemm<ConvProblem<float, tc::kFmtTf32x3>, BN, STAGES32, tc::kFmtTf32x3>(
        p, sms, to, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

bool conv_tc_supported(const ConvShape& s, ConvDtype dt, const void* x, const void* w,
                       const void* y) noexcept {
  if (dt != ConvDtype::kBF16) return false;
  if (s.groups != 1 || s.stride_h != 1 || s.stride_w != 1) return false;
  if (!s.filter_krsc) return false;
  if (!packed_nhwc(s.x) || !packed_nhwc(s.y)) return false;
  if (s.x.c % tc::kBK != 0 || s.y.c % 8 != 0) return false;
  if (!aligned_to(x, 16) || !aligned_to(w, 16) || !aligned_to(y, 16)) return false;
  const long long total = static_cast<long long>(s.y.n) * s.y.h * s.y.w;
  if (total * s.y.c * s.x.c * s.kh * s.kw < (1ll << 22)) return false;  // tiny: direct kernel
  return true;
}

cudaError_t launch_conv_tc(const void* x, const void* w, void* y, const ConvShape& s,
                           ConvDtype dt, float alpha, float beta, cudaStream_t stream) noexcept {
  if (!conv_tc_supported(s, dt, x, w, y)) return cudaErrorNotSupported;
  return run16<__nv_bfloat16, 1>(x, w, y, s, alpha, beta, stream);
}

std::size_t conv_tf32x3_workspace(const ConvShape& s) noexcept {
  if (!tf32_geometry_ok(s)) return 0;
  const Tf32Plan pl = plan_tf32(s);
  return pl.chunk > 0 ? pl.bytes() : 0;
}

cudaError_t launch_conv_tf32x3(const void* x, const void* w, void* y, const ConvShape& s,
                               float alpha, float beta, void* workspace, std::size_t ws_bytes,
                               cudaStream_t stream) noexcept {
  if (!tf32_geometry_ok(s)) return cudaErrorNotSupported;
  const Tf32Plan pl = plan_tf32(s);
  if (pl.chunk <= 0 || workspace == nullptr || ws_bytes < pl.bytes() ||
      !aligned_to(workspace, 16) || !aligned_to(y, 16) || !aligned_to(x, 4) ||
      !aligned_to(w, 4))
    return cudaErrorNotSupported;
  return run_tf32x3(static_cast<const float*>(x), static_cast<const float*>(w),
                    static_cast<float*>(y), s, alpha, beta, static_cast<float*>(workspace), pl,
                    stream);
}

}  // namespace mb200::dnn
