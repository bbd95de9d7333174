// conv_tc_kernels.cu — NHWC implicit-GEMM convolution forward on tcgen05 (bf16, fp32).
//
// The convolution is the GEMM  Y[pixel][k] = sum_{r,s,c} X[pixel shifted by (r,s)][c] *
// W[k][r][s][c]  with the output pixels as rows (M), the output channels as columns
// (N) and (r, s, c) as the reduction, both operands contiguous in c (K-major).
// It runs on the persistent tcgen05 main loop of tc_gemm_core.cuh; only the
// loads and the epilogue are specific:
//   - the 128 rows of an output tile are 128 consecutive output pixels in NHW order
//     (crossing row and image boundaries), loaded for reduction block (r, s, c0) by
//     one im2col-mode TMA load: the tensor map's bounding box makes the base pixels
//     walk the P x Q output positions (corners -pad and pad - (S-1)*dil), the load's
//     im2col offsets (s*dil, r*dil) pick the tap, and input positions outside the
//     image (the zero padding) come back as zeros from the TMA unit, with no index
//     math or predication in the main loop and no padded rows in the tile;
//   - the weight block is a {64, 256} box of the KRSC filter viewed as a
//     (R*S*C) x K matrix; CUDNN_CONVOLUTION (flipped filter) just selects the
//     mirrored tap;
//   - the epilogue writes tile row r to output pixel m0 + r, i.e. the contiguous
//     channels at y + (m0 + r) * K of the packed NHWC output.
// Arithmetic: products accumulated in fp32, then y = fma(alpha, acc, beta == 0 ?
// 0 : beta * y) (the reference's direct kernel, cudnn_kernels.metal:20-62).  bf16
// tensors are this library's extension.  fp32 tensors (the reference's only
// type: libraries/dnn/src/cudnn_ops.mm:134-137) run in split-tf32 form: one pass
// writes x and w as hi/lo tf32 planes (x stays NHWC, a KRSC or KCRS filter becomes
// KRSC) into the handle's workspace; the x planes form a 5-D tensor (c, w, h, image,
// plane) loaded with two 5-D im2col loads per k-block (hi, lo), k-blocks are 32
// channels, and each K step issues lo*hi + hi*lo + hi*hi (within 1.5 * 2^-20
// relative per product, fp32-class accuracy).
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

constexpr int BN = 256;     // tile width of the 16-bit path
constexpr int STAGES = 4;
// Split tf32: the tile width follows the output channels (a 64-channel layer on a
// 256-wide tile would leave three quarters of every MMA idle); stages fill about
// 192 KB: A planes 32 KB + B planes BN/4 KB per stage.
template <int TBN>
constexpr int kStages32 = TBN == 64 ? 4 : (TBN == 128 ? 3 : 2);
constexpr std::size_t kWorkspaceCap = std::size_t{4} << 30;

__device__ unsigned int g_conv_tc_timeouts;

template <typename T, int FMT, int TBN = BN>
struct ConvProblem {
  static constexpr int kBN = TBN;  // output channels per tile
  static constexpr bool kSplit = FMT == tc::kFmtTf32x3;
  static constexpr int KB = kSplit ? tc::kBK32 : tc::kBK;  // channels per k-block
  // im2col map of the NHWC input (c, w, h, n); split tf32: of the planes
  // (c, w, h, n, plane) with the images as the third spatial dimension
  CUtensorMap mx;
  CUtensorMap mw;  // KRSC filter as (R*S*C) x K (x plane): dims (rsc, k, planes), box {KB, BN, planes}
  long long tiles_total;
  int pixels;  // output pixels N * P * Q (below 2^31)
  int num_kb;
  int P, Q, K, C, R, S, cblocks, tiles_k;
  int pad_h, pad_w, dil_h, dil_w, flip;
  T* y;  // packed NHWC: output pixel m at y + m * K
  float alpha, beta;

  __device__ void prefetch() const {
    tc::prefetch_tensormap(&mx);
    tc::prefetch_tensormap(&mw);
  }

  // (128-pixel tile, -, output-channel block); the channel block varies fastest so
  // the tiles that read the same input pixels run together.
  __device__ void coords(long long t, int (&c3)[3]) const {
    c3[0] = static_cast<int>(t / tiles_k);
    c3[1] = 0;
    c3[2] = static_cast<int>(t % tiles_k);
  }

  __device__ void load(const int (&c3)[3], int kb, void* sa, void* sb, std::uint64_t* bar) const {
    const int rs = kb / cblocks;
    const int cb = kb % cblocks;
    const int r = rs / S;
    const int s = rs % S;
    const int fr = flip ? R - 1 - r : r;
    const int fs = flip ? S - 1 - s : s;
    // first base pixel of the tile: output pixel m0 = (n, p, q) -> (q - pad, p - pad, n)
    const int m0 = c3[0] * tc::kBM;
    const int pq = P * Q;
    const int n = m0 / pq;
    const int rem = m0 - n * pq;
    const int bh = rem / Q - pad_h;
    const int bw = rem % Q - pad_w;
    const auto ow = static_cast<std::uint16_t>(s * dil_w);
    const auto oh = static_cast<std::uint16_t>(r * dil_h);
    if constexpr (kSplit) {
      constexpr int plane = tc::kBM * tc::kRowBytes;
      std::uint8_t* a = static_cast<std::uint8_t*>(sa);
      tc::tma_load_im2col_5d(a, &mx, cb * KB, bw, bh, n, 0, ow, oh, 0, bar);          // hi
      tc::tma_load_im2col_5d(a + plane, &mx, cb * KB, bw, bh, n, 1, ow, oh, 0, bar);  // lo
    } else {
      tc::tma_load_im2col_4d(sa, &mx, cb * KB, bw, bh, n, ow, oh, bar);
    }
    tc::tma_load_3d(sb, &mw, (fr * S + fs) * C + cb * KB, c3[2] * kBN, 0, bar);
  }

  __device__ void scalars(float& a, float& b) const {
    a = alpha;
    b = beta;
  }

  __device__ void store(const int (&c3)[3], int row, int col0, const float (&v)[32], float a,
                        float b) const {
    const int m = c3[0] * tc::kBM + row;
    if (m >= pixels) return;
    const int k0 = c3[2] * kBN + col0;
    T* out = y + static_cast<long long>(m) * K + k0;
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

// The im2col tensor map holds the base-pixel bounding box corners and the load
// offsets in narrow fields: 4-D maps take corners in [-128, 127] and offsets up to
// 255, 5-D maps [-16, 15] and 31.
bool im2col_ok(const ConvShape& s, int rank) {
  const int lo = rank == 4 ? -128 : -16, hi = rank == 4 ? 127 : 15, omax = rank == 4 ? 255 : 31;
  const int ow = (s.kw - 1) * s.dil_w, oh = (s.kh - 1) * s.dil_h;
  auto in = [&](int v) { return v >= lo && v <= hi; };
  return ow >= 0 && oh >= 0 && ow <= omax && oh <= omax && in(-s.pad_w) && in(-s.pad_h) &&
         in(s.pad_w - ow) && in(s.pad_h - oh);
}

// Geometry shared by both formats for `images` images (a chunk of the batch for
// split tf32) whose output starts at y.
template <typename T, int FMT, int TBN>
void fill_geometry(ConvProblem<T, FMT, TBN>& p, const ConvShape& s, void* y, int images,
                   float alpha, float beta) {
  using P = ConvProblem<T, FMT, TBN>;
  p.P = s.y.h;
  p.Q = s.y.w;
  p.K = s.y.c;
  p.C = s.x.c;
  p.R = s.kh;
  p.S = s.kw;
  p.tiles_k = (p.K + TBN - 1) / TBN;
  p.cblocks = p.C / P::KB;
  p.num_kb = p.R * p.S * p.cblocks;
  p.pixels = images * p.P * p.Q;
  p.tiles_total = (p.pixels + tc::kBM - 1) / tc::kBM * p.tiles_k;
  p.pad_h = s.pad_h;
  p.pad_w = s.pad_w;
  p.dil_h = s.dil_h;
  p.dil_w = s.dil_w;
  p.flip = s.convolution ? 1 : 0;
  p.y = static_cast<T*>(y);
  p.alpha = alpha;
  p.beta = beta;
}

// Bounding box of the base pixels: from -pad to (dim - 1) + pad - (taps - 1) * dil.
void im2col_corners(const ConvShape& s, int (&lower)[3], int (&upper)[3]) {
  lower[0] = -s.pad_w;
  lower[1] = -s.pad_h;
  lower[2] = 0;
  upper[0] = s.pad_w - (s.kw - 1) * s.dil_w;
  upper[1] = s.pad_h - (s.kh - 1) * s.dil_h;
  upper[2] = 0;
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
  int lower[3], upper[3];
  im2col_corners(s, lower, upper);
  const long long rsc = static_cast<long long>(p.R) * p.S * C;
  const cuuint64_t wd[3] = {static_cast<cuuint64_t>(rsc), static_cast<cuuint64_t>(K), 1u};
  const cuuint64_t ws[2] = {static_cast<cuuint64_t>(rsc * 2),
                            static_cast<cuuint64_t>(((rsc * K * 2 + 15) / 16) * 16)};
  const cuuint32_t wb[3] = {static_cast<cuuint32_t>(tc::kBK), static_cast<cuuint32_t>(BN), 1u};
  if (!tc::encode_im2col(&p.mx, FMT, x, 4, xd, xs, lower, upper, tc::kBK, tc::kBM) ||
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
  if (!packed_nhwc(s.x) || !packed_nhwc(s.y) || !im2col_ok(s, 5)) return false;
  if (static_cast<long long>(s.y.n) * s.y.h * s.y.w >= (1ll << 31)) return false;
  if (s.x.c % tc::kBK32 != 0 || s.y.c % 4 != 0) return false;
  const long long total = static_cast<long long>(s.y.n) * s.y.h * s.y.w;
  return total * s.y.c * s.x.c * s.kh * s.kw >= (1ll << 24);  // smaller: direct kernel
}

template <int TBN>
cudaError_t run_tf32x3_bn(const float* x, const float* w, float* y, const ConvShape& s,
                          float alpha, float beta, float* ws, const Tf32Plan& pl,
                          cudaStream_t stream) {
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
    ConvProblem<float, tc::kFmtTf32x3, TBN> p{};
    fill_geometry(p, s, y + z0 * s.y.ns, nb, alpha, beta);
    const cuuint64_t xd[5] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W),
                              static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(nb), 2u};
    const cuuint64_t xs[4] = {static_cast<cuuint64_t>(C) * 4, static_cast<cuuint64_t>(W) * C * 4,
                              static_cast<cuuint64_t>(H) * W * C * 4,
                              static_cast<cuuint64_t>(pixels) * C * 4};
    int lower[3], upper[3];
    im2col_corners(s, lower, upper);
    const long long rsc = static_cast<long long>(s.kh) * s.kw * C;
    const cuuint64_t wd[3] = {static_cast<cuuint64_t>(rsc), static_cast<cuuint64_t>(K), 2u};
    const cuuint64_t wst[2] = {static_cast<cuuint64_t>(rsc * 4),
                               static_cast<cuuint64_t>(rsc * K * 4)};
    const cuuint32_t wb[3] = {static_cast<cuuint32_t>(tc::kBK32), static_cast<cuuint32_t>(TBN),
                              2u};
    if (!tc::encode_im2col(&p.mx, 2, xp, 5, xd, xs, lower, upper, tc::kBK32, tc::kBM) ||
        !tc::encode_tiled(&p.mw, 2, wp, 3, wd, wst, wb))
      return cudaErrorNotSupported;
    e = tc::launch_tc_gemm<ConvProblem<float, tc::kFmtTf32x3, TBN>, TBN, kStages32<TBN>,
                           tc::kFmtTf32x3>(p, sms, to, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t run_tf32x3(const float* x, const float* w, float* y, const ConvShape& s, float alpha,
                       float beta, float* ws, const Tf32Plan& pl, cudaStream_t stream) {
  if (s.y.c <= 64) return run_tf32x3_bn<64>(x, w, y, s, alpha, beta, ws, pl, stream);
  if (s.y.c <= 128) return run_tf32x3_bn<128>(x, w, y, s, alpha, beta, ws, pl, stream);
  return run_tf32x3_bn<256>(x, w, y, s, alpha, beta, ws, pl, stream);
}

}  // namespace

bool conv_tc_supported(const ConvShape& s, ConvDtype dt, const void* x, const void* w,
                       const void* y) noexcept {
  if (dt != ConvDtype::kBF16) return false;
  if (s.groups != 1 || s.stride_h != 1 || s.stride_w != 1) return false;
  if (!s.filter_krsc) return false;
  if (!packed_nhwc(s.x) || !packed_nhwc(s.y) || !im2col_ok(s, 4)) return false;
  if (static_cast<long long>(s.y.n) * s.y.h * s.y.w >= (1ll << 31)) return false;
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
