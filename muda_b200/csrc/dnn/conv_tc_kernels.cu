// conv_tc_kernels.cu — NHWC implicit-GEMM convolution forward on tcgen05 (bf16 / fp16).
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
// Arithmetic: products of the 16-bit inputs accumulated in fp32 (the reference's
// convolution is fp32-only: libraries/dnn/src/cudnn_ops.mm:134-137), then
// y = fma(alpha, acc, beta == 0 ? 0 : beta * y) rounded to the 16-bit type.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <mutex>

#include "blas/tc_gemm_core.cuh"
#include "common/device.hpp"
#include "dnn/dnn.hpp"

namespace mb200::dnn {
namespace {

constexpr int BN = 256;
constexpr int STAGES = 4;

__device__ unsigned int g_conv_tc_timeouts;

template <typename T>
struct ConvProblem {
  CUtensorMap mx;  // NHWC input: dims (c, w, h, n), box {64, WB, HB, 1}
  CUtensorMap mw;  // KRSC filter as (R*S*C) x K: dims (rsc, k), box {64, BN}
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
    tc::tma_load_4d(sa, &mx, cb * tc::kBK, tq * WB + s * dil_w - pad_w,
                    tp * HB + r * dil_h - pad_h, c3[0], bar);
    tc::tma_load_3d(sb, &mw, (fr * S + fs) * C + cb * tc::kBK, c3[2] * BN, 0, bar);
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
      // 32 channels = 64 contiguous bytes: four 16-byte stores
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        T h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = from_float(a * v[g * 8 + j]);
        *reinterpret_cast<uint4*>(out + g * 8) = *reinterpret_cast<const uint4*>(h);
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
    if constexpr (std::is_same_v<T, __half>) {
      return __half2float(v);
    } else {
      return __bfloat162float(v);
    }
  }
  __device__ static T from_float(float v) {
    if constexpr (std::is_same_v<T, __half>) {
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

template <typename T, int FMT>
cudaError_t run(const void* x, const void* w, void* y, const ConvShape& s, float alpha,
                float beta, cudaStream_t stream) {
  ConvProblem<T> p{};
  const int N = s.x.n, H = s.x.h, W = s.x.w, C = s.x.c, K = s.y.c;
  p.P = s.y.h;
  p.Q = s.y.w;
  p.K = K;
  p.C = C;
  p.R = s.kh;
  p.S = s.kw;
  p.WB = pow2_at_least(p.Q, 8, 64);
  p.HB = tc::kBM / p.WB;
  p.tiles_p = (p.P + p.HB - 1) / p.HB;
  p.tiles_q = (p.Q + p.WB - 1) / p.WB;
  p.tiles_k = (K + BN - 1) / BN;
  p.cblocks = C / tc::kBK;
  p.num_kb = p.R * p.S * p.cblocks;
  p.tiles_total = static_cast<long long>(N) * p.tiles_p * p.tiles_q * p.tiles_k;
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
  return tc::launch_tc_gemm<ConvProblem<T>, BN, STAGES, FMT>(p, sm_count(current_device()), to,
                                                             stream);
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
  return run<__nv_bfloat16, 1>(x, w, y, s, alpha, beta, stream);
}

}  // namespace mb200::dnn
