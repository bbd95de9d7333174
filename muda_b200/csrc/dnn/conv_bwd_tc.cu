// conv_bwd_tc.cu — convolution backward data and backward filter on the tensor
// cores (split tf32, fp32 results), for groups 1.
//
// Backward data, stride 1: with the forward tap map i = o - pad + r*dil,
//   dx[i] = sum_r dy[i + pad - r*dil] W(r) = sum_r' dy[i - pad' + r'*dil] W(R-1-r'),
//   pad' = (R-1)*dil - pad,
// a forward convolution of dy (K input channels) with the filter transposed (K <-> C)
// and the mode swapped (a cross-correlation's backward pass is a convolution-mode
// forward and vice versa).  The transposed filter goes to the workspace, then the
// forward split-tf32 implicit GEMM (conv_tc_kernels.cu) runs on NHWC dy / dx.
//
// Backward filter: T (K x C*R*S) = dY^T (K x N*P*Q) * Xcol (N*P*Q x C*R*S), Xcol the
// im2col of x in the filter's (r, s, c) or (c, r, s) order, as one split-tf32 GEMM
// (gemm_tc_kernels.cu) per chunk of N*P*Q rows accumulating into T; a last pass
// writes dw = alpha * T^T + beta * dw in the filter layout.  For packed NHWC x and a
// KRSC filter the orientation flips: dw (CRS x K) = Xcol^T dY straight into the
// filter (alpha, beta on the first chunk, then beta 1), with im2col_planes writing
// Xcol as the GEMM's split-tf32 A planes in one pass (no fp32 im2col matrix, no
// separate split, no T).  CRS then fills the 128-row side of the tile and K the
// narrow side, instead of K = 64 leaving half of each 128-row MMA idle.
// dY is read in place when each pixel's K gradients are contiguous (NHWC), else it
// is gathered into a dense N*P*Q x K matrix first.
//
// Each output's sum runs in a different order than the reference's sequential loop,
// with the split-tf32 error (about 1e-6 normwise, at or below the fp32 FMA loop's).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "blas/gemm.hpp"
#include "blas/tf32_split.hpp"
#include "common/device.hpp"
#include "dnn/dnn.hpp"

namespace mb200::dnn {
namespace {

constexpr int kThreads = 256;
constexpr std::size_t kColsCap = std::size_t{1} << 30;  // bytes of im2col per chunk

unsigned grid_for(std::int64_t work) {
  const int sms = sm_count(current_device());
  const std::int64_t want = (work + kThreads - 1) / kThreads;
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * 16;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

bool packed_nhwc(const View4& v) {
  return v.cs == 1 && v.ws == v.c && v.hs == static_cast<std::int64_t>(v.w) * v.c &&
         v.ns == static_cast<std::int64_t>(v.h) * v.w * v.c;
}

// out[c][k][r][s] (KCRS) or out[c][r][s][k] (KRSC) = w[k][c][r][s] in w's format.
__global__ void __launch_bounds__(kThreads)
    transpose_filter(const float* __restrict__ w, int K, int C, int R, int S, bool krsc,
                     float* __restrict__ out) {
  const std::int64_t total = static_cast<std::int64_t>(K) * C * R * S;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    // t indexes the output
    int c, k, r, s;
    if (krsc) {  // out[c][r][s][k]
      k = static_cast<int>(t % K);
      std::int64_t q = t / K;
      s = static_cast<int>(q % S);
      q /= S;
      r = static_cast<int>(q % R);
      c = static_cast<int>(q / R);
      out[t] = w[((static_cast<std::int64_t>(k) * R + r) * S + s) * C + c];
    } else {  // out[c][k][r][s]
      s = static_cast<int>(t % S);
      std::int64_t q = t / S;
      r = static_cast<int>(q % R);
      q /= R;
      k = static_cast<int>(q % K);
      c = static_cast<int>(q / K);
      out[t] = w[((static_cast<std::int64_t>(k) * C + c) * R + r) * S + s];
    }
  }
}

// cols[row][col] for pixels npq0 .. npq0 + rows of the output, col in the filter's
// order ((r, s, c) for KRSC, (c, r, s) for KCRS); x at the input tap that weight
// column meets (zero outside the image).
__global__ void __launch_bounds__(kThreads)
    im2col(const float* __restrict__ x, ConvShape s, std::int64_t npq0, std::int64_t rows,
           float* __restrict__ cols) {
  const int C = s.x.c, R = s.kh, S = s.kw;
  const std::int64_t crs = static_cast<std::int64_t>(C) * R * S;
  const std::int64_t total = rows * crs;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t row = t / crs;
    const int col = static_cast<int>(t - row * crs);
    int c, fr, fs;
    if (s.filter_krsc) {
      c = col % C;
      fs = (col / C) % S;
      fr = col / (C * S);
    } else {
      fs = col % S;
      fr = (col / S) % R;
      c = col / (R * S);
    }
    const std::int64_t npq = npq0 + row;
    const int q = static_cast<int>(npq % s.y.w);
    const std::int64_t bp = npq / s.y.w;
    const int p = static_cast<int>(bp % s.y.h);
    const int b = static_cast<int>(bp / s.y.h);
    const int r = s.convolution ? R - 1 - fr : fr;
    const int sv = s.convolution ? S - 1 - fs : fs;
    const int iy = p * s.stride_h - s.pad_h + r * s.dil_h;
    const int ix = q * s.stride_w - s.pad_w + sv * s.dil_w;
    float v = 0.0f;
    if (iy >= 0 && iy < s.x.h && ix >= 0 && ix < s.x.w)
      v = x[b * s.x.ns + c * s.x.cs + iy * s.x.hs + ix * s.x.ws];
    cols[t] = v;
  }
}

// The same for packed NHWC x and (r, s, c) column order with C % 4 == 0: one thread
// per (pixel, 4 channels), the pixel decomposed once and the R*S taps copied as
// 16-byte vectors.
__global__ void __launch_bounds__(kThreads)
    im2col_nhwc4(const float* __restrict__ x, ConvShape s, std::int64_t npq0, std::int64_t rows,
                 float* __restrict__ cols) {
  const int C4 = s.x.c / 4, R = s.kh, S = s.kw;
  const std::int64_t crs = static_cast<std::int64_t>(s.x.c) * R * S;
  const std::int64_t total = rows * C4;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t row = t / C4;
    const int c4 = static_cast<int>(t - row * C4);
    const std::int64_t npq = npq0 + row;
    const int q = static_cast<int>(npq % s.y.w);
    const std::int64_t bp = npq / s.y.w;
    const int p = static_cast<int>(bp % s.y.h);
    const int b = static_cast<int>(bp / s.y.h);
    const float4* xb = reinterpret_cast<const float4*>(x + b * s.x.ns) + c4;
    float4* out = reinterpret_cast<float4*>(cols + row * crs) + c4;
    for (int fr = 0; fr < R; ++fr) {
      const int r = s.convolution ? R - 1 - fr : fr;
      const int iy = p * s.stride_h - s.pad_h + r * s.dil_h;
      for (int fs = 0; fs < S; ++fs) {
        const int sv = s.convolution ? S - 1 - fs : fs;
        const int ix = q * s.stride_w - s.pad_w + sv * s.dil_w;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (iy >= 0 && iy < s.x.h && ix >= 0 && ix < s.x.w)
          v = __ldg(xb + (static_cast<std::int64_t>(iy) * s.x.w + ix) * C4);
        out[(fr * S + fs) * C4] = v;
      }
    }
  }
}

// im2col of packed NHWC x in (r, s, c) column order written straight as the GEMM's
// split-tf32 B planes: planes[p][crs][row] (row = pixel within the chunk, ldk floats
// a column, p = 0 hi, 1 lo), so neither the fp32 im2col matrix nor its transpose is
// ever stored.  A CTA takes 32 pixels x 32 channels and walks the R*S taps: each
// pixel is decomposed once (32-bit: the plan keeps N*P*Q below 2^31), each tap reads
// along the channels (contiguous in x, which stays in L2 across the taps),
// transposes in shared memory and writes along the pixels.
constexpr int kPlaneTile = 32;

__global__ void __launch_bounds__(kThreads)
    im2col_planes(const float* __restrict__ x, ConvShape s, std::int64_t npq0, std::int64_t rows,
                  std::int64_t ldk, float* __restrict__ planes) {
  __shared__ float tile[kPlaneTile][kPlaneTile + 1];  // [channel][pixel]
  constexpr int kRows = kThreads / kPlaneTile;
  constexpr int kPer = kPlaneTile / kRows;  // pixel rows a thread loads per tap
  const int C = s.x.c, R = s.kh, S = s.kw;
  const std::int64_t plane = static_cast<std::int64_t>(C) * R * S * ldk;
  const int ctiles = (C + kPlaneTile - 1) / kPlaneTile;
  const std::int64_t total = ((rows + kPlaneTile - 1) / kPlaneTile) * ctiles;
  const int tx = threadIdx.x % kPlaneTile, ty = threadIdx.x / kPlaneTile;
  for (std::int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int ct = static_cast<int>(t % ctiles);
    const std::int64_t row0 = (t / ctiles) * kPlaneTile;
    const int c = ct * kPlaneTile + tx;
    // this thread's pixel rows: image base offset and top-left input corner
    std::int64_t base[kPer];
    int y0[kPer], x0[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const std::int64_t row = row0 + ty + i * kRows;
      if (row < rows && c < C) {
        const int npq = static_cast<int>(npq0 + row);
        const int q = npq % s.y.w;
        const int bp = npq / s.y.w;
        const int p = bp % s.y.h;
        const int b = bp / s.y.h;
        base[i] = static_cast<std::int64_t>(b) * s.x.ns + c;
        y0[i] = p * s.stride_h - s.pad_h;
        x0[i] = q * s.stride_w - s.pad_w;
      } else {
        base[i] = 0;
        y0[i] = -(1 << 30);  // never inside the image
        x0[i] = 0;
      }
    }
    for (int fr = 0; fr < R; ++fr) {
      const int r = s.convolution ? R - 1 - fr : fr;
      for (int fs = 0; fs < S; ++fs) {
        const int sv = s.convolution ? S - 1 - fs : fs;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int iy = y0[i] + r * s.dil_h;
          const int ix = x0[i] + sv * s.dil_w;
          float v = 0.0f;
          if (iy >= 0 && iy < s.x.h && ix >= 0 && ix < s.x.w)
            v = __ldg(x + base[i] + (static_cast<std::int64_t>(iy) * s.x.w + ix) * C);
          tile[tx][ty + i * kRows] = v;
        }
        __syncthreads();
        const std::int64_t col0 = static_cast<std::int64_t>(fr * S + fs) * C;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int a = ty + i * kRows;
          const int cc = ct * kPlaneTile + a;
          const std::int64_t row = row0 + tx;
          if (cc < C && row < rows) {
            float hi, lo;
            tc::tf32_split_value(tile[a][tx], hi, lo);
            const std::int64_t at = (col0 + cc) * ldk + row;
            planes[at] = hi;
            planes[plane + at] = lo;
          }
        }
        __syncthreads();
      }
    }
  }
}

// dw = alpha * T^T + beta * dw, T the K x CRS column-major GEMM result (T[k + crs*K])
// and dw the filter layout k*CRS + crs.
__global__ void __launch_bounds__(kThreads)
    finish_filter(const float* __restrict__ t, float* __restrict__ dw, int K, std::int64_t crs,
                  float alpha, float beta) {
  const std::int64_t total = crs * K;
  for (std::int64_t i = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i / crs);
    const std::int64_t c = i - k * crs;
    const float prev = (beta == 0.0f) ? 0.0f : beta * dw[i];
    dw[i] = fmaf(alpha, t[k + c * K], prev);
  }
}

// dense[row][k] = dy at pixel npq0 + row, channel k.
__global__ void __launch_bounds__(kThreads)
    gather_dy(const float* __restrict__ dy, View4 v, std::int64_t npq0, std::int64_t rows,
              float* __restrict__ dense) {
  const std::int64_t total = rows * v.c;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const std::int64_t row = t / v.c;
    const int k = static_cast<int>(t - row * v.c);
    const std::int64_t npq = npq0 + row;
    const int q = static_cast<int>(npq % v.w);
    const std::int64_t bp = npq / v.w;
    const int p = static_cast<int>(bp % v.h);
    const int b = static_cast<int>(bp / v.h);
    dense[t] = dy[b * v.ns + k * v.cs + p * v.hs + q * v.ws];
  }
}

// Forward geometry whose result is the backward data of s.
ConvShape data_shape(const ConvShape& s) {
  ConvShape t = s;
  t.x = s.y;  // dy: K channels in
  t.y = s.x;  // dx: C channels out
  t.pad_h = (s.kh - 1) * s.dil_h - s.pad_h;
  t.pad_w = (s.kw - 1) * s.dil_w - s.pad_w;
  t.convolution = !s.convolution;
  return t;
}

struct FilterPlan {
  std::int64_t npq = 0, chunk = 0;  // rows per GEMM
  std::size_t cols_bytes = 0, dy_bytes = 0, t_bytes = 0, gemm_bytes = 0;
  bool dy_direct = false;
  bool planes = false;  // im2col written as split planes (packed NHWC x, KRSC filter)
  std::size_t bytes() const { return cols_bytes + dy_bytes + t_bytes + gemm_bytes; }
};

std::size_t round256(std::size_t v) { return (v + 255) / 256 * 256; }

// T (K x CRS, column-major) += dY^T Xcol over one chunk: the K side on the
// 128-row side of the tensor-core tile and CRS on its 256-column side.
blas::GemmArgs filter_gemm(const ConvShape& s, std::int64_t rows, const float* cols,
                           const float* dy, std::int64_t ldy, float* t, float beta) {
  const std::int64_t crs = static_cast<std::int64_t>(s.x.c) * s.kh * s.kw;
  blas::GemmArgs g{};
  g.type = blas::Elem::kF32;
  g.trans_a = false;  // dY^T: element (k, p) at dy[p * ldy + k]
  g.trans_b = true;   // Xcol: element (p, crs) at cols[p * crs + crs]
  g.m = s.y.c;
  g.n = static_cast<int>(crs);
  g.k = static_cast<int>(rows);
  g.a = dy;
  g.lda = ldy;
  g.b = cols;
  g.ldb = crs;
  g.c = t;
  g.ldc = s.y.c;
  g.batch = 1;
  g.alpha = 1.0f;
  g.beta = beta;
  return g;
}

// dw (KRSC: element (crs, k) at dw[k * CRS + crs], a CRS x K column-major matrix)
// = alpha * Xcol^T dY + beta * dw over one chunk, Xcol given as split planes: CRS on
// the 128-row side of the tensor-core tile, K on its 64/128/256-column side.
blas::GemmArgs filter_gemm_planes(const ConvShape& s, std::int64_t rows, const float* dy,
                                  std::int64_t ldy, float* dw, float alpha, float beta) {
  const std::int64_t crs = static_cast<std::int64_t>(s.x.c) * s.kh * s.kw;
  blas::GemmArgs g{};
  g.type = blas::Elem::kF32;
  g.trans_b = true;  // dY: element (p, k) at dy[p * ldy + k]
  g.m = static_cast<int>(crs);
  g.n = s.y.c;
  g.k = static_cast<int>(rows);
  g.b = dy;
  g.ldb = ldy;
  g.c = dw;
  g.ldc = crs;
  g.batch = 1;
  g.alpha = alpha;
  g.beta = beta;
  return g;
}

FilterPlan plan_filter(const ConvShape& s) {
  FilterPlan pl{};
  if (s.groups != 1) return pl;
  const std::int64_t crs = static_cast<std::int64_t>(s.x.c) * s.kh * s.kw;
  pl.npq = static_cast<std::int64_t>(s.y.n) * s.y.h * s.y.w;
  if (pl.npq <= 0 || crs <= 0 || pl.npq >= (std::int64_t{1} << 31) || crs >= (1 << 30)) return pl;
  pl.planes = s.filter_krsc && packed_nhwc(s.x);
  const std::int64_t cap =
      static_cast<std::int64_t>(kColsCap / (crs * 4 * (pl.planes ? 2 : 1))) / 4 * 4;
  if (cap <= 0) return {};
  // equal chunks (the last one at most nchunks - 1 rows shorter), each a GEMM the
  // tensor-core path accepts
  const std::int64_t nchunks = (pl.npq + cap - 1) / cap;
  pl.chunk = (pl.npq + nchunks - 1) / nchunks;
  const std::int64_t last = pl.npq - (nchunks - 1) * pl.chunk;
  pl.dy_direct = packed_nhwc(s.y);
  pl.cols_bytes =
      pl.planes
          ? round256(static_cast<std::size_t>(2 * crs * blas::tf32_plane_ldk(pl.chunk) * 4))
          : round256(static_cast<std::size_t>(pl.chunk * crs * 4));
  pl.dy_bytes = pl.dy_direct ? 0 : round256(static_cast<std::size_t>(pl.chunk) * s.y.c * 4);
  pl.t_bytes = pl.planes ? 0 : round256(static_cast<std::size_t>(crs) * s.y.c * 4);
  auto ws = [&](std::int64_t rows) {
    if (pl.planes)
      return blas::gemm_tf32x3_aplanes_workspace(
          filter_gemm_planes(s, rows, nullptr, s.y.c, nullptr, 1.0f, 0.0f));
    return blas::gemm_tf32x3_workspace(filter_gemm(s, rows, nullptr, nullptr, s.y.c, nullptr, 0));
  };
  const std::size_t g_full = ws(pl.chunk);
  const std::size_t g_last = ws(last);
  if (g_full == 0 || g_last == 0) return {};
  pl.gemm_bytes = std::max(g_full, g_last);
  return pl;
}

}  // namespace

std::size_t conv_bwd_data_tc_workspace(const ConvShape& s) noexcept {
  if (s.groups != 1 || s.stride_h != 1 || s.stride_w != 1) return 0;
  const std::size_t need = conv_tf32x3_workspace(data_shape(s));
  if (need == 0) return 0;
  return round256(static_cast<std::size_t>(s.y.c) * s.x.c * s.kh * s.kw * 4) + need;
}

cudaError_t launch_conv_bwd_data_tc(const float* w, const float* dy, float* dx,
                                    const ConvShape& s, float alpha, float beta, void* workspace,
                                    std::size_t ws_bytes, cudaStream_t stream) noexcept {
  const std::size_t need = conv_bwd_data_tc_workspace(s);
  if (need == 0 || ws_bytes < need || !aligned_to(workspace, 256)) return cudaErrorNotSupported;
  float* wt = static_cast<float*>(workspace);
  const std::size_t wt_bytes = round256(static_cast<std::size_t>(s.y.c) * s.x.c * s.kh * s.kw * 4);
  transpose_filter<<<grid_for(static_cast<std::int64_t>(s.y.c) * s.x.c * s.kh * s.kw), kThreads, 0,
                     stream>>>(w, s.y.c, s.x.c, s.kh, s.kw, s.filter_krsc, wt);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_conv_tf32x3(dy, wt, dx, data_shape(s), alpha, beta,
                            static_cast<char*>(workspace) + wt_bytes, ws_bytes - wt_bytes, stream);
}

std::size_t conv_bwd_filter_tc_workspace(const ConvShape& s) noexcept {
  const FilterPlan pl = plan_filter(s);
  return pl.chunk > 0 ? pl.bytes() : 0;
}

cudaError_t launch_conv_bwd_filter_tc(const float* x, const float* dy, float* dw,
                                      const ConvShape& s, float alpha, float beta,
                                      void* workspace, std::size_t ws_bytes,
                                      cudaStream_t stream) noexcept {
  const FilterPlan pl = plan_filter(s);
  if (pl.chunk <= 0 || ws_bytes < pl.bytes() || !aligned_to(workspace, 256))
    return cudaErrorNotSupported;
  auto* base = static_cast<char*>(workspace);
  float* cols = reinterpret_cast<float*>(base);
  float* dense = reinterpret_cast<float*>(base + pl.cols_bytes);
  float* tmat = reinterpret_cast<float*>(base + pl.cols_bytes + pl.dy_bytes);
  void* gws = base + pl.cols_bytes + pl.dy_bytes + pl.t_bytes;
  const std::int64_t crs = static_cast<std::int64_t>(s.x.c) * s.kh * s.kw;
  const bool vec = s.filter_krsc && packed_nhwc(s.x) && s.x.c % 4 == 0 && aligned_to(x, 16);
  for (std::int64_t r0 = 0; r0 < pl.npq; r0 += pl.chunk) {
    const std::int64_t rows = std::min(pl.chunk, pl.npq - r0);
    const std::int64_t ldk = blas::tf32_plane_ldk(rows);
    if (pl.planes) {
      const std::int64_t tiles =
          ((rows + kPlaneTile - 1) / kPlaneTile) * ((s.x.c + kPlaneTile - 1) / kPlaneTile);
      im2col_planes<<<grid_for(tiles * kThreads), kThreads, 0, stream>>>(x, s, r0, rows, ldk,
                                                                          cols);
    } else if (vec) {
      im2col_nhwc4<<<grid_for(rows * (s.x.c / 4)), kThreads, 0, stream>>>(x, s, r0, rows, cols);
    } else {
      im2col<<<grid_for(rows * crs), kThreads, 0, stream>>>(x, s, r0, rows, cols);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const float* dmat = dy + r0 * s.y.c;
    if (!pl.dy_direct) {
      gather_dy<<<grid_for(rows * s.y.c), kThreads, 0, stream>>>(dy, s.y, r0, rows, dense);
      e = cudaGetLastError();
      if (e != cudaSuccess) return e;
      dmat = dense;
    }
    if (pl.planes) {
      const blas::GemmArgs g =
          filter_gemm_planes(s, rows, dmat, s.y.c, dw, alpha, r0 == 0 ? beta : 1.0f);
      e = blas::launch_gemm_tf32x3_aplanes(g, cols, gws, pl.gemm_bytes, stream);
    } else {
      const blas::GemmArgs g =
          filter_gemm(s, rows, cols, dmat, s.y.c, tmat, r0 == 0 ? 0.0f : 1.0f);
      e = blas::launch_gemm_tf32x3(g, gws, pl.gemm_bytes, stream);
    }
    if (e != cudaSuccess) return e;
  }
  if (pl.planes) return cudaSuccess;  // the GEMM wrote dw
  finish_filter<<<grid_for(crs * s.y.c), kThreads, 0, stream>>>(tmat, dw, s.y.c, crs, alpha,
                                                                 beta);
  return cudaGetLastError();
}

}  // namespace mb200::dnn
