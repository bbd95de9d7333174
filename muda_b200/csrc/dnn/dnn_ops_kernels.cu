// dnn_ops_kernels.cu — cuDNN neighbours of the convolution for sm_100a:
// backward data / filter / bias, AddTensor, activation, pooling, batch norm.
//
// Arithmetic per output follows the reference kernels
// (libraries/dnn/shaders/cudnn_kernels.metal:194-714) operation by operation, fp32
// with fma where the reference has fma, so the element-wise and per-output kernels
// (backward data, AddTensor, ReLU / clipped ReLU / identity, pooling) give the
// reference's bits.  The reductions the reference runs as one long sequential loop
// per output (backward filter over N*P*Q, backward bias and batch-norm statistics
// over N*H*W) are split across threads and combined in a fixed order:
// deterministic, within rounding of the sequential sum.
#include <cuda_runtime.h>

#include <cstdint>

#include "common/device.hpp"
#include "dnn/dnn.hpp"

namespace mb200::dnn {
namespace {

constexpr int kThreads = 256;

unsigned grid_for(std::int64_t work, int per_sm = 16) {
  const int sms = sm_count(current_device());
  const std::int64_t want = (work + kThreads - 1) / kThreads;
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * per_sm;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

__device__ __forceinline__ std::int64_t at(const View4& v, int b, int c, int h, int w) {
  return b * v.ns + c * v.cs + h * v.hs + w * v.ws;
}

// (n, c, h, w) of linear index t in w-fastest order; 32-bit divisions when t fits
// (a 64-bit division costs several times as many instructions).
__device__ __forceinline__ void unflatten(std::int64_t t, int c, int h, int w, int& b, int& ic,
                                          int& ih, int& iw) {
  if (t >= 0 && t <= 0x7fffffff) {
    unsigned u = static_cast<unsigned>(t);
    iw = static_cast<int>(u % static_cast<unsigned>(w));
    u /= static_cast<unsigned>(w);
    ih = static_cast<int>(u % static_cast<unsigned>(h));
    u /= static_cast<unsigned>(h);
    ic = static_cast<int>(u % static_cast<unsigned>(c));
    b = static_cast<int>(u / static_cast<unsigned>(c));
    return;
  }
  iw = static_cast<int>(t % w);
  t /= w;
  ih = static_cast<int>(t % h);
  t /= h;
  ic = static_cast<int>(t % c);
  b = static_cast<int>(t / c);
}

__device__ __forceinline__ std::int64_t filter_at(const ConvShape& s, int oc, int cg, int fr,
                                                  int fs) {
  const int cin_g = s.x.c / s.groups;
  return s.filter_krsc ? ((static_cast<std::int64_t>(oc) * s.kh + fr) * s.kw + fs) * cin_g + cg
                       : ((static_cast<std::int64_t>(oc) * cin_g + cg) * s.kh + fr) * s.kw + fs;
}

// ------------------------------------------------------- backward data --
// dx[b, ic, iy, ix] = alpha * sum over (oc of the group, r, s) of dy * w + beta * dx,
// taps visited in the reference's order (cudnn_kernels.metal:194-243).
__global__ void __launch_bounds__(kThreads)
    conv_bwd_data(const float* __restrict__ w, const float* __restrict__ dy, float* __restrict__ dx,
                  ConvShape s, float alpha, float beta) {
  const std::int64_t total = static_cast<std::int64_t>(s.x.n) * s.x.c * s.x.h * s.x.w;
  const int cin_g = s.x.c / s.groups, cout_g = s.y.c / s.groups;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    int b, ic, iy, ix;
    unflatten(t, s.x.c, s.x.h, s.x.w, b, ic, iy, ix);
    const int g = ic / cin_g, cg = ic - g * cin_g;
    float acc = 0.0f;
    for (int ol = 0; ol < cout_g; ++ol) {
      const int oc = g * cout_g + ol;
      for (int r = 0; r < s.kh; ++r) {
        const int ny = iy + s.pad_h - r * s.dil_h;
        if (ny < 0 || ny % s.stride_h != 0) continue;
        const int oy = ny / s.stride_h;
        if (oy >= s.y.h) continue;
        const int fr = s.convolution ? (s.kh - 1 - r) : r;
        for (int q = 0; q < s.kw; ++q) {
          const int nx = ix + s.pad_w - q * s.dil_w;
          if (nx < 0 || nx % s.stride_w != 0) continue;
          const int ox = nx / s.stride_w;
          if (ox >= s.y.w) continue;
          const int fs = s.convolution ? (s.kw - 1 - q) : q;
          acc = fmaf(dy[at(s.y, b, oc, oy, ox)], w[filter_at(s, oc, cg, fr, fs)], acc);
        }
      }
    }
    const std::int64_t xi = at(s.x, b, ic, iy, ix);
    const float prev = (beta == 0.0f) ? 0.0f : beta * dx[xi];
    dx[xi] = fmaf(alpha, acc, prev);
  }
}

// ----------------------------------------------------- backward filter --
// dw[oc, cg, fr, fs] = alpha * sum over (b, oy, ox) of x * dy + beta * dw
// (cudnn_kernels.metal:245-286).  The N*P*Q reduction is cut into `chunks`
// contiguous ranges of the flattened (b, oy, ox) index: stage 1 writes one partial
// sum per (chunk, filter element), in the reference's order within the range;
// stage 2 adds the partials in chunk order.
__global__ void __launch_bounds__(kThreads)
    conv_bwd_filter_partial(const float* __restrict__ x, const float* __restrict__ dy,
                            float* __restrict__ partial, ConvShape s, int chunks) {
  const int cin_g = s.x.c / s.groups, cout_g = s.y.c / s.groups;
  const std::int64_t welems = static_cast<std::int64_t>(s.y.c) * cin_g * s.kh * s.kw;
  const std::int64_t m = static_cast<std::int64_t>(s.y.n) * s.y.h * s.y.w;
  const std::int64_t per = (m + chunks - 1) / chunks;
  const std::int64_t total = welems * chunks;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    // chunk-major: consecutive threads take consecutive filter elements of a chunk
    const int chunk = static_cast<int>(t / welems);
    const std::int64_t wl = t - chunk * welems;
    const int fs = static_cast<int>(wl % s.kw);
    std::int64_t rem = wl / s.kw;
    const int fr = static_cast<int>(rem % s.kh);
    rem /= s.kh;
    const int cg = static_cast<int>(rem % cin_g);
    const int oc = static_cast<int>(rem / cin_g);
    const int ic = (oc / cout_g) * cin_g + cg;
    const int r = s.convolution ? (s.kh - 1 - fr) : fr;
    const int q = s.convolution ? (s.kw - 1 - fs) : fs;
    const std::int64_t i0 = chunk * per;
    const std::int64_t i1 = (i0 + per < m) ? i0 + per : m;
    float acc = 0.0f;
    for (std::int64_t i = i0; i < i1; ++i) {
      const int ox = static_cast<int>(i % s.y.w);
      const std::int64_t bq = i / s.y.w;
      const int oy = static_cast<int>(bq % s.y.h);
      const int b = static_cast<int>(bq / s.y.h);
      const int iy = oy * s.stride_h - s.pad_h + r * s.dil_h;
      const int ix = ox * s.stride_w - s.pad_w + q * s.dil_w;
      if (iy < 0 || iy >= s.x.h || ix < 0 || ix >= s.x.w) continue;
      acc = fmaf(x[at(s.x, b, ic, iy, ix)], dy[at(s.y, b, oc, oy, ox)], acc);
    }
    partial[t] = acc;
  }
}

__global__ void __launch_bounds__(kThreads)
    conv_bwd_filter_finish(const float* __restrict__ partial, float* __restrict__ dw, ConvShape s,
                           int chunks, float alpha, float beta) {
  const int cin_g = s.x.c / s.groups;
  const std::int64_t welems = static_cast<std::int64_t>(s.y.c) * cin_g * s.kh * s.kw;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       t < welems; t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    float acc = 0.0f;
    for (int c = 0; c < chunks; ++c) acc += partial[c * welems + t];
    const int fs = static_cast<int>(t % s.kw);
    std::int64_t rem = t / s.kw;
    const int fr = static_cast<int>(rem % s.kh);
    rem /= s.kh;
    const int cg = static_cast<int>(rem % cin_g);
    const int oc = static_cast<int>(rem / cin_g);
    const std::int64_t wi = filter_at(s, oc, cg, fr, fs);
    const float prev = (beta == 0.0f) ? 0.0f : beta * dw[wi];
    dw[wi] = fmaf(alpha, acc, prev);
  }
}

// Block-wide sum of one value per thread, combined in a fixed order (warp
// shuffle tree, then the warp sums in warp order).  Every thread gets the total.
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) total += scratch[i];
  __syncthreads();
  return total;
}

// ------------------------------------------------------- backward bias --
// db[c] = alpha * sum over (b, h, w) of dy + beta * db (cudnn_kernels.metal:288-305);
// one CTA per channel.
constexpr int kRedThreads = 512;

__global__ void __launch_bounds__(kRedThreads)
    conv_bwd_bias(const float* __restrict__ dy, View4 v, float* __restrict__ db, float alpha,
                  float beta) {
  __shared__ float scratch[kRedThreads / 32];
  const int c = blockIdx.x;
  const std::int64_t hw = static_cast<std::int64_t>(v.h) * v.w;
  const std::int64_t m = v.n * hw;
  float acc = 0.0f;
  for (std::int64_t i = threadIdx.x; i < m; i += kRedThreads) {
    const int b = static_cast<int>(i / hw);
    const std::int64_t p = i - b * hw;
    const int h = static_cast<int>(p / v.w);
    acc += dy[at(v, b, c, h, static_cast<int>(p - h * v.w))];
  }
  const float total = block_sum<kRedThreads>(acc, scratch);
  if (threadIdx.x == 0) {
    const float prev = (beta == 0.0f) ? 0.0f : beta * db[c];
    db[c] = fmaf(alpha, total, prev);
  }
}

// ---------------------------------------------------------- AddTensor --
// c = alpha * a + beta * c with a broadcast along its size-1 dimensions
// (cudnn_kernels.metal:307-331).
__global__ void __launch_bounds__(kThreads)
    add_tensor(const float* __restrict__ a, View4 av, float* __restrict__ c, View4 cv, float alpha,
               float beta) {
  const std::int64_t total = static_cast<std::int64_t>(cv.n) * cv.c * cv.h * cv.w;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    int b, ic, ih, iw;
    unflatten(t, cv.c, cv.h, cv.w, b, ic, ih, iw);
    const float va = a[at(av, av.n == 1 ? 0 : b, av.c == 1 ? 0 : ic, av.h == 1 ? 0 : ih,
                          av.w == 1 ? 0 : iw)];
    const std::int64_t ci = at(cv, b, ic, ih, iw);
    const float prev = (beta == 0.0f) ? 0.0f : beta * c[ci];
    c[ci] = fmaf(alpha, va, prev);
  }
}

// --------------------------------------------------------- activation --
// Modes of cudnn_kernels.metal:333-384: 0 sigmoid, 1 ReLU, 2 tanh, 3 clipped ReLU,
// 4 ELU, 5 identity, 6 swish.  max / clamp follow IEEE fmax / fmin (NaN -> 0).
__device__ __forceinline__ float activate(float v, int mode, float coef) {
  switch (mode) {
    case 0: return 1.0f / (1.0f + expf(-v));
    case 1: return fmaxf(v, 0.0f);
    case 2: return tanhf(v);
    case 3: return fminf(fmaxf(v, 0.0f), coef);
    case 4: return v >= 0.0f ? v : coef * (expf(v) - 1.0f);
    case 6: return v / (1.0f + expf(-v));
    default: return v;
  }
}

__global__ void __launch_bounds__(kThreads)
    activation_strided(const float* __restrict__ x, View4 xv, float* __restrict__ y, View4 yv,
                       int mode, float coef, float alpha, float beta) {
  const std::int64_t total = static_cast<std::int64_t>(xv.n) * xv.c * xv.h * xv.w;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    int b, ic, ih, iw;
    unflatten(t, xv.c, xv.h, xv.w, b, ic, ih, iw);
    const float act = activate(x[at(xv, b, ic, ih, iw)], mode, coef);
    const std::int64_t yi = at(yv, b, ic, ih, iw);
    const float prev = (beta == 0.0f) ? 0.0f : beta * y[yi];
    y[yi] = fmaf(alpha, act, prev);
  }
}

// Packed tensors: four elements per thread with 16-byte loads and stores.
__global__ void __launch_bounds__(kThreads)
    activation_vec4(const float4* __restrict__ x, float4* __restrict__ y, std::int64_t n4, int mode,
                    float coef, float alpha, float beta) {
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n4;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = x[t];
    float4 p = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (beta != 0.0f) {
      const float4 q = y[t];
      p = make_float4(beta * q.x, beta * q.y, beta * q.z, beta * q.w);
    }
    y[t] = make_float4(fmaf(alpha, activate(v.x, mode, coef), p.x),
                       fmaf(alpha, activate(v.y, mode, coef), p.y),
                       fmaf(alpha, activate(v.z, mode, coef), p.z),
                       fmaf(alpha, activate(v.w, mode, coef), p.w));
  }
}

// ------------------------------------------------------------ pooling --
// cudnn_kernels.metal:401-445: max (modes 0, 3) or average over the window's
// in-bounds taps, divided by the full window (mode 1) or by the in-bounds count
// (mode 2).
__global__ void __launch_bounds__(kThreads)
    pooling_fwd(const float* __restrict__ x, float* __restrict__ y, PoolShape p, float alpha,
                float beta) {
  const std::int64_t total = static_cast<std::int64_t>(p.y.n) * p.y.c * p.y.h * p.y.w;
  const bool is_max = p.mode == 0 || p.mode == 3;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    int b, ic, oy, ox;
    unflatten(t, p.y.c, p.y.h, p.y.w, b, ic, oy, ox);
    float acc = is_max ? -INFINITY : 0.0f;
    int count = 0;
    for (int r = 0; r < p.win_h; ++r) {
      const int iy = oy * p.stride_h - p.pad_h + r;
      if (iy < 0 || iy >= p.x.h) continue;
      for (int q = 0; q < p.win_w; ++q) {
        const int ix = ox * p.stride_w - p.pad_w + q;
        if (ix < 0 || ix >= p.x.w) continue;
        const float v = x[at(p.x, b, ic, iy, ix)];
        acc = is_max ? fmaxf(acc, v) : acc + v;
        ++count;
      }
    }
    float out = acc;
    if (!is_max) {
      const int denom = (p.mode == 1) ? p.win_h * p.win_w : (count > 1 ? count : 1);
      out = acc / static_cast<float>(denom);
    }
    const std::int64_t yi = at(p.y, b, ic, oy, ox);
    const float prev = (beta == 0.0f) ? 0.0f : beta * y[yi];
    y[yi] = fmaf(alpha, out, prev);
  }
}

// Packed NCHW input and output: blockIdx.y is the (n, c) plane, so the index math is
// 32-bit within a plane and the plane offset is formed once.  For a window known at
// compile time (WH, WW > 0) every in-range tap is loaded before the first is used,
// so the loads overlap instead of waiting on each other through the running result;
// the taps are then combined in the same order as pooling_fwd, out-of-range taps
// skipped (bit-identical results).
template <int WH, int WW>
__global__ void __launch_bounds__(kThreads)
    pooling_planes(const float* __restrict__ x, float* __restrict__ y, PoolShape p, float alpha,
                   float beta) {
  const int OW = p.y.w, OH = p.y.h, W = p.x.w, H = p.x.h;
  const int per_plane = OH * OW;
  const std::int64_t plane = blockIdx.y;
  const float* xp = x + plane * (static_cast<std::int64_t>(H) * W);
  float* yp = y + plane * static_cast<std::int64_t>(per_plane);
  const bool is_max = p.mode == 0 || p.mode == 3;
  const int wh = WH > 0 ? WH : p.win_h, ww = WW > 0 ? WW : p.win_w;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < per_plane; t += gridDim.x * blockDim.x) {
    const int oy = t / OW, ox = t - oy * OW;
    const int y0 = oy * p.stride_h - p.pad_h, x0 = ox * p.stride_w - p.pad_w;
    float acc = is_max ? -INFINITY : 0.0f;
    int count = 0;
    if constexpr (WH > 0 && WW > 0) {
      float v[WH][WW];
      bool in[WH][WW];
#pragma unroll
      for (int r = 0; r < WH; ++r) {
#pragma unroll
        for (int q = 0; q < WW; ++q) {
          const int iy = y0 + r, ix = x0 + q;
          in[r][q] = iy >= 0 && iy < H && ix >= 0 && ix < W;
          v[r][q] = in[r][q] ? __ldg(xp + iy * W + ix) : 0.0f;
        }
      }
#pragma unroll
      for (int r = 0; r < WH; ++r) {
#pragma unroll
        for (int q = 0; q < WW; ++q) {
          if (in[r][q]) {
            acc = is_max ? fmaxf(acc, v[r][q]) : acc + v[r][q];
            ++count;
          }
        }
      }
    } else {
      for (int r = 0; r < wh; ++r) {
        const int iy = y0 + r;
        if (iy < 0 || iy >= H) continue;
        const float* row = xp + iy * W;
        for (int q = 0; q < ww; ++q) {
          const int ix = x0 + q;
          if (ix < 0 || ix >= W) continue;
          const float v = __ldg(row + ix);
          acc = is_max ? fmaxf(acc, v) : acc + v;
          ++count;
        }
      }
    }
    float out = acc;
    if (!is_max) {
      const int denom = (p.mode == 1) ? wh * ww : (count > 1 ? count : 1);
      out = acc / static_cast<float>(denom);
    }
    const float prev = (beta == 0.0f) ? 0.0f : beta * yp[t];
    yp[t] = fmaf(alpha, out, prev);
  }
}

// --------------------------------------------------------- batch norm --
// Inference (cudnn_kernels.metal:570-611): y = alpha * (((x - mean) * inv_std) *
// scale + bias) + beta * y with inv_std = rsqrt(var + eps); parameters per
// (c, h, w) (per-activation) or per c (spatial).
__global__ void __launch_bounds__(kThreads)
    bn_inference(const float* __restrict__ x, View4 xv, float* __restrict__ y, View4 yv,
                 const float* __restrict__ scale, const float* __restrict__ bias,
                 const float* __restrict__ mean, const float* __restrict__ var, bool per_activation,
                 float eps, float alpha, float beta) {
  const std::int64_t total = static_cast<std::int64_t>(xv.n) * xv.c * xv.h * xv.w;
  for (std::int64_t t = static_cast<std::int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    int b, ic, ih, iw;
    unflatten(t, xv.c, xv.h, xv.w, b, ic, ih, iw);
    const std::int64_t pi =
        per_activation ? (static_cast<std::int64_t>(ic) * xv.h + ih) * xv.w + iw : ic;
    const float inv_std = rsqrtf(var[pi] + eps);
    const float nv = fmaf((x[at(xv, b, ic, ih, iw)] - mean[pi]) * inv_std, scale[pi], bias[pi]);
    const std::int64_t yi = at(yv, b, ic, ih, iw);
    const float prev = (beta == 0.0f) ? 0.0f : beta * y[yi];
    y[yi] = fmaf(alpha, nv, prev);
  }
}

// Training (cudnn_kernels.metal:613-714), one CTA per channel: batch mean, then the
// biased variance about it, inv_std = rsqrt(var + eps); optional saved mean /
// inv_std and running averages (1 - f) * running + f * value with the unbiased
// variance; then y as in inference.  Sums are block reductions in a fixed order.
__global__ void __launch_bounds__(kRedThreads)
    bn_training(const float* __restrict__ x, View4 xv, float* __restrict__ y, View4 yv,
                const float* __restrict__ scale, const float* __restrict__ bias,
                float* __restrict__ running_mean, float* __restrict__ running_var,
                float* __restrict__ save_mean, float* __restrict__ save_inv_var, float factor,
                float eps, float alpha, float beta) {
  __shared__ float scratch[kRedThreads / 32];
  const int c = blockIdx.x;
  const std::int64_t hw = static_cast<std::int64_t>(xv.h) * xv.w;
  const std::int64_t m = xv.n * hw;
  const float inv_m = 1.0f / static_cast<float>(m);
  float acc = 0.0f;
  for (std::int64_t i = threadIdx.x; i < m; i += kRedThreads) {
    const int b = static_cast<int>(i / hw);
    const std::int64_t p = i - b * hw;
    const int h = static_cast<int>(p / xv.w);
    acc += x[at(xv, b, c, h, static_cast<int>(p - h * xv.w))];
  }
  const float mean = block_sum<kRedThreads>(acc, scratch) * inv_m;
  float sq = 0.0f;
  for (std::int64_t i = threadIdx.x; i < m; i += kRedThreads) {
    const int b = static_cast<int>(i / hw);
    const std::int64_t p = i - b * hw;
    const int h = static_cast<int>(p / xv.w);
    const float d = x[at(xv, b, c, h, static_cast<int>(p - h * xv.w))] - mean;
    sq = fmaf(d, d, sq);
  }
  const float total_sq = block_sum<kRedThreads>(sq, scratch);
  const float var = total_sq * inv_m;
  const float inv_std = rsqrtf(var + eps);
  if (threadIdx.x == 0) {
    const float unbiased = (m > 1) ? total_sq / static_cast<float>(m - 1) : var;
    if (save_mean != nullptr) {
      save_mean[c] = mean;
      save_inv_var[c] = inv_std;
    }
    if (running_mean != nullptr) {
      running_mean[c] = (1.0f - factor) * running_mean[c] + factor * mean;
      running_var[c] = (1.0f - factor) * running_var[c] + factor * unbiased;
    }
  }
  const float sc = scale[c], bi = bias[c];
  for (std::int64_t i = threadIdx.x; i < m; i += kRedThreads) {
    const int b = static_cast<int>(i / hw);
    const std::int64_t p = i - b * hw;
    const int h = static_cast<int>(p / xv.w);
    const int w = static_cast<int>(p - h * xv.w);
    const float nv = fmaf((x[at(xv, b, c, h, w)] - mean) * inv_std, sc, bi);
    const std::int64_t yi = at(yv, b, c, h, w);
    const float prev = (beta == 0.0f) ? 0.0f : beta * y[yi];
    y[yi] = fmaf(alpha, nv, prev);
  }
}

// Split form of the training pass for large N*H*W: each channel's elements are
// cut into `splits` contiguous ranges, one CTA each (grid splits x C).
//   stage 0: partial sums of x per (channel, range);
//   stage 1: every CTA forms the mean from its channel's partial sums (in range
//            order), then partial sums of (x - mean)^2;
//   stage 2: every CTA forms mean and variance the same way, range 0 writes the
//            saved and running statistics, all write y over their range.
__device__ __forceinline__ void bn_range(std::int64_t m, int splits, int part, std::int64_t& i0,
                                         std::int64_t& i1) {
  const std::int64_t per = (m + splits - 1) / splits;
  i0 = part * per;
  i1 = i0 + per < m ? i0 + per : m;
}

// Image b and pixel p (within the H x W plane) of element i of a channel's N*H*W
// range, stepped by kRedThreads without dividing (a 64-bit division per element
// would cost more than the memory traffic).
struct PlaneWalk {
  int b;
  std::int64_t p, hw;
  __device__ PlaneWalk(std::int64_t i, std::int64_t hw_) : hw(hw_) {
    b = static_cast<int>(i / hw_);
    p = i - static_cast<std::int64_t>(b) * hw_;
  }
  __device__ void next() {
    p += kRedThreads;
    while (p >= hw) {
      p -= hw;
      ++b;
    }
  }
};

// Offset of (b, c, pixel p) in a view; one multiply-add when a plane's rows are
// contiguous (hs == w * ws).
__device__ __forceinline__ std::int64_t plane_at(const View4& v, int b, int c, std::int64_t p) {
  if (v.hs == static_cast<std::int64_t>(v.w) * v.ws) return b * v.ns + c * v.cs + p * v.ws;
  const int h = static_cast<int>(p / v.w);
  return at(v, b, c, h, static_cast<int>(p - static_cast<std::int64_t>(h) * v.w));
}

template <int STAGE>
__global__ void __launch_bounds__(kRedThreads)
    bn_training_split(const float* __restrict__ x, View4 xv, float* __restrict__ y, View4 yv,
                      const float* __restrict__ scale, const float* __restrict__ bias,
                      float* __restrict__ running_mean, float* __restrict__ running_var,
                      float* __restrict__ save_mean, float* __restrict__ save_inv_var,
                      float* __restrict__ partial, int splits, float factor, float eps,
                      float alpha, float beta) {
  __shared__ float scratch[kRedThreads / 32];
  const int part = blockIdx.x, c = blockIdx.y;
  const std::int64_t hw = static_cast<std::int64_t>(xv.h) * xv.w;
  const std::int64_t m = xv.n * hw;
  const float inv_m = 1.0f / static_cast<float>(m);
  float* psum = partial + static_cast<std::int64_t>(c) * splits;               // [C][splits]
  float* psq = partial + static_cast<std::int64_t>(xv.c) * splits + c * splits;  // [C][splits]
  std::int64_t i0, i1;
  bn_range(m, splits, part, i0, i1);
  PlaneWalk pw(i0 + threadIdx.x, hw);
  float mean = 0.0f;
  if (STAGE >= 1) {
    float t = 0.0f;
    for (int q = 0; q < splits; ++q) t += psum[q];
    mean = t * inv_m;
  }
  if (STAGE == 0) {
    float acc = 0.0f;
    for (std::int64_t i = i0 + threadIdx.x; i < i1; i += kRedThreads, pw.next())
      acc += x[plane_at(xv, pw.b, c, pw.p)];
    const float total = block_sum<kRedThreads>(acc, scratch);
    if (threadIdx.x == 0) psum[part] = total;
  } else if (STAGE == 1) {
    float sq = 0.0f;
    for (std::int64_t i = i0 + threadIdx.x; i < i1; i += kRedThreads, pw.next()) {
      const float d = x[plane_at(xv, pw.b, c, pw.p)] - mean;
      sq = fmaf(d, d, sq);
    }
    const float total = block_sum<kRedThreads>(sq, scratch);
    if (threadIdx.x == 0) psq[part] = total;
  } else {
    float total_sq = 0.0f;
    for (int q = 0; q < splits; ++q) total_sq += psq[q];
    const float var = total_sq * inv_m;
    const float inv_std = rsqrtf(var + eps);
    if (part == 0 && threadIdx.x == 0) {
      const float unbiased = (m > 1) ? total_sq / static_cast<float>(m - 1) : var;
      if (save_mean != nullptr) {
        save_mean[c] = mean;
        save_inv_var[c] = inv_std;
      }
      if (running_mean != nullptr) {
        running_mean[c] = (1.0f - factor) * running_mean[c] + factor * mean;
        running_var[c] = (1.0f - factor) * running_var[c] + factor * unbiased;
      }
    }
    const float sc = scale[c], bi = bias[c];
    for (std::int64_t i = i0 + threadIdx.x; i < i1; i += kRedThreads, pw.next()) {
      const float nv = fmaf((x[plane_at(xv, pw.b, c, pw.p)] - mean) * inv_std, sc, bi);
      const std::int64_t yi = plane_at(yv, pw.b, c, pw.p);
      const float prev = (beta == 0.0f) ? 0.0f : beta * y[yi];
      y[yi] = fmaf(alpha, nv, prev);
    }
  }
}

}  // namespace

cudaError_t launch_conv_bwd_data(const float* w, const float* dy, float* dx, const ConvShape& s,
                                 float alpha, float beta, cudaStream_t stream) noexcept {
  const std::int64_t total = static_cast<std::int64_t>(s.x.n) * s.x.c * s.x.h * s.x.w;
  if (total <= 0) return cudaSuccess;
  conv_bwd_data<<<grid_for(total, 64), kThreads, 0, stream>>>(w, dy, dx, s, alpha, beta);
  return cudaGetLastError();
}

int conv_bwd_filter_chunks(const ConvShape& s) noexcept {
  const std::int64_t welems =
      static_cast<std::int64_t>(s.y.c) * (s.x.c / s.groups) * s.kh * s.kw;
  const std::int64_t m = static_cast<std::int64_t>(s.y.n) * s.y.h * s.y.w;
  if (welems <= 0 || m <= 0) return 1;
  // enough threads to fill the GPU several times, at least 64 terms per thread
  const std::int64_t want = (static_cast<std::int64_t>(148) * 2048 * 4 + welems - 1) / welems;
  std::int64_t chunks = want < 1 ? 1 : want;
  const std::int64_t max_by_len = (m + 63) / 64;
  if (chunks > max_by_len) chunks = max_by_len;
  if (chunks > 4096) chunks = 4096;
  return static_cast<int>(chunks < 1 ? 1 : chunks);
}

std::size_t conv_bwd_filter_workspace(const ConvShape& s) noexcept {
  const std::int64_t welems =
      static_cast<std::int64_t>(s.y.c) * (s.x.c / s.groups) * s.kh * s.kw;
  return static_cast<std::size_t>(welems) * conv_bwd_filter_chunks(s) * sizeof(float);
}

cudaError_t launch_conv_bwd_filter(const float* x, const float* dy, float* dw, const ConvShape& s,
                                   float alpha, float beta, float* workspace,
                                   cudaStream_t stream) noexcept {
  const std::int64_t welems =
      static_cast<std::int64_t>(s.y.c) * (s.x.c / s.groups) * s.kh * s.kw;
  if (welems <= 0) return cudaSuccess;
  const int chunks = conv_bwd_filter_chunks(s);
  conv_bwd_filter_partial<<<grid_for(welems * chunks, 64), kThreads, 0, stream>>>(
      x, dy, workspace, s, chunks);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  conv_bwd_filter_finish<<<grid_for(welems, 16), kThreads, 0, stream>>>(workspace, dw, s, chunks,
                                                                        alpha, beta);
  return cudaGetLastError();
}

cudaError_t launch_conv_bwd_bias(const float* dy, const View4& v, float* db, float alpha,
                                 float beta, cudaStream_t stream) noexcept {
  if (v.c <= 0) return cudaSuccess;
  conv_bwd_bias<<<v.c, kRedThreads, 0, stream>>>(dy, v, db, alpha, beta);
  return cudaGetLastError();
}

cudaError_t launch_add_tensor(const float* a, const View4& av, float* c, const View4& cv,
                              float alpha, float beta, cudaStream_t stream) noexcept {
  const std::int64_t total = static_cast<std::int64_t>(cv.n) * cv.c * cv.h * cv.w;
  if (total <= 0) return cudaSuccess;
  add_tensor<<<grid_for(total), kThreads, 0, stream>>>(a, av, c, cv, alpha, beta);
  return cudaGetLastError();
}

cudaError_t launch_activation(const float* x, const View4& xv, float* y, const View4& yv,
                              int mode, float coef, float alpha, float beta,
                              cudaStream_t stream) noexcept {
  const std::int64_t total = static_cast<std::int64_t>(xv.n) * xv.c * xv.h * xv.w;
  if (total <= 0) return cudaSuccess;
  auto packed = [](const View4& v) {
    return v.ws == 1 && v.hs == v.w && v.cs == static_cast<std::int64_t>(v.h) * v.w &&
           v.ns == static_cast<std::int64_t>(v.c) * v.h * v.w;
  };
  if (packed(xv) && packed(yv) && total % 4 == 0 && aligned_to(x, 16) && aligned_to(y, 16)) {
    activation_vec4<<<grid_for(total / 4), kThreads, 0, stream>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), total / 4, mode, coef,
        alpha, beta);
  } else {
    activation_strided<<<grid_for(total), kThreads, 0, stream>>>(x, xv, y, yv, mode, coef, alpha,
                                                                 beta);
  }
  return cudaGetLastError();
}

cudaError_t launch_pooling(const float* x, float* y, const PoolShape& p, float alpha, float beta,
                           cudaStream_t stream) noexcept {
  const std::int64_t total = static_cast<std::int64_t>(p.y.n) * p.y.c * p.y.h * p.y.w;
  if (total <= 0) return cudaSuccess;
  auto packed = [](const View4& v) {
    return v.ws == 1 && v.hs == v.w && v.cs == static_cast<std::int64_t>(v.h) * v.w &&
           v.ns == static_cast<std::int64_t>(v.c) * v.h * v.w;
  };
  const std::int64_t planes = static_cast<std::int64_t>(p.y.n) * p.y.c;
  const std::int64_t per_plane = static_cast<std::int64_t>(p.y.h) * p.y.w;
  const std::int64_t in_plane = static_cast<std::int64_t>(p.x.h) * p.x.w;
  if (packed(p.x) && packed(p.y) && planes <= 65535 && per_plane < (1 << 30) &&
      in_plane < (1 << 30)) {
    const std::int64_t cta = (per_plane + kThreads - 1) / kThreads;
    const dim3 grid(static_cast<unsigned>(cta < 64 ? cta : 64), static_cast<unsigned>(planes));
    if (p.win_h == 3 && p.win_w == 3)
      pooling_planes<3, 3><<<grid, kThreads, 0, stream>>>(x, y, p, alpha, beta);
    else if (p.win_h == 2 && p.win_w == 2)
      pooling_planes<2, 2><<<grid, kThreads, 0, stream>>>(x, y, p, alpha, beta);
    else
      pooling_planes<0, 0><<<grid, kThreads, 0, stream>>>(x, y, p, alpha, beta);
    return cudaGetLastError();
  }
  pooling_fwd<<<grid_for(total), kThreads, 0, stream>>>(x, y, p, alpha, beta);
  return cudaGetLastError();
}

cudaError_t launch_bn_inference(const float* x, const View4& xv, float* y, const View4& yv,
                                const float* scale, const float* bias, const float* mean,
                                const float* var, bool per_activation, float eps, float alpha,
                                float beta, cudaStream_t stream) noexcept {
  const std::int64_t total = static_cast<std::int64_t>(xv.n) * xv.c * xv.h * xv.w;
  if (total <= 0) return cudaSuccess;
  bn_inference<<<grid_for(total), kThreads, 0, stream>>>(x, xv, y, yv, scale, bias, mean, var,
                                                         per_activation, eps, alpha, beta);
  return cudaGetLastError();
}

int bn_training_splits(const View4& xv) noexcept {
  const std::int64_t m = static_cast<std::int64_t>(xv.n) * xv.h * xv.w;
  if (xv.c <= 0 || m <= 0) return 1;
  // about four CTAs per SM in total, each range at least 4096 elements
  const int sms = sm_count(current_device());
  std::int64_t want = (static_cast<std::int64_t>(sms > 0 ? sms : 148) * 4 + xv.c - 1) / xv.c;
  const std::int64_t by_len = m / 4096;
  if (want > by_len) want = by_len;
  if (want > 1024) want = 1024;
  return static_cast<int>(want < 1 ? 1 : want);
}

std::size_t bn_training_workspace(const View4& xv) noexcept {
  const int splits = bn_training_splits(xv);
  return splits > 1 ? static_cast<std::size_t>(2) * xv.c * splits * sizeof(float) : 0;
}

cudaError_t launch_bn_training(const float* x, const View4& xv, float* y, const View4& yv,
                               const float* scale, const float* bias, float* running_mean,
                               float* running_var, float* save_mean, float* save_inv_var,
                               float factor, float eps, float alpha, float beta, float* workspace,
                               cudaStream_t stream) noexcept {
  if (xv.c <= 0) return cudaSuccess;
  const int splits = bn_training_splits(xv);
  if (splits <= 1 || workspace == nullptr) {
    bn_training<<<xv.c, kRedThreads, 0, stream>>>(x, xv, y, yv, scale, bias, running_mean,
                                                  running_var, save_mean, save_inv_var, factor,
                                                  eps, alpha, beta);
    return cudaGetLastError();
  }
  const dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(xv.c));
  bn_training_split<0><<<grid, kRedThreads, 0, stream>>>(
      x, xv, y, yv, scale, bias, running_mean, running_var, save_mean, save_inv_var, workspace,
      splits, factor, eps, alpha, beta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  bn_training_split<1><<<grid, kRedThreads, 0, stream>>>(
      x, xv, y, yv, scale, bias, running_mean, running_var, save_mean, save_inv_var, workspace,
      splits, factor, eps, alpha, beta);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  bn_training_split<2><<<grid, kRedThreads, 0, stream>>>(
      x, xv, y, yv, scale, bias, running_mean, running_var, save_mean, save_inv_var, workspace,
      splits, factor, eps, alpha, beta);
  return cudaGetLastError();
}

}  // namespace mb200::dnn
