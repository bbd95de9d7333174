// dnn.cpp — restatement of the reference's convolution and softmax arithmetic.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
//   oracle_conv2d_fwd       libraries/dnn/shaders/cudnn_kernels.metal:13-62 (direct kernel:
//                           filter_offset, flip for CUDNN_CONVOLUTION, groups, dilation,
//                           sequential fp32 fma over (c, r, s), fma(alpha, acc, beta*y))
//   oracle_softmax_fwd      dispatch of libraries/dnn/src/cudnn_ops.mm:656-719 over
//                           cudnn_kernels.metal:529-568 (contiguous warp kernel) and
//                           cudnn_kernels.metal:447-527 (generic kernel)
// bf16 tensors (this library's extension) are widened exactly to float, use the same
// fp32 arithmetic, and the result is rounded to nearest-even bf16.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>

#include "oracle.h"
#include "parallel.h"

namespace {

float bf16_to_f32(std::uint16_t b) {
  const std::uint32_t u = static_cast<std::uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

std::uint16_t f32_to_bf16(float f) {
  std::uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<std::uint16_t>((u >> 16) | 0x40u);
  const std::uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return static_cast<std::uint16_t>(u >> 16);
}

float load(const void* p, std::int64_t i, int bf16) {
  return bf16 ? bf16_to_f32(static_cast<const std::uint16_t*>(p)[i])
              : static_cast<const float*>(p)[i];
}

void store(void* p, std::int64_t i, float v, int bf16) {
  if (bf16) {
    static_cast<std::uint16_t*>(p)[i] = f32_to_bf16(v);
  } else {
    static_cast<float*>(p)[i] = v;
  }
}

// cudnn_kernels.metal:13-18
std::int64_t filter_offset(int k, int c_g, int r, int s, int c_per_group, int kh, int kw,
                           int fmt) {
  if (fmt == 0) return ((static_cast<std::int64_t>(k) * c_per_group + c_g) * kh + r) * kw + s;
  return ((static_cast<std::int64_t>(k) * kh + r) * kw + s) * c_per_group + c_g;
}

}  // namespace

extern "C" float oracle_bf16_round(float v) { return bf16_to_f32(f32_to_bf16(v)); }

extern "C" void oracle_conv2d_fwd(const void* x, const void* w, void* y,
                                  const OracleConvParams* pp, int bf16, int accum_f64,
                                  int threads) {
  const OracleConvParams p = *pp;
  const std::int64_t total = static_cast<std::int64_t>(p.n) * p.c_out * p.h_out * p.w_out;
  const int c_in_per_g = p.c_in / p.groups;
  const int c_out_per_g = p.c_out / p.groups;
  oracle_detail::parallel_for(0, total, threads, [&](std::int64_t tid) {
    const int ox = static_cast<int>(tid % p.w_out);
    std::int64_t rem = tid / p.w_out;
    const int oy = static_cast<int>(rem % p.h_out);
    rem /= p.h_out;
    const int oc = static_cast<int>(rem % p.c_out);
    const int b = static_cast<int>(rem / p.c_out);
    const int g = oc / c_out_per_g;
    const int ic_start = g * c_in_per_g;
    float acc = 0.0f;
    double acc_d = 0.0;
    for (int c_g = 0; c_g < c_in_per_g; ++c_g) {
      const int ic = ic_start + c_g;
      for (int r = 0; r < p.kh; ++r) {
        const int fr = (p.conv_mode == 0) ? (p.kh - 1 - r) : r;
        const int iy = oy * p.stride_h - p.pad_h + r * p.dil_h;
        if (iy < 0 || iy >= p.h_in) continue;
        for (int s = 0; s < p.kw; ++s) {
          const int fs = (p.conv_mode == 0) ? (p.kw - 1 - s) : s;
          const int ix = ox * p.stride_w - p.pad_w + s * p.dil_w;
          if (ix < 0 || ix >= p.w_in) continue;
          const std::int64_t x_idx = b * p.x_ns + ic * p.x_cs + iy * p.x_hs + ix * p.x_ws;
          const std::int64_t w_idx =
              filter_offset(oc, c_g, fr, fs, c_in_per_g, p.kh, p.kw, p.w_format);
          const float xv = load(x, x_idx, bf16);
          const float wv = load(w, w_idx, bf16);
          if (accum_f64) {
            acc_d += static_cast<double>(xv) * static_cast<double>(wv);
          } else {
            acc = std::fma(xv, wv, acc);
          }
        }
      }
    }
    const std::int64_t y_idx = b * p.y_ns + oc * p.y_cs + oy * p.y_hs + ox * p.y_ws;
    if (accum_f64) {
      const double prev = (p.beta == 0.0f) ? 0.0 : static_cast<double>(p.beta) * load(y, y_idx, bf16);
      store(y, y_idx, static_cast<float>(static_cast<double>(p.alpha) * acc_d + prev), bf16);
    } else {
      const float prev = (p.beta == 0.0f) ? 0.0f : (p.beta * load(y, y_idx, bf16));
      store(y, y_idx, std::fma(p.alpha, acc, prev), bf16);
    }
  });
}

namespace {

// cudnn_kernels.metal:529-568 for one slice: lane-strided partial max / sums over
// 32 lanes, combined by a butterfly (the order of a SIMD-group reduction).
void softmax_contiguous_slice(const float* x, float* y, std::uint32_t len, int algo, float alpha,
                              float beta) {
  float max_v = 0.0f;
  if (algo != 0) {
    float lane_max[32];
    for (int l = 0; l < 32; ++l) {
      lane_max[l] = -std::numeric_limits<float>::infinity();
      for (std::uint32_t i = l; i < len; i += 32) lane_max[l] = std::fmax(lane_max[l], x[i]);
    }
    for (int o = 16; o > 0; o >>= 1)
      for (int l = 0; l < o; ++l) lane_max[l] = std::fmax(lane_max[l], lane_max[l + o]);
    max_v = lane_max[0];
  }
  float lane_sum[32];
  for (int l = 0; l < 32; ++l) {
    lane_sum[l] = 0.0f;
    for (std::uint32_t i = l; i < len; i += 32) lane_sum[l] += std::exp(x[i] - max_v);
  }
  for (int o = 16; o > 0; o >>= 1)
    for (int l = 0; l < o; ++l) lane_sum[l] = lane_sum[l] + lane_sum[l + o];
  const float sum_exp = lane_sum[0];
  const float log_sum = std::log(sum_exp);
  const float inv_sum = 1.0f / sum_exp;
  for (std::uint32_t i = 0; i < len; ++i) {
    const float shifted = x[i] - max_v;
    const float val = (algo == 2) ? (shifted - log_sum) : (std::exp(shifted) * inv_sum);
    const float prev_y = (beta == 0.0f) ? 0.0f : (beta * y[i]);
    y[i] = std::fma(alpha, val, prev_y);
  }
}

}  // namespace

extern "C" void oracle_softmax_fwd(const float* x, float* y, const OracleTensor4* xd,
                                   const OracleTensor4* yd, int algo, int mode_channel,
                                   float alpha, float beta, int threads) {
  const OracleTensor4 X = *xd, Y = *yd;
  const std::int64_t hw = static_cast<std::int64_t>(X.h) * X.w;
  const std::int64_t chw = X.c * hw;
  const bool contiguous = X.ws == 1 && X.hs == X.w && X.cs == hw && X.ns == chw && Y.ws == 1 &&
                          Y.hs == Y.w && Y.cs == hw && Y.ns == chw;
  if (contiguous && (!mode_channel || (X.h == 1 && X.w == 1))) {
    oracle_detail::parallel_for(0, X.n, threads, [&](std::int64_t s) {
      softmax_contiguous_slice(x + s * chw, y + s * chw, static_cast<std::uint32_t>(chw), algo,
                               alpha, beta);
    });
    return;
  }
  // cudnn_kernels.metal:447-527
  const std::int64_t groups = mode_channel ? X.n * hw : X.n;
  oracle_detail::parallel_for(0, groups, threads, [&](std::int64_t tid) {
    int b, h0 = 0, w0 = 0, h1 = X.h, w1 = X.w;
    if (mode_channel) {
      w0 = static_cast<int>(tid % X.w);
      h0 = static_cast<int>((tid / X.w) % X.h);
      b = static_cast<int>(tid / hw);
      h1 = h0 + 1;
      w1 = w0 + 1;
    } else {
      b = static_cast<int>(tid);
    }
    auto xi = [&](int c, int h, int w) { return b * X.ns + c * X.cs + h * X.hs + w * X.ws; };
    auto yi = [&](int c, int h, int w) { return b * Y.ns + c * Y.cs + h * Y.hs + w * Y.ws; };
    float max_v = -std::numeric_limits<float>::infinity();
    if (algo != 0) {
      for (int c = 0; c < X.c; ++c)
        for (int h = h0; h < h1; ++h)
          for (int w = w0; w < w1; ++w) max_v = std::fmax(max_v, x[xi(c, h, w)]);
    } else {
      max_v = 0.0f;
    }
    float sum_exp = 0.0f;
    for (int c = 0; c < X.c; ++c)
      for (int h = h0; h < h1; ++h)
        for (int w = w0; w < w1; ++w) sum_exp += std::exp(x[xi(c, h, w)] - max_v);
    const float log_sum = std::log(sum_exp);
    for (int c = 0; c < X.c; ++c)
      for (int h = h0; h < h1; ++h)
        for (int w = w0; w < w1; ++w) {
          const float shifted = x[xi(c, h, w)] - max_v;
          const float val = (algo == 2) ? (shifted - log_sum) : (std::exp(shifted) / sum_exp);
          const float prev_y = (beta == 0.0f) ? 0.0f : (beta * y[yi(c, h, w)]);
          y[yi(c, h, w)] = std::fma(alpha, val, prev_y);
        }
  });
}
