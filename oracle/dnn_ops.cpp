// dnn_ops.cpp — restatement of the reference's convolution backward, AddTensor,
// activation, pooling and batch-norm kernels.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Follows libraries/dnn/shaders/cudnn_kernels.metal operation by operation:
//   conv2d_bwd_data      :194-243     conv2d_bwd_filter  :245-286
//   conv2d_bwd_bias      :288-305     add_tensor         :307-331
//   activation_fwd       :333-384     pooling2d_fwd      :401-445
//   batchnorm inference  :570-611     batchnorm training :613-714
// with accum_f64 != 0 the sums are taken in double instead (ground truth for the
// reductions the B200 kernels split).  Transcendentals come from the host libm
// (std::exp, std::tanh), the reciprocal square root as 1 / sqrt.
#include <cmath>
#include <cstdint>
#include <vector>

#include "oracle.h"
#include "parallel.h"

namespace {

inline int64_t at(const OracleTensor4& v, int b, int c, int h, int w) {
  return b * v.ns + c * v.cs + h * v.hs + w * v.ws;
}

// cudnn_kernels.metal:13-18 (0 = KCRS, 1 = KRSC)
inline int64_t filter_at(const OracleConvParams& p, int k, int cg, int r, int s) {
  const int cpg = p.c_in / p.groups;
  if (p.w_format == 0) return ((static_cast<int64_t>(k) * cpg + cg) * p.kh + r) * p.kw + s;
  return ((static_cast<int64_t>(k) * p.kh + r) * p.kw + s) * cpg + cg;
}

inline int64_t x_at(const OracleConvParams& p, int b, int c, int h, int w) {
  return b * p.x_ns + c * p.x_cs + h * p.x_hs + w * p.x_ws;
}
inline int64_t y_at(const OracleConvParams& p, int b, int c, int h, int w) {
  return b * p.y_ns + c * p.y_cs + h * p.y_hs + w * p.y_ws;
}

template <class T>
inline T store(float alpha, T acc, float beta, float prev_raw) {
  const T prev = (beta == 0.0f) ? T(0) : T(beta) * T(prev_raw);
  return std::fma(T(alpha), acc, prev);
}

}  // namespace

extern "C" void oracle_conv_bwd_data(const float* w, const float* dy, float* dx,
                                     const OracleConvParams* pp, int accum_f64, int threads) {
  const OracleConvParams p = *pp;
  const int64_t total = static_cast<int64_t>(p.n) * p.c_in * p.h_in * p.w_in;
  const int cin_g = p.c_in / p.groups, cout_g = p.c_out / p.groups;
  oracle_detail::parallel_for(0, total, threads, [&](int64_t t) {
    const int ix = static_cast<int>(t % p.w_in);
    int64_t rem = t / p.w_in;
    const int iy = static_cast<int>(rem % p.h_in);
    rem /= p.h_in;
    const int ic = static_cast<int>(rem % p.c_in);
    const int b = static_cast<int>(rem / p.c_in);
    const int g = ic / cin_g, cg = ic - g * cin_g;
    float acc = 0.0f;
    double accd = 0.0;
    for (int ol = 0; ol < cout_g; ++ol) {
      const int oc = g * cout_g + ol;
      for (int r = 0; r < p.kh; ++r) {
        const int ny = iy + p.pad_h - r * p.dil_h;
        if (ny < 0 || ny % p.stride_h != 0) continue;
        const int oy = ny / p.stride_h;
        if (oy >= p.h_out) continue;
        const int fr = (p.conv_mode == 0) ? (p.kh - 1 - r) : r;
        for (int s = 0; s < p.kw; ++s) {
          const int nx = ix + p.pad_w - s * p.dil_w;
          if (nx < 0 || nx % p.stride_w != 0) continue;
          const int ox = nx / p.stride_w;
          if (ox >= p.w_out) continue;
          const int fs = (p.conv_mode == 0) ? (p.kw - 1 - s) : s;
          const float a = dy[y_at(p, b, oc, oy, ox)], c = w[filter_at(p, oc, cg, fr, fs)];
          acc = std::fma(a, c, acc);
          accd += static_cast<double>(a) * c;
        }
      }
    }
    const int64_t xi = x_at(p, b, ic, iy, ix);
    dx[xi] = accum_f64 ? static_cast<float>(store<double>(p.alpha, accd, p.beta, dx[xi]))
                       : store<float>(p.alpha, acc, p.beta, dx[xi]);
  });
}

extern "C" void oracle_conv_bwd_filter(const float* x, const float* dy, float* dw,
                                       const OracleConvParams* pp, int accum_f64, double* mag,
                                       int threads) {
  const OracleConvParams p = *pp;
  const int cin_g = p.c_in / p.groups, cout_g = p.c_out / p.groups;
  const int64_t total = static_cast<int64_t>(p.c_out) * cin_g * p.kh * p.kw;
  oracle_detail::parallel_for(0, total, threads, [&](int64_t t) {
    const int fs = static_cast<int>(t % p.kw);
    int64_t rem = t / p.kw;
    const int fr = static_cast<int>(rem % p.kh);
    rem /= p.kh;
    const int cg = static_cast<int>(rem % cin_g);
    const int oc = static_cast<int>(rem / cin_g);
    const int ic = (oc / cout_g) * cin_g + cg;
    const int r = (p.conv_mode == 0) ? (p.kh - 1 - fr) : fr;
    const int s = (p.conv_mode == 0) ? (p.kw - 1 - fs) : fs;
    float acc = 0.0f;
    double accd = 0.0, m = 0.0;
    for (int b = 0; b < p.n; ++b)
      for (int oy = 0; oy < p.h_out; ++oy) {
        const int iy = oy * p.stride_h - p.pad_h + r * p.dil_h;
        if (iy < 0 || iy >= p.h_in) continue;
        for (int ox = 0; ox < p.w_out; ++ox) {
          const int ix = ox * p.stride_w - p.pad_w + s * p.dil_w;
          if (ix < 0 || ix >= p.w_in) continue;
          const float a = x[x_at(p, b, ic, iy, ix)], c = dy[y_at(p, b, oc, oy, ox)];
          acc = std::fma(a, c, acc);
          accd += static_cast<double>(a) * c;
          m += std::fabs(static_cast<double>(a) * c);
        }
      }
    const int64_t wi = filter_at(p, oc, cg, fr, fs);
    if (mag != nullptr) mag[wi] = m;
    dw[wi] = accum_f64 ? static_cast<float>(store<double>(p.alpha, accd, p.beta, dw[wi]))
                       : store<float>(p.alpha, acc, p.beta, dw[wi]);
  });
}

extern "C" void oracle_conv_bwd_bias(const float* dy, const OracleTensor4* vp, float* db,
                                     float alpha, float beta, int accum_f64, double* mag) {
  const OracleTensor4 v = *vp;
  for (int c = 0; c < v.c; ++c) {
    float acc = 0.0f;
    double accd = 0.0, m = 0.0;
    for (int b = 0; b < v.n; ++b)
      for (int h = 0; h < v.h; ++h)
        for (int w = 0; w < v.w; ++w) {
          const float d = dy[at(v, b, c, h, w)];
          acc += d;
          accd += d;
          m += std::fabs(static_cast<double>(d));
        }
    if (mag != nullptr) mag[c] = m;
    db[c] = accum_f64 ? static_cast<float>(store<double>(alpha, accd, beta, db[c]))
                      : store<float>(alpha, acc, beta, db[c]);
  }
}

extern "C" void oracle_add_tensor(const float* a, const OracleTensor4* avp, float* c,
                                  const OracleTensor4* cvp, float alpha, float beta) {
  const OracleTensor4 av = *avp, cv = *cvp;
  for (int b = 0; b < cv.n; ++b)
    for (int ic = 0; ic < cv.c; ++ic)
      for (int h = 0; h < cv.h; ++h)
        for (int w = 0; w < cv.w; ++w) {
          const float va = a[at(av, av.n == 1 ? 0 : b, av.c == 1 ? 0 : ic, av.h == 1 ? 0 : h,
                                av.w == 1 ? 0 : w)];
          const int64_t ci = at(cv, b, ic, h, w);
          c[ci] = store<float>(alpha, va, beta, c[ci]);
        }
}

namespace {

// cudnn_kernels.metal:356-369; max / clamp with IEEE fmax / fmin semantics.
inline float activate(float v, int mode, float coef) {
  switch (mode) {
    case 0: return 1.0f / (1.0f + std::exp(-v));
    case 1: return std::fmax(v, 0.0f);
    case 2: return std::tanh(v);
    case 3: return std::fmin(std::fmax(v, 0.0f), coef);
    case 4: return v >= 0.0f ? v : coef * (std::exp(v) - 1.0f);
    case 6: return v / (1.0f + std::exp(-v));
    default: return v;
  }
}

}  // namespace

extern "C" void oracle_activation(const float* x, const OracleTensor4* xvp, float* y,
                                  const OracleTensor4* yvp, int mode, float coef, float alpha,
                                  float beta) {
  const OracleTensor4 xv = *xvp, yv = *yvp;
  for (int b = 0; b < xv.n; ++b)
    for (int c = 0; c < xv.c; ++c)
      for (int h = 0; h < xv.h; ++h)
        for (int w = 0; w < xv.w; ++w) {
          const int64_t yi = at(yv, b, c, h, w);
          y[yi] = store<float>(alpha, activate(x[at(xv, b, c, h, w)], mode, coef), beta, y[yi]);
        }
}

extern "C" void oracle_pooling(const float* x, const OracleTensor4* xvp, float* y,
                               const OracleTensor4* yvp, int win_h, int win_w, int pad_h,
                               int pad_w, int stride_h, int stride_w, int mode, float alpha,
                               float beta) {
  const OracleTensor4 xv = *xvp, yv = *yvp;
  const bool is_max = mode == 0 || mode == 3;
  for (int b = 0; b < yv.n; ++b)
    for (int c = 0; c < yv.c; ++c)
      for (int oy = 0; oy < yv.h; ++oy)
        for (int ox = 0; ox < yv.w; ++ox) {
          float acc = is_max ? -INFINITY : 0.0f;
          int count = 0;
          for (int r = 0; r < win_h; ++r) {
            const int iy = oy * stride_h - pad_h + r;
            if (iy < 0 || iy >= xv.h) continue;
            for (int s = 0; s < win_w; ++s) {
              const int ix = ox * stride_w - pad_w + s;
              if (ix < 0 || ix >= xv.w) continue;
              const float v = x[at(xv, b, c, iy, ix)];
              acc = is_max ? std::fmax(acc, v) : acc + v;
              ++count;
            }
          }
          float out = acc;
          if (!is_max) {
            const int denom = (mode == 1) ? win_h * win_w : (count > 1 ? count : 1);
            out = acc / static_cast<float>(denom);
          }
          const int64_t yi = at(yv, b, c, oy, ox);
          y[yi] = store<float>(alpha, out, beta, y[yi]);
        }
}

extern "C" void oracle_bn_inference(const float* x, const OracleTensor4* xvp, float* y,
                                    const OracleTensor4* yvp, const float* scale,
                                    const float* bias, const float* mean, const float* var,
                                    int per_activation, float eps, float alpha, float beta) {
  const OracleTensor4 xv = *xvp, yv = *yvp;
  for (int b = 0; b < xv.n; ++b)
    for (int c = 0; c < xv.c; ++c)
      for (int h = 0; h < xv.h; ++h)
        for (int w = 0; w < xv.w; ++w) {
          const int64_t pi = per_activation ? (static_cast<int64_t>(c) * xv.h + h) * xv.w + w : c;
          const float inv_std = 1.0f / std::sqrt(var[pi] + eps);
          const float nv = std::fma((x[at(xv, b, c, h, w)] - mean[pi]) * inv_std, scale[pi],
                                    bias[pi]);
          const int64_t yi = at(yv, b, c, h, w);
          y[yi] = store<float>(alpha, nv, beta, y[yi]);
        }
}

// Sequential sums in (b, h, w) order as the reference's single thread would take
// them (accum_f64 = 0), or in double (accum_f64 = 1).
extern "C" void oracle_bn_training(const float* x, const OracleTensor4* xvp, float* y,
                                   const OracleTensor4* yvp, const float* scale, const float* bias,
                                   float* running_mean, float* running_var, float* save_mean,
                                   float* save_inv_var, float factor, float eps, float alpha,
                                   float beta, int accum_f64) {
  const OracleTensor4 xv = *xvp, yv = *yvp;
  const int64_t m = static_cast<int64_t>(xv.n) * xv.h * xv.w;
  for (int c = 0; c < xv.c; ++c) {
    float mean, var, total_sq;
    if (accum_f64) {
      double s = 0.0;
      for (int b = 0; b < xv.n; ++b)
        for (int h = 0; h < xv.h; ++h)
          for (int w = 0; w < xv.w; ++w) s += x[at(xv, b, c, h, w)];
      const double md = s / static_cast<double>(m);
      double q = 0.0;
      for (int b = 0; b < xv.n; ++b)
        for (int h = 0; h < xv.h; ++h)
          for (int w = 0; w < xv.w; ++w) {
            const double d = x[at(xv, b, c, h, w)] - md;
            q += d * d;
          }
      mean = static_cast<float>(md);
      total_sq = static_cast<float>(q);
      var = static_cast<float>(q / static_cast<double>(m));
    } else {
      const float inv_m = 1.0f / static_cast<float>(m);
      float s = 0.0f;
      for (int b = 0; b < xv.n; ++b)
        for (int h = 0; h < xv.h; ++h)
          for (int w = 0; w < xv.w; ++w) s += x[at(xv, b, c, h, w)];
      mean = s * inv_m;
      float q = 0.0f;
      for (int b = 0; b < xv.n; ++b)
        for (int h = 0; h < xv.h; ++h)
          for (int w = 0; w < xv.w; ++w) {
            const float d = x[at(xv, b, c, h, w)] - mean;
            q = std::fma(d, d, q);
          }
      total_sq = q;
      var = q * inv_m;
    }
    const float unbiased = (m > 1) ? total_sq / static_cast<float>(m - 1) : var;
    const float inv_std = 1.0f / std::sqrt(var + eps);
    if (save_mean != nullptr) {
      save_mean[c] = mean;
      save_inv_var[c] = inv_std;
    }
    if (running_mean != nullptr) {
      running_mean[c] = (1.0f - factor) * running_mean[c] + factor * mean;
      running_var[c] = (1.0f - factor) * running_var[c] + factor * unbiased;
    }
    for (int b = 0; b < xv.n; ++b)
      for (int h = 0; h < xv.h; ++h)
        for (int w = 0; w < xv.w; ++w) {
          const float nv = std::fma((x[at(xv, b, c, h, w)] - mean) * inv_std, scale[c], bias[c]);
          const int64_t yi = at(yv, b, c, h, w);
          y[yi] = store<float>(alpha, nv, beta, y[yi]);
        }
  }
}
