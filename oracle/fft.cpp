// fft.cpp — restatement of the reference's C2C FFT arithmetic.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Follows libraries/fft/src/cufft_exec.mm:101-211 and the kernels it drives:
//   gather   in[b*idist + e*istride] -> work[b][e]           cufft_kernels.metal:13-26
//   per axis, innermost first (inner_stride = product of later dims):
//     power of two: log2(L) radix-2 Stockham stages           cufft_kernels.metal:255-296,
//                   (half_m = 1, 2, 4, ...), ping-pong        cufft_exec.mm:58-74
//     otherwise:    O(L^2) DFT                                cufft_kernels.metal:298-325
//   scatter  work[b][e] -> out[b*odist + e*ostride]          cufft_kernels.metal:28-41
// sign -1 forward, +1 inverse, no scaling.  T = float restates the reference's
// single-precision arithmetic (twiddle by sincos of a float angle); T = double is
// the ground truth used for error bounds.
#include <cmath>
#include <complex>
#include <cstdint>
#include <vector>

#include "oracle.h"
#include "parallel.h"

namespace {

template <typename T>
using cx = std::complex<T>;

template <typename T>
cx<T> cmul_ref(cx<T> a, cx<T> b) {
  // float2(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x))  (cufft_kernels.metal:10-12)
  return cx<T>(std::fma(a.real(), b.real(), -a.imag() * b.imag()),
               std::fma(a.real(), b.imag(), a.imag() * b.real()));
}

template <typename T>
void stockham_stage(const cx<T>* src, cx<T>* dst, std::uint32_t total, std::uint32_t axis_len,
                    std::uint32_t inner_stride, std::uint32_t half_m, T sign) {
  const std::uint32_t axis_mask = axis_len - 1u;
  std::uint32_t log2_len = 0;
  while ((1u << log2_len) < axis_len) ++log2_len;
  for (std::uint32_t tid = 0; tid < total; ++tid) {
    std::uint32_t inner_idx = 0, k, outer_idx;
    if (inner_stride == 1u) {
      k = tid & axis_mask;
      outer_idx = tid >> log2_len;
    } else {
      inner_idx = tid % inner_stride;
      const std::uint32_t temp = tid / inner_stride;
      k = temp & axis_mask;
      outer_idx = temp >> log2_len;
    }
    const std::uint32_t m = half_m << 1u;
    const std::uint32_t r = k & (m - 1u);
    const std::uint32_t r_mod = k & (half_m - 1u);
    const std::uint32_t j_half_m = (k & ~(m - 1u)) >> 1u;
    const std::uint32_t base = outer_idx * (axis_len * inner_stride) + inner_idx;
    const std::uint32_t idx0 = base + (j_half_m + r_mod) * inner_stride;
    const std::uint32_t idx1 = idx0 + (axis_len >> 1u) * inner_stride;
    const T angle = sign * (static_cast<T>(3.14159265358979323846) * static_cast<T>(r_mod)) /
                    static_cast<T>(half_m);
    const cx<T> w(std::cos(angle), std::sin(angle));
    const cx<T> u = src[idx0];
    const cx<T> v = cmul_ref(w, src[idx1]);
    dst[tid] = (r < half_m) ? (u + v) : (u - v);
  }
}

template <typename T>
void axis_dft(const cx<T>* src, cx<T>* dst, std::uint32_t total, std::uint32_t axis_len,
              std::uint32_t inner_stride, T sign) {
  for (std::uint32_t tid = 0; tid < total; ++tid) {
    const std::uint32_t inner_idx = tid % inner_stride;
    const std::uint32_t temp = tid / inner_stride;
    const std::uint32_t k = temp % axis_len;
    const std::uint32_t outer_idx = temp / axis_len;
    const std::uint32_t base = outer_idx * (axis_len * inner_stride) + inner_idx;
    cx<T> acc(0, 0);
    if constexpr (sizeof(T) == 4) {
      const T base_angle =
          sign * (static_cast<T>(6.28318530717958647692) * static_cast<T>(k)) /
          static_cast<T>(axis_len);
      for (std::uint32_t n = 0; n < axis_len; ++n) {
        const T angle = base_angle * static_cast<T>(n);
        acc += cmul_ref(src[base + n * inner_stride], cx<T>(std::cos(angle), std::sin(angle)));
      }
    } else {
      // ground truth: exact angle index (n*k mod L)
      for (std::uint32_t n = 0; n < axis_len; ++n) {
        const std::uint64_t nk = (static_cast<std::uint64_t>(n) * k) % axis_len;
        const T angle = sign * static_cast<T>(6.283185307179586476925286766559) *
                        static_cast<T>(nk) / static_cast<T>(axis_len);
        acc += src[base + n * inner_stride] * cx<T>(std::cos(angle), std::sin(angle));
      }
    }
    dst[tid] = acc;
  }
}

template <typename T>
void transform_one(const float* in, float* out, int rank, const int* dims, std::int64_t b,
                   std::int64_t istride, std::int64_t idist, std::int64_t ostride,
                   std::int64_t odist, int sign) {
  std::uint32_t total = 1;
  for (int i = 0; i < rank; ++i) total *= static_cast<std::uint32_t>(dims[i]);
  std::vector<cx<T>> cur(total), scr(total);
  for (std::uint32_t e = 0; e < total; ++e) {
    const std::int64_t s = 2 * (b * idist + static_cast<std::int64_t>(e) * istride);
    cur[e] = cx<T>(in[s], in[s + 1]);
  }
  std::uint32_t inner = 1;
  for (int axis = rank - 1; axis >= 0; --axis) {
    const auto len = static_cast<std::uint32_t>(dims[axis]);
    if (len > 1) {
      if ((len & (len - 1)) == 0) {
        for (std::uint32_t half_m = 1; half_m < len; half_m <<= 1) {
          stockham_stage<T>(cur.data(), scr.data(), total, len, inner, half_m,
                            static_cast<T>(sign));
          cur.swap(scr);
        }
      } else {
        axis_dft<T>(cur.data(), scr.data(), total, len, inner, static_cast<T>(sign));
        cur.swap(scr);
      }
    }
    inner *= len;
  }
  for (std::uint32_t e = 0; e < total; ++e) {
    const std::int64_t d = 2 * (b * odist + static_cast<std::int64_t>(e) * ostride);
    out[d] = static_cast<float>(cur[e].real());
    out[d + 1] = static_cast<float>(cur[e].imag());
  }
}

}  // namespace

extern "C" void oracle_fft_c2c(const float* in, float* out, int rank, const int* dims,
                               int64_t batch, int64_t istride, int64_t idist, int64_t ostride,
                               int64_t odist, int sign, int use_double, double* out_f64,
                               int threads) {
  oracle_detail::parallel_for(0, batch, threads, [&](std::int64_t b) {
    if (use_double) {
      // ground truth written to out_f64 (interleaved re, im) with the output layout
      std::uint32_t total = 1;
      for (int i = 0; i < rank; ++i) total *= static_cast<std::uint32_t>(dims[i]);
      std::vector<cx<double>> cur(total), scr(total);
      for (std::uint32_t e = 0; e < total; ++e) {
        const std::int64_t s = 2 * (b * idist + static_cast<std::int64_t>(e) * istride);
        cur[e] = cx<double>(in[s], in[s + 1]);
      }
      std::uint32_t inner = 1;
      for (int axis = rank - 1; axis >= 0; --axis) {
        const auto len = static_cast<std::uint32_t>(dims[axis]);
        if (len > 1) {
          if ((len & (len - 1)) == 0) {
            for (std::uint32_t half_m = 1; half_m < len; half_m <<= 1) {
              stockham_stage<double>(cur.data(), scr.data(), total, len, inner, half_m, sign);
              cur.swap(scr);
            }
          } else {
            axis_dft<double>(cur.data(), scr.data(), total, len, inner, sign);
            cur.swap(scr);
          }
        }
        inner *= len;
      }
      for (std::uint32_t e = 0; e < total; ++e) {
        const std::int64_t d = 2 * (b * odist + static_cast<std::int64_t>(e) * ostride);
        out_f64[d] = cur[e].real();
        out_f64[d + 1] = cur[e].imag();
      }
    } else {
      transform_one<float>(in, out, rank, dims, b, istride, idist, ostride, odist, sign);
    }
  });
}
