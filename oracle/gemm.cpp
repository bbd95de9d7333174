// gemm.cpp — restatement of the reference's GEMM arithmetic.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Follows muda_cublas_sgemm_strided_batched and muda_cublas_hgemm_strided_batched
// (libraries/blas/shaders/cublas_kernels.metal:969-1045): column-major, for each
// (batch, row, col) acc = fma(op(A)[row][p], op(B)[p][col], acc) for p = 0..K-1,
// then C = fma(alpha, acc, beta == 0 ? 0 : beta * C).  16-bit operands (fp16 as in
// the reference, bf16 as this library's extension) are widened exactly to float
// and the result is rounded to nearest even.  accum_f64 accumulates in double
// instead (ground truth for error bounds); rows/cols restrict the evaluated
// entries (a sampled check of a large product).
#include <cmath>
#include <cstdint>
#include <cstring>

#include "oracle.h"
#include "parallel.h"

namespace {

float half_to_f32(std::uint16_t h) {
  const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
  std::uint32_t exp = (h >> 10) & 0x1Fu;
  std::uint32_t man = h & 0x3FFu;
  std::uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      exp = 113;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --exp;
      }
      bits = sign | (exp << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

std::uint16_t f32_to_half(float f) {
  std::uint32_t x;
  std::memcpy(&x, &f, 4);
  const std::uint32_t sign = (x >> 16) & 0x8000u;
  const std::uint32_t ax = x & 0x7FFFFFFFu;
  if (ax > 0x7F800000u) return static_cast<std::uint16_t>(sign | 0x7E00u);  // NaN
  if (ax >= 0x477FF000u) return static_cast<std::uint16_t>(sign | 0x7C00u);  // overflow -> inf
  if (ax < 0x38800000u) {  // subnormal half (or zero)
    const float a = std::fabs(f) * 16777216.0f;  // scale by 2^24, exact
    const float r = std::nearbyint(a);            // round to nearest even
    return static_cast<std::uint16_t>(sign | static_cast<std::uint32_t>(r));
  }
  const std::uint32_t lsb = (ax >> 13) & 1u;
  const std::uint32_t rounded = ax + 0xFFFu + lsb;
  return static_cast<std::uint16_t>(sign | ((rounded - 0x38000000u) >> 13));
}

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
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<std::uint16_t>(u >> 16);
}

float load(const void* p, std::int64_t i, int type) {
  if (type == 0) return static_cast<const float*>(p)[i];
  const std::uint16_t v = static_cast<const std::uint16_t*>(p)[i];
  return type == 1 ? half_to_f32(v) : bf16_to_f32(v);
}

void store(void* p, std::int64_t i, float v, int type) {
  if (type == 0) {
    static_cast<float*>(p)[i] = v;
  } else {
    static_cast<std::uint16_t*>(p)[i] = type == 1 ? f32_to_half(v) : f32_to_bf16(v);
  }
}

}  // namespace

extern "C" float oracle_half_round(float v) { return half_to_f32(f32_to_half(v)); }

extern "C" void oracle_gemm(int type, int transa, int transb, int m, int n, int k, float alpha,
                            const void* A, int64_t lda, int64_t stride_a, const void* B,
                            int64_t ldb, int64_t stride_b, float beta, void* C, int64_t ldc,
                            int64_t stride_c, int batch, int accum_f64, const int32_t* rows,
                            const int32_t* cols, int64_t n_entries, int threads) {
  const std::int64_t total =
      (rows != nullptr) ? n_entries : static_cast<std::int64_t>(batch) * m * n;
  oracle_detail::parallel_for(0, total, threads, [&](std::int64_t t) {
    std::int64_t z, row, col;
    if (rows != nullptr) {
      // sampled entries of batch 0..batch-1: (rows[t], cols[t]) encode row and
      // batch*n + col
      row = rows[t];
      z = cols[t] / n;
      col = cols[t] % n;
    } else {
      row = t % m;
      col = (t / m) % n;
      z = t / (static_cast<std::int64_t>(m) * n);
    }
    const std::int64_t ab = z * stride_a, bb = z * stride_b, cb = z * stride_c;
    float acc = 0.0f;
    double acc_d = 0.0;
    for (int p = 0; p < k; ++p) {
      const float a = transa ? load(A, ab + p + row * lda, type) : load(A, ab + row + p * lda, type);
      const float b = transb ? load(B, bb + col + p * ldb, type) : load(B, bb + p + col * ldb, type);
      if (accum_f64) {
        acc_d += static_cast<double>(a) * static_cast<double>(b);
      } else {
        acc = std::fma(a, b, acc);
      }
    }
    const std::int64_t ci = cb + row + col * ldc;
    if (accum_f64) {
      const double prev = (beta == 0.0f) ? 0.0 : static_cast<double>(beta) * load(C, ci, type);
      store(C, ci, static_cast<float>(static_cast<double>(alpha) * acc_d + prev), type);
    } else {
      const float prev = (beta == 0.0f) ? 0.0f : (beta * load(C, ci, type));
      store(C, ci, std::fma(alpha, acc, prev), type);
    }
  });
}
