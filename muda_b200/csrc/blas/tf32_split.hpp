// tf32_split.hpp — fp32 -> (hi, lo) tf32 planes for the split-tf32 tensor-core path.
//
// hi = x truncated toward zero to tf32 (exactly representable, same sign as x),
// lo = x - hi (exact, |lo| < 2^-10 |x|, same sign as x) rounded to the nearest
// tf32 value.  x*y = hi_x*hi_y + hi_x*lo_y + lo_x*hi_y + lo_x*lo_y; the
// tensor-core kernels drop the last term (below 2^-20 |x*y|) and lo's rounding
// costs at most 2^-22 |x| per operand, so each product is within about 1.5 * 2^-20
// relative.
// Special values follow fp32 arithmetic: hi and lo always share the sign of x,
// an x that tf32 holds exactly gets lo = x * 2^-40 instead of 0 (a relative
// change of 2^-40, far below fp32 rounding) so that an infinite partner never
// meets a zero lo (inf * 0 = nan), and inf / nan are stored in both planes.
// Products with an infinity therefore come out infinite with the right sign,
// and nan propagates.
#pragma once

#include <cuda_runtime_api.h>

#include <cstdint>

namespace mb200::tc {

#ifdef __CUDACC__
// The (hi, lo) pair of one value, as described above.
__device__ __forceinline__ void tf32_split_value(float x, float& hi, float& lo) {
  const unsigned b = __float_as_uint(x);
  if ((b & 0x7F800000u) == 0x7F800000u) {  // inf / nan: both planes carry x
    hi = x;
    lo = x;
    return;
  }
  hi = __uint_as_float(b & 0xFFFFE000u);  // toward zero: lo keeps the sign of x
  float r = __fsub_rn(x, hi);              // exact
  if (r == 0.0f) r = __fmul_rn(x, 0x1p-40f);
  unsigned t;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(r));
  lo = __uint_as_float(t);
}
#endif

// Element (r, k) of matrix z of a strided fp32 batch lives at
// src[z*zs + r*rs + k*ks].  Writes the planes K-major:
//   dst[((p*batch + z)*rows + r)*ldk + k],  p = 0 (hi) or 1 (lo),  0 <= k < cols,
// leaving the padding columns cols <= k < ldk untouched.  Reads are coalesced
// along whichever of k or r is contiguous (ks == 1 or rs == 1); writes along k.
cudaError_t launch_tf32_split(const float* src, long long rows, long long cols, int batch,
                              long long rs, long long ks, long long zs, float* dst,
                              long long ldk, cudaStream_t stream) noexcept;

// One matrix of a split pass: the arguments of launch_tf32_split.
struct SplitJob {
  const float* src;
  long long rows, cols;
  int batch;
  long long rs, ks, zs;
  float* dst;
  long long ldk;
};

// Splits two matrices in one launch (e.g. both GEMM operands).
cudaError_t launch_tf32_split_pair(const SplitJob& a, const SplitJob& b,
                                   cudaStream_t stream) noexcept;

// Convolution filter of K output channels, C input channels and R x S taps,
// stored KRSC (krsc) or KCRS, written as planes dst[p][k][(r*S + s)*C + c].
cudaError_t launch_tf32_split_filter(const float* w, int K, int C, int R, int S, bool krsc,
                                     float* dst, cudaStream_t stream) noexcept;

}  // namespace mb200::tc
