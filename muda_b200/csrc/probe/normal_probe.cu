// normal_probe.cu — error budget of the cuRAND normal transform, measured exhaustively.
//
// Not part of the drop-in API.  The normal transform (rand/box_muller.cuh, the code the
// Philox fill kernels run) takes -2 ln u and sin / cos from the hardware's approximate
// lg2 / sin / cos where those are accurate enough.  Its error bound rests on three
// maxima, each over every fp32 value its step can see; mb200ProbeNormalError measures
// them against double precision and writes, as floats into out[0..5]:
//   0  max |r - sqrt(-2 ln u)| / max(1, sqrt(-2 ln u)) over all u in [2^-32, 1], r the
//      shipped radius (hardware lg2, the series in d = u - 1 above u = 0.995);
//   1  max |cos - cos(theta)|, 2  max |sin - sin(theta)| over all theta in
//      [0, float(2 pi)], hardware sin / cos after the pi reduction (the common path);
//   3  max |cos - cos(theta)|, 4  max |sin - sin(theta)| for the polynomial path (the
//      fallback for radii above 3.75);
//   5  the largest radius for which the hardware path is used (3.75).
#include <cuda_runtime.h>

#include <cstdint>

#include "rand/box_muller.cuh"

#pragma GCC visibility push(default)
#include "mb200_probe.h"
#pragma GCC visibility pop

namespace mb200::rand {

__device__ __forceinline__ void record(unsigned* slot, double err) {
  float v = static_cast<float>(fabs(err));
  if (!(v == v)) v = 3.0e38f;  // NaN counts as the worst error
  atomicMax(slot, __float_as_uint(v));
}

__global__ void radius_probe(unsigned lo, unsigned hi, unsigned* res) {
  for (unsigned b = lo + blockIdx.x * blockDim.x + threadIdx.x; b <= hi && b >= lo;
       b += gridDim.x * blockDim.x) {
    const float u = __uint_as_float(b);
    const Pair w = neg2_log_hw<true>(Pair{u, u});
    const float r = sqrt_approx(w.x);
    const double re = sqrt(-2.0 * log(static_cast<double>(u)));
    record(res + 0, (r - re) / fmax(1.0, re));
    if (b == hi) break;
  }
}

__global__ void angle_probe(unsigned lo, unsigned hi, unsigned* res) {
  for (unsigned b = lo + blockIdx.x * blockDim.x + threadIdx.x; b <= hi && b >= lo;
       b += gridDim.x * blockDim.x) {
    const float th = __uint_as_float(b);
    const double c = cos(static_cast<double>(th)), s = sin(static_cast<double>(th));
    Pair p0, p1, zc, zs;
    // radius 1: the products r*cos, r*sin are the bare cos / sin
    polar_pairs_hw<true>(Pair{th, th}, Pair{1.0f, 1.0f}, p0, p1);
    record(res + 1, p0.x - c);
    record(res + 2, p0.y - s);
    polar2<true, true>(Pair{th, th}, Pair{1.0f, 1.0f}, zc, zs);
    record(res + 3, zc.x - c);
    record(res + 4, zs.x - s);
    if (b == hi) break;
  }
}

__global__ void write_threshold(unsigned* res) { res[5] = __float_as_uint(kRadHw); }

}  // namespace mb200::rand

extern "C" int mb200ProbeNormalError(float* out, cudaStream_t stream) {
  using namespace mb200::rand;
  if (out == nullptr) return 1;
  unsigned* res = reinterpret_cast<unsigned*>(out);
  if (cudaMemsetAsync(res, 0, 6 * sizeof(unsigned), stream) != cudaSuccess) return 2;
  radius_probe<<<148 * 8, 256, 0, stream>>>(0x2F800000u, 0x3F800000u, res);  // 2^-32 .. 1
  angle_probe<<<148 * 8, 256, 0, stream>>>(0u, 0x40C90FDBu, res);            // 0 .. 2 pi
  write_threshold<<<1, 1, 0, stream>>>(res);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}
