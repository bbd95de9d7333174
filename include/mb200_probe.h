/* mb200_probe.h — benchmark probes of this repository (not part of the drop-in API).
 *
 * No counterpart in the reference: these entry points exist only to measure a
 * hardware ceiling against which a library kernel is judged. */
#ifndef MUDA_B200_PROBE_H_
#define MUDA_B200_PROBE_H_

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Streams n int32 indices (per_lane 1, or 4 read as one 16-byte load; idx then
 * 16-byte aligned) and gathers x[idx[i]] with L2-only loads, writing one partial sum
 * per thread to out (grid * 256 floats).  Returns 0 on success, 1 on a bad argument,
 * 2 on a launch error.  The indices must lie inside x. */
int mb200ProbeGather(const float* x, const int* idx, long long n, int per_lane, float* out,
                     unsigned grid, cudaStream_t stream);

/* Streams n int32 indices (per_lane as for mb200ProbeGather) and adds 1.0f to
 * y[idx[i]] for each by a reduction that returns nothing (red.global.add.f32), so that
 * y[j] gains the count of j in idx (exact below 2^24 per element).  Returns 0 on
 * success, 1 on a bad argument, 2 on a launch error.  The indices must lie inside y. */
int mb200ProbeScatter(float* y, const int* idx, long long n, int per_lane, unsigned grid,
                      cudaStream_t stream);

/* For each of n int32 indices, gathers row idx[i] of a row-major float matrix of 64
 * columns (b 16-byte aligned; 16 lanes load one 16-byte slice each, L2-only) and writes
 * one partial sum per thread to out (grid * 256 floats).  Returns 0 on success, 1 on a
 * bad argument, 2 on a launch error.  The indices must lie inside b's rows. */
int mb200ProbeRowGather(const float* b, const int* idx, long long n, float* out, unsigned grid,
                        cudaStream_t stream);

/* Error budget of the cuRAND normal transform, every fp32 input of each step: writes
 * six floats to device memory `out` (radius error / max(1, r); hardware cos, sin error;
 * polynomial cos, sin error; the radius threshold of the hardware path).  Returns 0 on
 * success, 1 on a bad argument, 2 on a launch error. */
int mb200ProbeNormalError(float* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_PROBE_H_ */
