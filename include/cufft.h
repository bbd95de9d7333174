/*
 * cufft.h — C ABI of the B200-native batched C2C FFT.
 *
 * Drop-in for the MUDA cuFFT shim's hot path: names, argument lists and numeric
 * values follow libraries/fft/include/cufft.h of the reference (directions
 * cufft.h:20-21, results cufft.h:26-43, types cufft.h:49-56, declarations
 * cufft.h:71-93).  Enums are int-width; cufftHandle is an opaque pointer, as in
 * the reference (cufft.h:68; NVIDIA's own cuFFT uses an int there).
 *
 * Conventions kept from the reference (libraries/fft/src/cufft_exec.mm):
 *   - X[k] = sum_n x[n] * exp(sign * 2*pi*i * n*k / N), sign -1 for CUFFT_FORWARD and
 *     +1 for CUFFT_INVERSE; the inverse is NOT scaled by 1/N (cufft_exec.mm:149);
 *   - idata == odata (in place) is allowed;
 *   - inembed/onembed == NULL forces unit stride and dense batch distance
 *     (cufft_plan.mm:68-83).
 */
#ifndef MUDA_B200_CUFFT_H_
#define MUDA_B200_CUFFT_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CUFFT_FORWARD (-1)
#define CUFFT_INVERSE (1)

typedef enum cufftResult_t {
  CUFFT_SUCCESS = 0,
  CUFFT_INVALID_PLAN = 1,
  CUFFT_ALLOC_FAILED = 2,
  CUFFT_INVALID_TYPE = 3,
  CUFFT_INVALID_VALUE = 4,
  CUFFT_INTERNAL_ERROR = 5,
  CUFFT_EXEC_FAILED = 6,
  CUFFT_SETUP_FAILED = 7,
  CUFFT_INVALID_SIZE = 8,
  CUFFT_UNALIGNED_DATA = 9,
  CUFFT_INCOMPLETE_PARAMETER_LIST = 10,
  CUFFT_INVALID_DEVICE = 11,
  CUFFT_PARSE_ERROR = 12,
  CUFFT_NO_WORKSPACE = 13,
  CUFFT_NOT_IMPLEMENTED = 14,
  CUFFT_NOT_SUPPORTED = 16
} cufftResult;

typedef enum cufftType_t {
  CUFFT_R2C = 0x2a,
  CUFFT_C2R = 0x2c,
  CUFFT_C2C = 0x29,
  CUFFT_D2Z = 0x6a,
  CUFFT_Z2D = 0x6c,
  CUFFT_Z2Z = 0x69
} cufftType;

typedef float cufftReal;
typedef float2 cufftComplex;

struct cufftContext;
typedef struct cufftContext* cufftHandle;

/* Plans — reference cufft_plan.mm:157-318 */
cufftResult cufftCreate(cufftHandle* handle);
cufftResult cufftPlan1d(cufftHandle* plan, int nx, cufftType type, int batch);
/* 2-D / 3-D plans (nx outermost, batch 1) — reference cufft_plan.mm:179-196, 227-261 */
cufftResult cufftPlan2d(cufftHandle* plan, int nx, int ny, cufftType type);
cufftResult cufftPlan3d(cufftHandle* plan, int nx, int ny, int nz, cufftType type);
cufftResult cufftMakePlan2d(cufftHandle plan, int nx, int ny, cufftType type, size_t* workSize);
cufftResult cufftMakePlan3d(cufftHandle plan, int nx, int ny, int nz, cufftType type,
                            size_t* workSize);
cufftResult cufftPlanMany(cufftHandle* plan, int rank, int* n, int* inembed, int istride, int idist,
                          int* onembed, int ostride, int odist, cufftType type, int batch);
cufftResult cufftMakePlan1d(cufftHandle plan, int nx, cufftType type, int batch, size_t* workSize);
cufftResult cufftMakePlanMany(cufftHandle plan, int rank, int* n, int* inembed, int istride,
                              int idist, int* onembed, int ostride, int odist, cufftType type,
                              int batch, size_t* workSize);
cufftResult cufftSetStream(cufftHandle plan, cudaStream_t stream);
cufftResult cufftGetSize(cufftHandle handle, size_t* workSize);
cufftResult cufftDestroy(cufftHandle plan);

/* Execution — reference cufft_exec.mm:101-211 */
cufftResult cufftExecC2C(cufftHandle plan, cufftComplex* idata, cufftComplex* odata, int direction);
/* Real-data transforms — reference cufft_exec.mm:213-438: R2C forward over all
   axes keeping entries 0 .. n/2 of the last axis; C2R the unnormalised inverse
   from that half spectrum (the imaginary parts of its first and, for even n,
   middle entries are ignored, as in the reference).  The input is not modified. */
cufftResult cufftExecR2C(cufftHandle plan, cufftReal* idata, cufftComplex* odata);
cufftResult cufftExecC2R(cufftHandle plan, cufftComplex* idata, cufftReal* odata);

/* Allocation-free execution.  No counterpart in the reference: an addition of
 * this library for callers that cannot allocate device memory when they need a
 * transform (inside an allocator or memory-pool callback, in real-time paths
 * that forbid allocation after start-up, or under a hard memory cap), since a
 * plan allocates its tables and workspace.
 *
 * Transforms `batch` contiguous sequences of n complex values (n a power of two,
 * 2 <= n <= 1048576; larger or non-power-of-two n returns CUFFT_INVALID_SIZE),
 * same conventions as cufftExecC2C (sign from `direction`, no scaling, in place
 * allowed), on `stream`.  Twiddle tables and the workspace live in one fixed
 * device array of about 16.3 MiB that the library reserves on every GPU it is
 * loaded on and keeps until the process exits; the call calls no cudaMalloc,
 * cudaFree or other allocator.  The first call on a device looks up that
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  Every call rewrites the tables and workspace it reads, so
 * no state carries over from one call to the next, but all calls share the one
 * array: calls that can overlap on the GPU (different streams, or different
 * host threads) race and must be serialised by the caller. */
cufftResult cufftExecC2CNoAlloc(cufftComplex* idata, cufftComplex* odata, long long n,
                                long long batch, int direction, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_CUFFT_H_ */
