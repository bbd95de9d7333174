/*
 * curand.h — C ABI of the B200-native Philox4x32-10 generator.
 *
 * Drop-in for the MUDA cuRAND shim: every name, argument list and numeric enum
 * value below follows libraries/rand/include/curand.h of the reference
 * (declarations at curand.h:84-128, enums at curand.h:33-75).  Enums here are
 * plain C enums (int width) instead of the reference's 8-bit enums, so that
 * x86-64 callers binding the return value as `int` read a clean value.
 *
 * Semantics shared by every generator (reference libraries/rand/src/curand_api.mm):
 *   - all RNG types map to Philox4x32-10 (curand_api.mm:44-56 never dispatches on type);
 *   - output j of Philox block i goes to out[4*i + j]; the counter of block i is
 *     i + (offset >> 2) and the key is the 64-bit seed (curand_context.mm:42-73);
 *   - each fp32/uint call advances the offset by 4*ceil(n/4) (curand_api.mm:275);
 *   - curandSetPseudoRandomGeneratorSeed resets the offset to 0 (curand_api.mm:112-113).
 * Device generators launch on the generator's stream and return without
 * synchronising; host generators (curandCreateGeneratorHost) fill host memory.
 */
#ifndef MUDA_B200_CURAND_H_
#define MUDA_B200_CURAND_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>
#include <library_types.h>

#ifdef __cplusplus
extern "C" {
#endif

struct curandGenerator_st;
typedef struct curandGenerator_st* curandGenerator_t;

/* reference curand.h:33-48 */
typedef enum curandStatus {
  CURAND_STATUS_SUCCESS = 0,
  CURAND_STATUS_VERSION_MISMATCH = 100,
  CURAND_STATUS_NOT_INITIALIZED = 101,
  CURAND_STATUS_ALLOCATION_FAILED = 102,
  CURAND_STATUS_TYPE_ERROR = 103,
  CURAND_STATUS_OUT_OF_RANGE = 104,
  CURAND_STATUS_INVALID_VALUE = 104,
  CURAND_STATUS_LENGTH_NOT_MULTIPLE = 105,
  CURAND_STATUS_DOUBLE_PRECISION_REQUIRED = 106,
  CURAND_STATUS_LAUNCH_FAILURE = 201,
  CURAND_STATUS_PREEXISTING_FAILURE = 202,
  CURAND_STATUS_INITIALIZATION_FAILED = 203,
  CURAND_STATUS_ARCH_MISMATCH = 204,
  CURAND_STATUS_INTERNAL_ERROR = 999
} curandStatus_t;

/* reference curand.h:50-63 */
typedef enum curandRngType {
  CURAND_RNG_TEST = 0,
  CURAND_RNG_PSEUDO_DEFAULT = 100,
  CURAND_RNG_PSEUDO_XORWOW = 101,
  CURAND_RNG_PSEUDO_MRG32K3A = 121,
  CURAND_RNG_PSEUDO_MTGP32 = 141,
  CURAND_RNG_PSEUDO_MT19937 = 142,
  CURAND_RNG_PSEUDO_PHILOX4_32_10 = 161,
  CURAND_RNG_QUASI_DEFAULT = 200,
  CURAND_RNG_QUASI_SOBOL32 = 201,
  CURAND_RNG_QUASI_SCRAMBLED_SOBOL32 = 202,
  CURAND_RNG_QUASI_SOBOL64 = 203,
  CURAND_RNG_QUASI_SCRAMBLED_SOBOL64 = 204
} curandRngType_t;

/* reference curand.h:65-70 */
typedef enum curandOrdering {
  CURAND_ORDERING_PSEUDO_BEST = 100,
  CURAND_ORDERING_PSEUDO_DEFAULT = 101,
  CURAND_ORDERING_PSEUDO_SEEDED = 102,
  CURAND_ORDERING_QUASI_DEFAULT = 201
} curandOrdering_t;

/* reference curand.h:72-79 */
typedef enum curandDirectionVectorSet {
  CURAND_DIRECTION_VECTORS_32_JOEKUO6 = 101,
  CURAND_SCRAMBLED_DIRECTION_VECTORS_32_JOEKUO6 = 102,
  CURAND_DIRECTION_VECTORS_64_JOEKUO6 = 103,
  CURAND_SCRAMBLED_DIRECTION_VECTORS_64_JOEKUO6 = 104
} curandDirectionVectorSet_t;
typedef unsigned int curandDirectionVectors32_t[32];

/* Lifecycle — reference curand_api.mm:44-82 */
curandStatus_t curandCreateGenerator(curandGenerator_t* generator, curandRngType_t rng_type);
curandStatus_t curandCreateGeneratorHost(curandGenerator_t* generator, curandRngType_t rng_type);
curandStatus_t curandDestroyGenerator(curandGenerator_t generator);

/* Configuration — reference curand_api.mm:84-149 */
curandStatus_t curandSetStream(curandGenerator_t generator, cudaStream_t stream);
curandStatus_t curandGetStream(curandGenerator_t generator, cudaStream_t* stream);
curandStatus_t curandSetPseudoRandomGeneratorSeed(curandGenerator_t generator,
                                                  unsigned long long seed);
curandStatus_t curandSetGeneratorOffset(curandGenerator_t generator, unsigned long long offset);
curandStatus_t curandSetGeneratorOrdering(curandGenerator_t generator, curandOrdering_t order);
/* reference curand_api.mm:137-149: 1 .. 20000 dimensions, stored (every generator
 * runs the Philox stream, as in the reference) */
curandStatus_t curandSetQuasiRandomGeneratorDimensions(curandGenerator_t generator,
                                                       unsigned int num_dimensions);
curandStatus_t curandGetVersion(int* version);
curandStatus_t curandGetProperty(libraryPropertyType type, int* value);

/* Generation — reference curand_api.mm:181-343 */
curandStatus_t curandGenerate(curandGenerator_t generator, unsigned int* outputPtr, size_t num);
curandStatus_t curandGenerateUniform(curandGenerator_t generator, float* outputPtr, size_t num);
curandStatus_t curandGenerateNormal(curandGenerator_t generator, float* outputPtr, size_t n,
                                    float mean, float stddev);
/* exp of the normal stream; offset advances as for curandGenerateNormal
 * (reference curand_api.mm:363-409) */
curandStatus_t curandGenerateLogNormal(curandGenerator_t generator, float* outputPtr, size_t n,
                                       float mean, float stddev);
/* Double precision: one Philox block per two values, block index offset / 2,
 * offset += 2 * ceil(n / 2) (reference curand_context.mm:115-223, curand_api.mm:279-297,
 * 344-361, 411-438).  The uniform is bit-identical to the reference. */
curandStatus_t curandGenerateUniformDouble(curandGenerator_t generator, double* outputPtr,
                                           size_t num);
curandStatus_t curandGenerateNormalDouble(curandGenerator_t generator, double* outputPtr, size_t n,
                                          double mean, double stddev);
curandStatus_t curandGenerateLogNormalDouble(curandGenerator_t generator, double* outputPtr,
                                             size_t n, double mean, double stddev);
/* Poisson counts, one Philox block index per output, offset += n (reference
 * curand_api.mm:440-479, curand_kernels.metal:212-264).  Device and host generators
 * produce the same stream: extra uniforms come from counter word 2 on both (the
 * reference's host path steps counter word 1 and computes in double instead). */
curandStatus_t curandGeneratePoisson(curandGenerator_t generator, unsigned int* outputPtr, size_t n,
                                     double lambda);

/* Direction vectors and scramble constants — reference curand_api.mm:488-507 */
curandStatus_t curandGetDirectionVectors32(curandDirectionVectors32_t* vectors[],
                                           curandDirectionVectorSet_t set);
curandStatus_t curandGetScrambleConstants32(const unsigned int** constants);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_CURAND_H_ */
