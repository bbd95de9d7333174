// curand_api.cpp — cuRAND C ABI over the sm_100a Philox kernels.
//
// Mirrors libraries/rand/src/curand_api.mm of the reference: same entry points,
// argument checks and status codes, same generator state (seed, offset, stream)
// and the same offset rule (offset += 4*ceil(n/4) per call, curand_api.mm:275).
// The generator mutex is held across the launch and the offset update, so
// concurrent calls on one generator serialise and each sees a distinct range
// (curand_api.mm:256-276).
//
// Host generators (curandCreateGeneratorHost) deliver into host memory.  The
// numbers are still produced by the GPU kernels: each call generates into a
// device staging buffer owned by the generator and copies the result to the
// caller's host array before returning (the reference returns only once a host
// generator has filled the array, curand_context.mm:95-113).
#pragma GCC visibility push(default)
#include "curand.h"
#pragma GCC visibility pop

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <memory>
#include <mutex>

#include "common/device.hpp"
#include "common/registry.hpp"
#include "rand/philox.hpp"

namespace {

using mb200::rand::Dist;

constexpr int kCurandVersion = 10200;
// Host generators stream through a staging buffer of at most this many words.
constexpr std::uint64_t kStagingWords = std::uint64_t{1} << 26;  // 256 MiB

struct Generator {
  std::mutex mu;
  curandRngType_t rng_type = CURAND_RNG_PSEUDO_DEFAULT;
  bool host_target = false;
  cudaStream_t stream = nullptr;
  std::uint64_t seed = 0;
  std::uint64_t offset = 0;
  curandOrdering_t ordering = CURAND_ORDERING_PSEUDO_DEFAULT;
  unsigned int dimensions = 1;
  void* staging = nullptr;  // device buffer of a host generator
  int staging_device = -1;

  ~Generator() {
    if (staging != nullptr) {
      int prev = -1;
      (void)cudaGetDevice(&prev);
      if (staging_device >= 0) (void)cudaSetDevice(staging_device);
      (void)cudaFree(staging);
      if (prev >= 0) (void)cudaSetDevice(prev);
    }
  }
};

using GeneratorTable = mb200::Registry<Generator, mb200::ObjKind::kRandGenerator>;

GeneratorTable& generators() {
  static GeneratorTable t;
  return t;
}

curandStatus_t create(curandGenerator_t* out, curandRngType_t type, bool host) {
  if (out == nullptr) return CURAND_STATUS_ALLOCATION_FAILED;  // curand_api.mm:45-47
  auto g = std::make_shared<Generator>();
  g->rng_type = type;
  g->host_target = host;
  curandGenerator_t h = generators().add<curandGenerator_t>(std::move(g));
  if (h == nullptr) return CURAND_STATUS_ALLOCATION_FAILED;
  *out = h;
  return CURAND_STATUS_SUCCESS;
}

// One generation request: which stream, its parameters, and the reference's
// offset rule for it.
struct Request {
  enum Kind { kF32, kF64, kPoisson } kind = kF32;
  Dist dist = Dist::kUint32;
  float mean = 0.0f, stddev = 1.0f;
  double mean_d = 0.0, stddev_d = 1.0;
  float lambda = 0.0f, exp_neg_lambda = 1.0f;

  std::size_t elem_bytes() const { return kind == kF64 ? 8 : 4; }
  std::uint64_t per_block() const { return kind == kF32 ? 4 : (kind == kF64 ? 2 : 1); }
  // Philox block of the first element (curand_api.mm:266, curand_context.mm:125, :255)
  std::uint64_t first_block(std::uint64_t offset) const {
    return kind == kF32 ? offset >> 2 : (kind == kF64 ? offset >> 1 : offset);
  }
  // offset advance of a call of n elements (curand_api.mm:275, curand_context.mm:141, :291)
  std::uint64_t advance(std::uint64_t n) const {
    const std::uint64_t pb = per_block();
    return pb * ((n + pb - 1) / pb);
  }
  cudaError_t launch(void* out, std::uint64_t n, std::uint64_t seed, std::uint64_t block,
                     cudaStream_t st) const {
    switch (kind) {
      case kF64:
        return mb200::rand::launch_philox_fill_f64(dist, static_cast<double*>(out), n, seed, block,
                                                   mean_d, stddev_d, st);
      case kPoisson:
        return mb200::rand::launch_philox_poisson(static_cast<unsigned int*>(out), n, seed, block,
                                                  lambda, exp_neg_lambda, st);
      default:
        return mb200::rand::launch_philox_fill(dist, out, n, seed, block, mean, stddev, st);
    }
  }
};

// Launches one device fill and advances the offset; caller holds g.mu.
curandStatus_t device_fill(Generator& g, const Request& q, void* out, std::uint64_t n) {
  const cudaError_t e = q.launch(out, n, g.seed, q.first_block(g.offset), g.stream);
  if (e != cudaSuccess) return CURAND_STATUS_LAUNCH_FAILURE;
  g.offset += q.advance(n);
  return CURAND_STATUS_SUCCESS;
}

// Host generator: chunks of the staging buffer, each a whole number of Philox
// blocks, so each chunk starts on a block boundary and the chunked stream equals
// the one-shot stream.
curandStatus_t host_fill(Generator& g, const Request& q, void* out, std::uint64_t n) {
  const int dev = mb200::current_device();
  if (dev < 0) return CURAND_STATUS_INITIALIZATION_FAILED;
  if (g.staging == nullptr || g.staging_device != dev) {
    if (g.staging != nullptr) (void)cudaFree(g.staging);
    g.staging = nullptr;
    if (cudaMalloc(&g.staging, kStagingWords * 4) != cudaSuccess) {
      (void)cudaGetLastError();
      return CURAND_STATUS_ALLOCATION_FAILED;
    }
    g.staging_device = dev;
  }
  const std::size_t eb = q.elem_bytes();
  const std::uint64_t pb = q.per_block();
  const std::uint64_t chunk = (kStagingWords * 4 / eb) / pb * pb;
  const std::uint64_t first = q.first_block(g.offset);
  auto* dst = static_cast<unsigned char*>(out);
  std::uint64_t done = 0;
  while (done < n) {
    const std::uint64_t len = std::min(chunk, n - done);
    // Kernel and copy share the generator's stream, so the next chunk's kernel
    // cannot overwrite the staging buffer before this chunk's copy has read it.
    const cudaError_t e = q.launch(g.staging, len, g.seed, first + done / pb, g.stream);
    if (e != cudaSuccess) return CURAND_STATUS_LAUNCH_FAILURE;
    if (cudaMemcpyAsync(dst + done * eb, g.staging, len * eb, cudaMemcpyDeviceToHost, g.stream) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      return CURAND_STATUS_LAUNCH_FAILURE;
    }
    done += len;
  }
  if (cudaStreamSynchronize(g.stream) != cudaSuccess) {
    (void)cudaGetLastError();
    return CURAND_STATUS_LAUNCH_FAILURE;
  }
  g.offset += q.advance(n);
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t generate(curandGenerator_t gen, const Request& q, void* out, std::size_t num) {
  if (out == nullptr && num > 0) return CURAND_STATUS_INVALID_VALUE;
  if (num == 0) return CURAND_STATUS_SUCCESS;
  auto g = generators().get(gen);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  if (!mb200::aligned_to(out, q.elem_bytes())) return CURAND_STATUS_INVALID_VALUE;
  std::lock_guard<std::mutex> lock(g->mu);
  if (g->host_target) return host_fill(*g, q, out, num);
  // An array the GPU cannot address would fault the kernel; the reference
  // reports an unresolvable buffer as ALLOCATION_FAILED (curand_api.mm:198-200).
  if (!mb200::device_span_ok(out, static_cast<std::size_t>(num) * q.elem_bytes()))
    return CURAND_STATUS_ALLOCATION_FAILED;
  return device_fill(*g, q, out, num);
}

Request f32(Dist d, float mean = 0.0f, float stddev = 1.0f) {
  Request q;
  q.dist = d;
  q.mean = mean;
  q.stddev = stddev;
  return q;
}

Request f64(Dist d, double mean = 0.0, double stddev = 1.0) {
  Request q;
  q.kind = Request::kF64;
  q.dist = d;
  q.mean_d = mean;
  q.stddev_d = stddev;
  return q;
}

// Sobol direction numbers of the first dimension (v_k = 2^(31-k)) and the
// scramble constant, as the reference publishes them (curand_api.mm:26-35).
const curandDirectionVectors32_t kDirections32[1] = {
    {0x80000000u, 0x40000000u, 0x20000000u, 0x10000000u, 0x08000000u, 0x04000000u, 0x02000000u,
     0x01000000u, 0x00800000u, 0x00400000u, 0x00200000u, 0x00100000u, 0x00080000u, 0x00040000u,
     0x00020000u, 0x00010000u, 0x00008000u, 0x00004000u, 0x00002000u, 0x00001000u, 0x00000800u,
     0x00000400u, 0x00000200u, 0x00000100u, 0x00000080u, 0x00000040u, 0x00000020u, 0x00000010u,
     0x00000008u, 0x00000004u, 0x00000002u, 0x00000001u}};
const unsigned int kScramble32[1] = {0x6543210fu};

}  // namespace

extern "C" {

curandStatus_t curandCreateGenerator(curandGenerator_t* generator, curandRngType_t rng_type) {
  return create(generator, rng_type, false);
}

curandStatus_t curandCreateGeneratorHost(curandGenerator_t* generator, curandRngType_t rng_type) {
  return create(generator, rng_type, true);
}

curandStatus_t curandDestroyGenerator(curandGenerator_t generator) {
  return generators().take(generator) ? CURAND_STATUS_SUCCESS : CURAND_STATUS_NOT_INITIALIZED;
}

curandStatus_t curandSetStream(curandGenerator_t generator, cudaStream_t stream) {
  auto g = generators().get(generator);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> lock(g->mu);
  g->stream = stream;
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t curandGetStream(curandGenerator_t generator, cudaStream_t* stream) {
  if (stream == nullptr) return CURAND_STATUS_INVALID_VALUE;
  auto g = generators().get(generator);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> lock(g->mu);
  *stream = g->stream;
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t curandSetPseudoRandomGeneratorSeed(curandGenerator_t generator,
                                                  unsigned long long seed) {
  auto g = generators().get(generator);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> lock(g->mu);
  g->seed = seed;
  g->offset = 0;
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t curandSetGeneratorOffset(curandGenerator_t generator, unsigned long long offset) {
  auto g = generators().get(generator);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> lock(g->mu);
  g->offset = offset;
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t curandSetGeneratorOrdering(curandGenerator_t generator, curandOrdering_t order) {
  auto g = generators().get(generator);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> lock(g->mu);
  g->ordering = order;
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t curandGetVersion(int* version) {
  if (version == nullptr) return CURAND_STATUS_INVALID_VALUE;
  *version = kCurandVersion;
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t curandGetProperty(libraryPropertyType type, int* value) {
  if (value == nullptr) return CURAND_STATUS_INVALID_VALUE;
  switch (type) {
    case MAJOR_VERSION:
      *value = 10;
      return CURAND_STATUS_SUCCESS;
    case MINOR_VERSION:
      *value = 2;
      return CURAND_STATUS_SUCCESS;
    case PATCH_LEVEL:
      *value = 0;
      return CURAND_STATUS_SUCCESS;
  }
  return CURAND_STATUS_INVALID_VALUE;
}

curandStatus_t curandGenerate(curandGenerator_t generator, unsigned int* outputPtr, size_t num) {
  return generate(generator, f32(Dist::kUint32), outputPtr, num);
}

curandStatus_t curandGenerateUniform(curandGenerator_t generator, float* outputPtr, size_t num) {
  return generate(generator, f32(Dist::kUniform), outputPtr, num);
}

curandStatus_t curandGenerateNormal(curandGenerator_t generator, float* outputPtr, size_t n,
                                    float mean, float stddev) {
  return generate(generator, f32(Dist::kNormal, mean, stddev), outputPtr, n);
}

curandStatus_t curandGenerateLogNormal(curandGenerator_t generator, float* outputPtr, size_t n,
                                       float mean, float stddev) {
  return generate(generator, f32(Dist::kLogNormal, mean, stddev), outputPtr, n);
}

curandStatus_t curandGenerateUniformDouble(curandGenerator_t generator, double* outputPtr,
                                           size_t num) {
  return generate(generator, f64(Dist::kUniformDouble), outputPtr, num);
}

curandStatus_t curandGenerateNormalDouble(curandGenerator_t generator, double* outputPtr, size_t n,
                                          double mean, double stddev) {
  return generate(generator, f64(Dist::kNormalDouble, mean, stddev), outputPtr, n);
}

curandStatus_t curandGenerateLogNormalDouble(curandGenerator_t generator, double* outputPtr,
                                             size_t n, double mean, double stddev) {
  return generate(generator, f64(Dist::kLogNormalDouble, mean, stddev), outputPtr, n);
}

curandStatus_t curandGeneratePoisson(curandGenerator_t generator, unsigned int* outputPtr, size_t n,
                                     double lambda) {
  Request q;
  q.kind = Request::kPoisson;
  // the kernel computes in fp32 as the reference's does (curand_api.mm:466); the
  // threshold exp(-lambda) is rounded once from double on the host
  q.lambda = static_cast<float>(lambda);
  q.exp_neg_lambda = static_cast<float>(std::exp(-static_cast<double>(q.lambda)));
  return generate(generator, q, outputPtr, n);
}

curandStatus_t curandSetQuasiRandomGeneratorDimensions(curandGenerator_t generator,
                                                       unsigned int num_dimensions) {
  auto g = generators().get(generator);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  if (num_dimensions < 1 || num_dimensions > 20000) return CURAND_STATUS_OUT_OF_RANGE;
  std::lock_guard<std::mutex> lock(g->mu);
  g->dimensions = num_dimensions;
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t curandGetDirectionVectors32(curandDirectionVectors32_t* vectors[],
                                           curandDirectionVectorSet_t set) {
  if (vectors == nullptr) return CURAND_STATUS_INVALID_VALUE;
  if (set == CURAND_DIRECTION_VECTORS_32_JOEKUO6 ||
      set == CURAND_SCRAMBLED_DIRECTION_VECTORS_32_JOEKUO6) {
    *vectors = const_cast<curandDirectionVectors32_t*>(kDirections32);
    return CURAND_STATUS_SUCCESS;
  }
  return CURAND_STATUS_OUT_OF_RANGE;
}

curandStatus_t curandGetScrambleConstants32(const unsigned int** constants) {
  if (constants == nullptr) return CURAND_STATUS_INVALID_VALUE;
  *constants = kScramble32;
  return CURAND_STATUS_SUCCESS;
}

}  // extern "C"
