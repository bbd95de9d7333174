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

// Launches one device fill and advances the offset; caller holds g.mu.
curandStatus_t device_fill(Generator& g, Dist dist, void* out, std::uint64_t n, float mean,
                           float stddev) {
  const cudaError_t e = mb200::rand::launch_philox_fill(dist, out, n, g.seed, g.offset >> 2, mean,
                                                        stddev, g.stream);
  if (e != cudaSuccess) return CURAND_STATUS_LAUNCH_FAILURE;
  g.offset += 4 * ((n + 3) / 4);
  return CURAND_STATUS_SUCCESS;
}

// Host generator: chunks of kStagingWords (a multiple of 4, so each chunk starts
// on a Philox block boundary and the chunked stream equals the one-shot stream).
curandStatus_t host_fill(Generator& g, Dist dist, void* out, std::uint64_t n, float mean,
                         float stddev) {
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
  auto* dst = static_cast<unsigned char*>(out);
  std::uint64_t done = 0;
  while (done < n) {
    const std::uint64_t len = std::min(kStagingWords, n - done);
    // Kernel and copy share the generator's stream, so the next chunk's kernel
    // cannot overwrite the staging buffer before this chunk's copy has read it.
    const cudaError_t e = mb200::rand::launch_philox_fill(
        dist, g.staging, len, g.seed, (g.offset >> 2) + done / 4, mean, stddev, g.stream);
    if (e != cudaSuccess) return CURAND_STATUS_LAUNCH_FAILURE;
    if (cudaMemcpyAsync(dst + done * 4, g.staging, len * 4, cudaMemcpyDeviceToHost, g.stream) !=
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
  g.offset += 4 * ((n + 3) / 4);
  return CURAND_STATUS_SUCCESS;
}

curandStatus_t generate(curandGenerator_t gen, Dist dist, void* out, std::size_t num, float mean,
                        float stddev) {
  if (out == nullptr && num > 0) return CURAND_STATUS_INVALID_VALUE;
  if (num == 0) return CURAND_STATUS_SUCCESS;
  auto g = generators().get(gen);
  if (!g) return CURAND_STATUS_NOT_INITIALIZED;
  if (!mb200::aligned_to(out, 4)) return CURAND_STATUS_INVALID_VALUE;
  std::lock_guard<std::mutex> lock(g->mu);
  if (g->host_target) return host_fill(*g, dist, out, num, mean, stddev);
  // An array the GPU cannot address would fault the kernel; the reference
  // reports an unresolvable buffer as ALLOCATION_FAILED (curand_api.mm:198-200).
  if (!mb200::device_span_ok(out, static_cast<std::size_t>(num) * 4))
    return CURAND_STATUS_ALLOCATION_FAILED;
  return device_fill(*g, dist, out, num, mean, stddev);
}

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
  return generate(generator, Dist::kUint32, outputPtr, num, 0.0f, 1.0f);
}

curandStatus_t curandGenerateUniform(curandGenerator_t generator, float* outputPtr, size_t num) {
  return generate(generator, Dist::kUniform, outputPtr, num, 0.0f, 1.0f);
}

curandStatus_t curandGenerateNormal(curandGenerator_t generator, float* outputPtr, size_t n,
                                    float mean, float stddev) {
  return generate(generator, Dist::kNormal, outputPtr, n, mean, stddev);
}

}  // extern "C"
