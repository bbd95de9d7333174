// shim.cpp — C entry points over the reference's own host generator.
//
// TEST INFRASTRUCTURE ONLY.  Linked by oracle/ref/build.py together with the
// reference's unmodified libraries/rand/src/curand_context.mm (compiled as C++,
// its two framework imports served by the compile-only headers in stubs/) into
// oracle/_ref/libcurand_ref.so.  Tests call these functions to pin both the
// oracle restatement (oracle/philox.cpp) and the GPU kernels to the reference's
// real code: PhiloxHostStep (curand_context.mm:42-73) and the GenerateHost*
// bodies (curand_context.mm:75-293) run exactly as the reference ships them.
//
// Each call builds a fresh CurandContext (curand_context.hpp:26-35) with the
// given seed and offset, so the reference's own offset rule (offset >> 2 for
// 4-word streams, >> 1 for 2-word streams, += n for Poisson) picks the blocks.
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

#include "curand_context.hpp"

namespace R = muda::libraries::rand;

namespace {

enum Kind : int {
  kUint = 0,
  kUniform = 1,
  kNormal = 2,
  kLogNormal = 3,
  kUniformDouble = 4,
  kNormalDouble = 5,
  kLogNormalDouble = 6,
  kPoisson = 7,
};

int generate(int kind, R::CurandContext& ctx, void* out, std::size_t n, double mean,
             double stddev, double lambda) {
  switch (kind) {
    case kUint:
      return R::GenerateHostUint(ctx, static_cast<unsigned int*>(out), n);
    case kUniform:
      return R::GenerateHostUniform(ctx, static_cast<float*>(out), n);
    case kNormal:
      return R::GenerateHostNormal(ctx, static_cast<float*>(out), n, static_cast<float>(mean),
                                   static_cast<float>(stddev));
    case kLogNormal:
      return R::GenerateHostLogNormal(ctx, static_cast<float*>(out), n,
                                      static_cast<float>(mean), static_cast<float>(stddev));
    case kUniformDouble:
      return R::GenerateHostUniformDouble(ctx, static_cast<double*>(out), n);
    case kNormalDouble:
      return R::GenerateHostNormalDouble(ctx, static_cast<double*>(out), n, mean, stddev);
    case kLogNormalDouble:
      return R::GenerateHostLogNormalDouble(ctx, static_cast<double*>(out), n, mean, stddev);
    case kPoisson:
      return R::GenerateHostPoisson(ctx, static_cast<unsigned int*>(out), n, lambda);
    default:
      return -1;
  }
}

std::size_t elem_size(int kind) {
  return kind >= kUniformDouble && kind <= kLogNormalDouble ? sizeof(double) : 4u;
}

}  // namespace

extern "C" {

// PhiloxHostStep(ctr_idx, seed, out).
void ref_philox_step(std::uint64_t ctr_idx, std::uint64_t seed, std::uint32_t out[4]) {
  R::PhiloxHostStep(ctr_idx, seed, out);
}

// One GenerateHost* call on a generator at (seed, offset).  Returns the status;
// *offset_out receives the generator offset after the call.
int ref_generate(int kind, std::uint64_t seed, std::uint64_t offset, void* out, std::size_t n,
                 double mean, double stddev, double lambda, std::uint64_t* offset_out) {
  R::CurandContext ctx;
  ctx.seed = seed;
  ctx.offset = offset;
  const int st = generate(kind, ctx, out, n, mean, stddev, lambda);
  if (offset_out != nullptr) *offset_out = ctx.offset;
  return st;
}

// m independent calls of `words` outputs each, call i on a generator at
// (seed, offsets[i]), written to out + i * words elements: sampled checks of a
// long stream without generating all of it.
int ref_generate_at(int kind, std::uint64_t seed, const std::uint64_t* offsets, std::size_t m,
                    std::size_t words, void* out, double mean, double stddev) {
  auto* base = static_cast<unsigned char*>(out);
  for (std::size_t i = 0; i < m; ++i) {
    R::CurandContext ctx;
    ctx.seed = seed;
    ctx.offset = offsets[i];
    const int st = generate(kind, ctx, base + i * words * elem_size(kind), words, mean, stddev, 0.0);
    if (st != 0) return st;
  }
  return 0;
}

// One logical call of n outputs from (seed, offset), split over `threads` host
// threads: thread t runs the reference's GenerateHost* on its own generator whose
// offset starts its slice.  Slices are whole Philox blocks (4 words; 2 for the
// double streams), and block i of the call is counter i + (offset >> 2) (>> 1)
// whichever thread computes it, so the output equals one single-threaded call bit
// for bit.  offset must be a multiple of the block size for that to hold (the
// benchmark's offsets are).  Returns the offset after the call.
std::uint64_t ref_generate_parallel(int kind, std::uint64_t seed, std::uint64_t offset, void* out,
                                    std::size_t n, double mean, double stddev, int threads) {
  const std::size_t per_block = kind >= kUniformDouble && kind <= kLogNormalDouble ? 2u : 4u;
  const std::size_t blocks = (n + per_block - 1) / per_block;
  if (threads < 1) threads = 1;
  std::vector<std::thread> pool;
  auto* base = static_cast<unsigned char*>(out);
  for (int t = 0; t < threads; ++t) {
    const std::size_t b0 = blocks * t / threads, b1 = blocks * (t + 1) / threads;
    if (b1 <= b0) continue;
    const std::size_t w0 = b0 * per_block;
    const std::size_t w1 = b1 * per_block < n ? b1 * per_block : n;
    pool.emplace_back([=] {
      R::CurandContext ctx;
      ctx.seed = seed;
      ctx.offset = offset + w0;
      generate(kind, ctx, base + w0 * elem_size(kind), w1 - w0, mean, stddev, 0.0);
    });
  }
  for (auto& th : pool) th.join();
  return offset + blocks * per_block;
}

}  // extern "C"
