/*
 * oracle.h — CPU restatements of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  The product (muda_b200/, include/) never links,
 * loads or calls anything here.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use this library, and only as
 * the checker or the timed CPU baseline.
 *
 * Each function names the reference file:line it restates.  The reference
 * (AshitomW/MUDA) is Objective-C++ plus Metal and builds only on macOS
 * (CMakeLists.txt:14-15), so it cannot be compiled or run here; these oracles are
 * pinned instead against every known-answer test the reference's own test suite
 * holds for the path (tests/curand_test.cpp, cublas_test.cpp, cufft_test.cpp,
 * cusparse_test.cpp, cudnn_test.cpp), restated in tests/test_oracle_pins.py.
 *
 * Built with -ffp-contract=off so that every float operation rounds separately,
 * as written in the restated source.
 */
#ifndef MUDA_B200_ORACLE_H_
#define MUDA_B200_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Philox4x32-10 (libraries/rand/src/curand_context.mm:42-185) ---- */
void oracle_philox_block(uint64_t ctr, uint64_t seed, uint32_t out[4]);
/* Writes n words of the stream that starts at generator offset `offset`;
 * returns the generator offset after the call (offset + 4*ceil(n/4)). */
uint64_t oracle_generate_uint(uint64_t seed, uint64_t offset, uint32_t* out, size_t n,
                              int threads);
uint64_t oracle_generate_uniform(uint64_t seed, uint64_t offset, float* out, size_t n,
                                 int threads);
uint64_t oracle_generate_normal(uint64_t seed, uint64_t offset, float* out, size_t n, float mean,
                                float stddev, int threads);
/* Blocks at arbitrary counters: out[4i..4i+3] = Philox(ctrs[i], seed). */
void oracle_philox_gather(const uint64_t* ctrs, size_t m, uint64_t seed, uint32_t* out,
                          int threads);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_ORACLE_H_ */
