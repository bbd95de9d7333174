// tc_ptx.cuh — thin wrappers over the sm_100a PTX used by the tensor-core kernels:
// mbarriers, TMA tensor loads (no multicast), tensor-memory allocation, tcgen05 MMA,
// commit and tensor-memory loads.  Every wait is bounded: it gives up after
// kWaitLimitNs of wall time and reports failure instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mb200::tc {

// A wait gives up after this much wall time (global timer, nanoseconds): far
// beyond any legitimate wait inside one CTA (microseconds), short enough to end
// a stuck kernel instead of holding the GPU.
constexpr std::uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ std::uint64_t global_ns() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ std::uint32_t smem_addr(const void* p) {
  return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(std::uint64_t* bar, std::uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(std::uint64_t* bar, std::uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(std::uint64_t* bar, std::uint32_t parity) {
  std::uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits until the phase with the given parity has completed; false on timeout.
__device__ __forceinline__ bool mbar_wait(std::uint64_t* bar, std::uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const std::uint64_t t0 = global_ns();
  for (std::uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u && global_ns() - t0 > kWaitLimitNs) return false;
  }
}

// 3-D tiled TMA load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, std::int32_t x,
                                            std::int32_t y, std::int32_t z, std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// 4-D tiled TMA load (e.g. an NHWC activation rectangle); coordinates outside the
// tensor read as zero.  The innermost coordinate must be 16-byte aligned.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, std::int32_t x,
                                            std::int32_t y, std::int32_t z, std::int32_t w,
                                            std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w),
      "r"(smem_addr(bar))
      : "memory");
}

// 5-D tiled TMA load (e.g. the hi/lo planes of an NHWC activation rectangle).
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, std::int32_t x,
                                            std::int32_t y, std::int32_t z, std::int32_t w,
                                            std::int32_t v, std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v),
      "r"(smem_addr(bar))
      : "memory");
}

// im2col TMA loads: the box is `pixels per column` consecutive base pixels of an
// NHWC (or NHWC-plus-plane) tensor, walked w fastest inside the tensor map's
// bounding box, then h, then the outer dimensions; each pixel contributes the
// map's channels-per-pixel channels read at (w + off_w, h + off_h), zero outside
// the tensor.  (c, w, h, ...) is the first base pixel; c must be 16-byte aligned.
__device__ __forceinline__ void tma_load_im2col_4d(void* dst, const CUtensorMap* map,
                                                   std::int32_t c, std::int32_t w, std::int32_t h,
                                                   std::int32_t n, std::uint16_t off_w,
                                                   std::uint16_t off_h, std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n),
      "r"(smem_addr(bar)), "h"(off_w), "h"(off_h)
      : "memory");
}

__device__ __forceinline__ void tma_load_im2col_5d(void* dst, const CUtensorMap* map,
                                                   std::int32_t c, std::int32_t w, std::int32_t h,
                                                   std::int32_t d, std::int32_t n,
                                                   std::uint16_t off_w, std::uint16_t off_h,
                                                   std::uint16_t off_d, std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], {%8, %9, %10};" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(d), "r"(n),
      "r"(smem_addr(bar)), "h"(off_w), "h"(off_h), "h"(off_d)
      : "memory");
}

// Untiled bulk copies (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src, std::uint32_t bytes,
                                          std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst_smem)),
      "l"(reinterpret_cast<std::uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_store(void* dst, const void* src_smem, std::uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<std::uint64_t>(dst)),
               "r"(smem_addr(src_smem)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Shared-memory source of every committed bulk store has been read.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Every committed bulk store but the most recent one has read its shared-memory source.
__device__ __forceinline__ void bulk_wait_read_but_one() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's generic shared-memory writes before later async-proxy
// (bulk copy) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<std::uint64_t>(map)) : "memory");
}

// Tensor memory allocation: executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(std::uint32_t* dst_smem, std::uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(std::uint32_t taddr, std::uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, one kind::f16 MMA issued by the calling thread.
__device__ __forceinline__ void mma_f16(std::uint32_t d_tmem, std::uint64_t adesc,
                                        std::uint64_t bdesc, std::uint32_t idesc,
                                        std::uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T with tf32 operands (fp32 words whose low 13
// mantissa bits are zero), one kind::tf32 MMA: K = 8 elements = 32 bytes per row.
__device__ __forceinline__ void mma_tf32(std::uint32_t d_tmem, std::uint64_t adesc,
                                         std::uint64_t bdesc, std::uint32_t idesc,
                                         std::uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(std::uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// 32 consecutive fp32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_load_32cols(std::uint32_t taddr, float* v) {
  std::uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_load_16cols(std::uint32_t taddr, float* v) {
  std::uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile stored as rows of
// 128 bytes with the 128-byte swizzle (8-row atoms of 1024 bytes, stacked along
// M/N): start address, leading offset 16 B (unused by this layout), stride
// offset 1024 B between 8-row groups, descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ std::uint64_t kmajor_sw128_desc(std::uint32_t saddr) {
  std::uint64_t d = 0;
  d |= static_cast<std::uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<std::uint64_t>(1u) << 16;            // leading byte offset (16 B units)
  d |= static_cast<std::uint64_t>(1024u >> 4) << 32;    // stride byte offset (16 B units)
  d |= static_cast<std::uint64_t>(1u) << 46;            // descriptor version
  d |= static_cast<std::uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor for an MN-major operand tile stored as the
// 128-byte-swizzle MN-major atoms a 64 x 64 TMA box of 16-bit elements produces:
// each K index is one 128-byte row of 64 consecutive M (or N) elements, 8 rows
// form a 1024-byte atom, atoms follow each other along K every 1024 bytes (stride
// byte offset) and 64-element column blocks along M/N every `mn_block_bytes`
// (leading byte offset), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ std::uint64_t mnmajor_sw128_desc(std::uint32_t saddr,
                                                            std::uint32_t mn_block_bytes) {
  std::uint64_t d = 0;
  d |= static_cast<std::uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<std::uint64_t>((mn_block_bytes >> 4) & 0x3FFFu) << 16;  // leading offset
  d |= static_cast<std::uint64_t>(1024u >> 4) << 32;                        // stride offset
  d |= static_cast<std::uint64_t>(1u) << 46;
  d |= static_cast<std::uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor of kind::f16 / kind::tf32: fp32 accumulate, A/B of the
// given format (0 = fp16, 1 = bf16, 2 = tf32), tile M x N; a_mn / b_mn mark an
// MN-major operand (bits 15 / 16; otherwise K-major).
__host__ __device__ constexpr std::uint32_t f16_idesc(int ab_format, int m, int n,
                                                      bool a_mn = false, bool b_mn = false) {
  return (1u << 4) | (static_cast<std::uint32_t>(ab_format) << 7) |
         (static_cast<std::uint32_t>(ab_format) << 10) |
         (static_cast<std::uint32_t>(a_mn ? 1u : 0u) << 15) |
         (static_cast<std::uint32_t>(b_mn ? 1u : 0u) << 16) |
         (static_cast<std::uint32_t>(n >> 3) << 17) | (static_cast<std::uint32_t>(m >> 4) << 24);
}

}  // namespace mb200::tc
