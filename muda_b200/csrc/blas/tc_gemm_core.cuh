// tc_gemm_core.cuh — persistent warp-specialized tcgen05 main loop shared by the
// bf16/fp16 GEMM and the NHWC implicit-GEMM convolution.
//
// One CTA per SM walks output tiles of 128 x BN (fp32 accumulators in tensor
// memory) with a K loop of blocks of one 128-byte row per operand row (64 16-bit
// or 32 fp32 elements):
//   warp 0     one thread issues the TMA loads of each k-block (A: 128 rows x 128 B,
//              B: BN rows x 128 B per plane, 128-byte swizzle) into a STAGES-deep ring;
//   warp 1     allocates 2*BN tensor-memory columns; one thread issues the MMAs of
//              each k-block (four 32-byte K steps) and commits each stage back to the
//              producer and each finished tile to the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of their 32-lane quarter, 32 columns at a time,
//              handed to the problem's store(); the second accumulator lets the
//              next tile's MMAs overlap this tile's epilogue.
//
// Operand formats (FMT): 0 fp16 and 1 bf16 run one kind::f16 MMA (M128 N=BN K16)
// per K step.  2 is split tf32 for fp32 data (tc_gemm_split_kernel below): each
// operand arrives as two planes,
// hi = x truncated to tf32 and lo = (x - hi) rounded to tf32 (tf32_split.hpp),
// stored one after the other in the stage (hi first), and each K step issues three
// kind::tf32 MMAs (M128 N=BN K8) accumulating lo*hi + hi*lo + hi*hi into the same
// fp32 tile.  The dropped lo*lo term and the rounding of lo leave a relative error
// below 1.5 * 2^-20 per product, the accuracy class of an fp32 FMA loop.
//
// The problem type P supplies the geometry (a __grid_constant__ kernel parameter,
// so its CUtensorMap members live in parameter space as TMA requires):
//   long long tiles_total;  int num_kb;
//   void prefetch() const;                                  // tensor-map prefetch
//   void coords(long long t, int (&c)[3]) const;            // tile index -> coordinates
//   void load(const int (&c)[3], int kb, void* sa, void* sb, uint64_t* bar) const;
//   void scalars(float& alpha, float& beta) const;
//   void store(const int (&c)[3], int row, int col0, const float (&v)[32], float alpha,
//              float beta) const;                           // row in [0,128), 32 columns
//
// Operands are K-major by default.  A problem may declare `static constexpr bool
// kAMn, kBMn`: an MN-major operand arrives as 64 x 64 boxes (64 M or N elements of
// 128 bytes per K row, 8 KB per box, boxes along M/N every 8 KB), which the MMA
// reads through MN-major descriptors (tc_ptx.cuh), each 16-element K step 16 rows
// (2048 bytes) further on.  Only the 16-bit kernel (FMT 0 / 1) accepts them.
//
// Every mbarrier wait is bounded (tc_ptx.cuh).  A wait that runs out marks the CTA
// aborted, counts the event in the problem's timeout counter, drains the copies and
// MMAs the CTA issued (bounded), frees its tensor memory and returns.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <type_traits>

#include "blas/tc_ptx.cuh"

namespace mb200::tc {

constexpr int kBM = 128;
constexpr int kBK = 64;        // 16-bit elements per k-block: one 128-byte swizzle row
constexpr int kBK32 = 32;      // fp32 elements per k-block
constexpr int kRowBytes = 128;
constexpr int kStepBytes = 32;  // K bytes consumed by one MMA (16 x 16-bit, 8 x tf32)
constexpr int kAcc = 2;
constexpr int kThreads = 192;
constexpr int kFmtTf32x3 = 2;

// Operand majorness of a problem type (see above): K-major unless it says otherwise.
template <class P, class = void>
struct OperandMajor {
  static constexpr bool a_mn = false, b_mn = false;
};
template <class P>
struct OperandMajor<P, std::void_t<decltype(P::kAMn), decltype(P::kBMn)>> {
  static constexpr bool a_mn = P::kAMn, b_mn = P::kBMn;
};

constexpr std::uint32_t kMnBoxBytes = 64 * kRowBytes;   // one 64 x 64 box of 16-bit elements
constexpr std::uint32_t kMnStepBytes = 16 * kRowBytes;  // 16 K rows per MMA K step

// Descriptor of K step k (16 elements) of an operand tile at shared address `base`.
template <bool MN>
__device__ __forceinline__ std::uint64_t operand_desc(std::uint32_t base, int k) {
  if constexpr (MN)
    return mnmajor_sw128_desc(base + static_cast<std::uint32_t>(k) * kMnStepBytes, kMnBoxBytes);
  else
    return kmajor_sw128_desc(base + static_cast<std::uint32_t>(k * kStepBytes));
}

template <int BN, int STAGES, int PLANES = 1>
struct CoreShape {
  static constexpr int A_PLANE = kBM * kRowBytes;
  static constexpr int B_PLANE = BN * kRowBytes;
  static constexpr int A_STAGE = PLANES * A_PLANE;
  static constexpr int B_STAGE = PLANES * B_PLANE;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * (A_STAGE + B_STAGE) + BAR_BYTES + 1024;
  static constexpr std::uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
};

template <class P, int BN, int STAGES, int FMT>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(const __grid_constant__ P p,
                                                              unsigned int* timeouts) {
  static_assert(FMT == 0 || FMT == 1, "16-bit operand kinds; split tf32 has its own kernel");
  using S = CoreShape<BN, STAGES, 1>;
  extern __shared__ std::uint8_t smem_raw[];
  std::uint8_t* base = reinterpret_cast<std::uint8_t*>(
      (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t{1023});
  std::uint8_t* sa = base;
  std::uint8_t* sb = base + STAGES * S::A_STAGE;
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(sb + STAGES * S::B_STAGE);
  std::uint64_t* empty = full + STAGES;
  std::uint64_t* acc_full = empty + STAGES;
  std::uint64_t* acc_empty = acc_full + kAcc;
  std::uint64_t* mma_done = acc_empty + kAcc;
  std::uint32_t* tmem_slot = reinterpret_cast<std::uint32_t*>(mma_done + 1);
  volatile int* aborted = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    *aborted = 0;
    mbar_fence_init();
    p.prefetch();
  }
  if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const std::uint32_t tmem_base = *tmem_slot;
  const int num_kb = p.num_kb;
  auto fail = [&]() {
    *aborted = 1;
    atomicAdd(timeouts, 1u);
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      std::uint32_t phase = 0;
      std::uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false;
      for (long long t = blockIdx.x; t < p.tiles_total && !*aborted; t += gridDim.x) {
        int c[3];
        p.coords(t, c);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            fail();
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::A_STAGE + S::B_STAGE);
          p.load(c, kb, sa + stage * S::A_STAGE, sb + stage * S::B_STAGE, &full[stage]);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every issued copy has landed before the CTA may retire.
      for (int s = 0; s < STAGES; ++s)
        if (issued[s] && !mbar_wait(&full[s], issued_phase[s])) fail();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr bool AMN = OperandMajor<P>::a_mn, BMN = OperandMajor<P>::b_mn;
      constexpr std::uint32_t idesc = f16_idesc(FMT, kBM, BN, AMN, BMN);
      int stage = 0;
      std::uint32_t phase = 0;
      int acc = 0;
      std::uint32_t acc_phase = 0;
      for (long long t = blockIdx.x; t < p.tiles_total && !*aborted; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u)) {
          fail();
          break;
        }
        tc_fence_after();
        const std::uint32_t d_tmem = tmem_base + static_cast<std::uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          const std::uint32_t a0 = smem_addr(sa + stage * S::A_STAGE);
          const std::uint32_t b0 = smem_addr(sb + stage * S::B_STAGE);
#pragma unroll
          for (int k = 0; k < kRowBytes / kStepBytes; ++k)
            mma_f16(d_tmem, operand_desc<AMN>(a0, k), operand_desc<BMN>(b0, k), idesc,
                    (kb | k) != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
        if (++acc == kAcc) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: all issued MMAs have completed before tensor memory is freed.
      mma_commit(mma_done);
      if (!mbar_wait(mma_done, 0)) fail();
    }
  } else {
    // ---------------- epilogue (warps 2..5, one 32-lane quarter each)
    const int quarter = warp & 3;
    float alpha, beta;
    p.scalars(alpha, beta);
    int acc = 0;
    std::uint32_t acc_phase = 0;
    for (long long t = blockIdx.x; t < p.tiles_total && !*aborted; t += gridDim.x) {
      int c[3];
      p.coords(t, c);
      if (!mbar_wait(&acc_full[acc], acc_phase)) {
        fail();
        break;
      }
      tc_fence_after();
      const int row = quarter * 32 + lane;
      const std::uint32_t t_row = tmem_base + (static_cast<std::uint32_t>(quarter * 32) << 16) +
                                  static_cast<std::uint32_t>(acc * BN);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_load_32cols(t_row + static_cast<std::uint32_t>(c0), v);
        p.store(c, row, c0, v, alpha, beta);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == kAcc) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Split-tf32 kernel (FMT 2): fp32 accuracy on the tensor cores.
//
// The tensor core's fp32 accumulation truncates: measured on B200, each MMA that
// adds into an accumulator loses about 0.44 ulp toward zero, so one chain of K/8 * 3
// MMAs drifts by roughly 2e-8 * K relative (8e-5 at K = 4096, against 8e-7 for an
// FFMA loop).  Here every chunk of CK k-blocks (CK * 12 MMAs) starts a fresh
// accumulator, and the epilogue adds each finished chunk into a running fp32 sum
// held in registers with round-to-nearest adds, which keeps the error at the FFMA
// loop's level.  Eight epilogue warps each own one 32-lane quarter and one
// 128-column half of the 128 x 256 tile (128 running sums per thread); two chunk
// accumulators alternate so the MMA issuer does not wait for the epilogue.
constexpr int kSplitThreads = 320;  // producer, MMA issuer, 8 epilogue warps
constexpr int kSplitEpiWarps = 8;

template <class P, int BN, int STAGES, int CK>
__global__ void __launch_bounds__(kSplitThreads, 1)
    tc_gemm_split_kernel(const __grid_constant__ P p, unsigned int* timeouts) {
  static_assert(BN == 256 || BN == 128 || BN == 64,
                "the epilogue splits the tile into two halves of 32-column groups");
  static_assert(!OperandMajor<P>::a_mn && !OperandMajor<P>::b_mn,
                "split tf32 reads K-major planes only");
  constexpr int HC = BN / 2;  // columns per epilogue warp
  using S = CoreShape<BN, STAGES, 2>;
  extern __shared__ std::uint8_t smem_raw[];
  std::uint8_t* base = reinterpret_cast<std::uint8_t*>(
      (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t{1023});
  std::uint8_t* sa = base;
  std::uint8_t* sb = base + STAGES * S::A_STAGE;
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(sb + STAGES * S::B_STAGE);
  std::uint64_t* empty = full + STAGES;
  std::uint64_t* acc_full = empty + STAGES;
  std::uint64_t* acc_empty = acc_full + kAcc;
  std::uint64_t* mma_done = acc_empty + kAcc;
  std::uint32_t* tmem_slot = reinterpret_cast<std::uint32_t*>(mma_done + 1);
  volatile int* aborted = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kSplitEpiWarps);
    }
    mbar_init(mma_done, 1);
    *aborted = 0;
    mbar_fence_init();
    p.prefetch();
  }
  if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const std::uint32_t tmem_base = *tmem_slot;
  const int num_kb = p.num_kb;
  auto fail = [&]() {
    *aborted = 1;
    atomicAdd(timeouts, 1u);
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both planes of A and B per stage)
      int stage = 0;
      std::uint32_t phase = 0;
      std::uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false;
      for (long long t = blockIdx.x; t < p.tiles_total && !*aborted; t += gridDim.x) {
        int c[3];
        p.coords(t, c);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            fail();
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::A_STAGE + S::B_STAGE);
          p.load(c, kb, sa + stage * S::A_STAGE, sb + stage * S::B_STAGE, &full[stage]);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (issued[s] && !mbar_wait(&full[s], issued_phase[s])) fail();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: one fresh accumulator per chunk of CK k-blocks
      constexpr std::uint32_t idesc = f16_idesc(kFmtTf32x3, kBM, BN);
      int stage = 0;
      std::uint32_t phase = 0;
      int acc = 0;
      std::uint32_t acc_phase = 0;
      bool ok = true;
      for (long long t = blockIdx.x; ok && t < p.tiles_total && !*aborted; t += gridDim.x) {
        for (int kb = 0; kb < num_kb; ++kb) {
          const bool first = kb % CK == 0;
          const bool last = kb % CK == CK - 1 || kb == num_kb - 1;
          if (first) {
            if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u)) {
              fail();
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (!mbar_wait(&full[stage], phase)) {
            fail();
            ok = false;
            break;
          }
          tc_fence_after();
          const std::uint32_t d_tmem = tmem_base + static_cast<std::uint32_t>(acc * BN);
          const std::uint32_t a0 = smem_addr(sa + stage * S::A_STAGE);
          const std::uint32_t b0 = smem_addr(sb + stage * S::B_STAGE);
#pragma unroll
          for (int k = 0; k < kRowBytes / kStepBytes; ++k) {
            const std::uint32_t ak = a0 + k * kStepBytes, bk = b0 + k * kStepBytes;
            // lo*hi, hi*lo, then hi*hi (planes: hi at offset 0, lo one plane on)
            mma_tf32(d_tmem, kmajor_sw128_desc(ak + S::A_PLANE), kmajor_sw128_desc(bk), idesc,
                     (first && k == 0) ? 0u : 1u);
            mma_tf32(d_tmem, kmajor_sw128_desc(ak), kmajor_sw128_desc(bk + S::B_PLANE), idesc, 1u);
            mma_tf32(d_tmem, kmajor_sw128_desc(ak), kmajor_sw128_desc(bk), idesc, 1u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (last) {
            mma_commit(&acc_full[acc]);
            if (++acc == kAcc) {
              acc = 0;
              acc_phase ^= 1u;
            }
          }
        }
      }
      mma_commit(mma_done);
      if (!mbar_wait(mma_done, 0)) fail();
    }
  } else {
    // ---------------- epilogue (warps 2..9): quarter = warp % 4, half = (warp - 2) / 4
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const std::uint32_t t_lane = tmem_base + (static_cast<std::uint32_t>(quarter * 32) << 16) +
                                 static_cast<std::uint32_t>(half * HC);
    const int chunks = (num_kb + CK - 1) / CK;
    float alpha, beta;
    p.scalars(alpha, beta);
    int acc = 0;
    std::uint32_t acc_phase = 0;
    bool ok = true;
    for (long long t = blockIdx.x; ok && t < p.tiles_total && !*aborted; t += gridDim.x) {
      int c[3];
      p.coords(t, c);
      float run[HC];
#pragma unroll
      for (int j = 0; j < HC; ++j) run[j] = 0.0f;
      for (int ch = 0; ch < chunks; ++ch) {
        if (!mbar_wait(&acc_full[acc], acc_phase)) {
          fail();
          ok = false;
          break;
        }
        tc_fence_after();
        const std::uint32_t ta = t_lane + static_cast<std::uint32_t>(acc * BN);
#pragma unroll
        for (int g = 0; g < HC / 16; ++g) {
          float v[16];
          tmem_load_16cols(ta + static_cast<std::uint32_t>(g * 16), v);
#pragma unroll
          for (int j = 0; j < 16; ++j) run[g * 16 + j] = __fadd_rn(run[g * 16 + j], v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        if (++acc == kAcc) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) break;
#pragma unroll
      for (int g = 0; g < HC / 32; ++g)
        p.store(c, row, half * HC + g * 32, *reinterpret_cast<const float(*)[32]>(run + g * 32),
                alpha, beta);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

// k-blocks per accumulator chunk of the split-tf32 kernel: 2 x 4 K steps x 3 MMAs =
// 24 truncating accumulations (about 1e-6 relative drift) per chunk.
constexpr int kSplitChunkKb = 2;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) !=
            cudaSuccess ||
        r != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(q);
  }();
  return fn;
}

// Tiled map over a tensor of `rank` dims (innermost first, strides in bytes for
// dims 1..rank-1) of fp16 (fmt 0), bf16 (1) or fp32 (2) elements, box `box`,
// 128-byte swizzle, zero fill out of bounds.
inline bool encode_tiled(CUtensorMap* map, int fmt, const void* base, int rank,
                         const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                         const cuuint32_t* box) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
  const CUtensorMapDataType dt = fmt == 2   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : fmt == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, dt,
            static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims, strides_bytes, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

using EncodeIm2colFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const int*, const int*,
                                    cuuint32_t, cuuint32_t, const cuuint32_t*,
                                    CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeIm2colFn encode_im2col_fn() {
  static EncodeIm2colFn fn = [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &q, cudaEnableDefault, &r) !=
            cudaSuccess ||
        r != cudaDriverEntryPointSuccess)
      return static_cast<EncodeIm2colFn>(nullptr);
    return reinterpret_cast<EncodeIm2colFn>(q);
  }();
  return fn;
}

// im2col map over a (c, w, h, [d,] n) tensor of `rank` dims: the box is
// `pixels` base pixels x `channels` channels, the spatial bounding box of the base
// pixels runs from `lower` to dim - 1 + `upper` in each of the rank - 2 spatial
// dimensions (w first), traversal stride 1, 128-byte swizzle, zero fill.
inline bool encode_im2col(CUtensorMap* map, int fmt, const void* base, int rank,
                          const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                          const int* lower, const int* upper, cuuint32_t channels,
                          cuuint32_t pixels) {
  EncodeIm2colFn fn = encode_im2col_fn();
  if (fn == nullptr) return false;
  const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
  const CUtensorMapDataType dt = fmt == 2   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : fmt == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims,
            strides_bytes, lower, upper, channels, pixels, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <class P, int BN, int STAGES, int FMT>
cudaError_t launch_tc_gemm(const P& p, int sms, unsigned int* timeouts, cudaStream_t stream) {
  constexpr bool split = FMT == kFmtTf32x3;
  using S = CoreShape<BN, STAGES, split ? 2 : 1>;
  void (*kern)(P, unsigned int*);
  if constexpr (split)
    kern = tc_gemm_split_kernel<P, BN, STAGES, kSplitChunkKb>;
  else
    kern = tc_gemm_kernel<P, BN, STAGES, FMT>;
  // the shared-memory opt-in is per device and per kernel: set it once
  static std::atomic<unsigned long long> attr_set{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  const unsigned long long bit = 1ull << (dev & 63);
  if ((attr_set.load(std::memory_order_acquire) & bit) == 0) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit, std::memory_order_release);
  }
  const long long grid = p.tiles_total < sms ? p.tiles_total : sms;
  if (grid <= 0) return cudaSuccess;
  kern<<<static_cast<unsigned>(grid), split ? kSplitThreads : kThreads, S::SMEM, stream>>>(
      p, timeouts);
  return cudaGetLastError();
}

}  // namespace mb200::tc
