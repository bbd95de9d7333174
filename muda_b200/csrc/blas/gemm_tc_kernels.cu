// gemm_tc_kernels.cu — tcgen05 tensor-core GEMM for bf16 / fp16 operands (sm_100a).
//
// Semantics are those of the reference's 16-bit GEMM (libraries/blas/shaders/
// cublas_kernels.metal:1008-1045): fp32 accumulation of op(A)*op(B), then
// C = alpha*acc + beta*C (beta == 0: C not read), rounded to the 16-bit type.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0     TMA producer: 128x64 A and 256x64 B boxes (128-byte swizzle) into a
//              4-stage shared-memory ring, one mbarrier pair per stage;
//   warp 1     allocates 512 tensor-memory columns (two 128x256 fp32 accumulators)
//              and one thread issues tcgen05.mma M128 N256 K16, four per stage,
//              committing each stage back to the producer and each finished tile
//              to the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of their 32-lane quarter of the accumulator,
//              alpha/beta, conversion, store to C; the second accumulator lets the
//              next tile's MMAs run during this tile's epilogue.
// Tiles are visited in groups of 16 tile-rows so the CTAs in flight share A and B
// panels in L2.  A and B must be K-major (cublas transa = T, transb = N) with
// 16-byte aligned leading dimensions; other layouts use the FFMA kernel.
//
// Every mbarrier wait is bounded (tc_ptx.cuh).  A wait that runs out marks the
// CTA aborted, counts the event in g_tc_timeouts, drains the copies and MMAs this
// CTA issued (again with bounded waits), frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "blas/gemm.hpp"
#include "blas/tc_ptx.cuh"
#include "common/device.hpp"

namespace mb200::blas {
namespace {

using namespace mb200::tc;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;            // 64 x 2 bytes = one 128-byte swizzle row
constexpr int UMMA_K = 16;
constexpr int STAGES = 4;
constexpr int ACC = 2;
constexpr int THREADS = 192;
constexpr std::uint32_t TMEM_COLS = 512;
constexpr int A_STAGE = BM * BK * 2;
constexpr int B_STAGE = BN * BK * 2;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = STAGES * (A_STAGE + B_STAGE) + BAR_BYTES + 1024;
constexpr int GROUP_M = 16;

struct TcParams {
  int m, n, k;
  int tiles_m, tiles_n;
  long long tiles_total;
  int a_batched, b_batched;
  void* c;
  long long ldc, stride_c;
  float alpha, beta;
  const float* alpha_dev;
  const float* beta_dev;
};

__device__ unsigned int g_tc_timeouts;

__device__ __forceinline__ void tile_coords(long long t, const TcParams& p, int& z, int& tm,
                                            int& tn) {
  const long long per = static_cast<long long>(p.tiles_m) * p.tiles_n;
  z = static_cast<int>(t / per);
  const int r = static_cast<int>(t % per);
  const int in_group = GROUP_M * p.tiles_n;
  const int first = (r / in_group) * GROUP_M;
  const int gsz = min(p.tiles_m - first, GROUP_M);
  tm = first + (r % in_group) % gsz;
  tn = (r % in_group) / gsz;
}

template <typename T>
__device__ __forceinline__ T cvt_out(float v) {
  if constexpr (std::is_same_v<T, __half>) {
    return __float2half_rn(v);
  } else {
    return __float2bfloat16_rn(v);
  }
}

template <typename T>
__device__ __forceinline__ float cvt_in(T v) {
  if constexpr (std::is_same_v<T, __half>) {
    return __half2float(v);
  } else {
    return __bfloat162float(v);
  }
}

template <typename T, int FMT>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a,
                   const __grid_constant__ CUtensorMap tm_b, const TcParams p) {
  extern __shared__ std::uint8_t smem_raw[];
  std::uint8_t* base = reinterpret_cast<std::uint8_t*>(
      (reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t{1023});
  std::uint8_t* sa = base;
  std::uint8_t* sb = base + STAGES * A_STAGE;
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(sb + STAGES * B_STAGE);
  std::uint64_t* empty = full + STAGES;
  std::uint64_t* acc_full = empty + STAGES;
  std::uint64_t* acc_empty = acc_full + ACC;
  std::uint64_t* mma_done = acc_empty + ACC;
  std::uint32_t* tmem_slot = reinterpret_cast<std::uint32_t*>(mma_done + 1);
  volatile int* aborted = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    *aborted = 0;
    mbar_fence_init();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const std::uint32_t tmem_base = *tmem_slot;
  const int num_kb = (p.k + BK - 1) / BK;
  auto fail = [&]() {
    *aborted = 1;
    atomicAdd(&g_tc_timeouts, 1u);
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
        int z, tm, tn;
        tile_coords(t, p, z, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            fail();
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_STAGE + B_STAGE);
          tma_load_3d(sa + stage * A_STAGE, &tm_a, kb * BK, tm * BM, p.a_batched ? z : 0,
                      &full[stage]);
          tma_load_3d(sb + stage * B_STAGE, &tm_b, kb * BK, tn * BN, p.b_batched ? z : 0,
                      &full[stage]);
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
      constexpr std::uint32_t idesc = f16_idesc(FMT, BM, BN);
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
          const std::uint32_t a0 = smem_addr(sa + stage * A_STAGE);
          const std::uint32_t b0 = smem_addr(sb + stage * B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            mma_f16(d_tmem, kmajor_sw128_desc(a0 + k * UMMA_K * 2),
                    kmajor_sw128_desc(b0 + k * UMMA_K * 2), idesc, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
        if (++acc == ACC) {
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
    const float alpha = p.alpha_dev ? *p.alpha_dev : p.alpha;
    const float beta = p.beta_dev ? *p.beta_dev : p.beta;
    int acc = 0;
    std::uint32_t acc_phase = 0;
    for (long long t = blockIdx.x; t < p.tiles_total && !*aborted; t += gridDim.x) {
      int z, tm, tn;
      tile_coords(t, p, z, tm, tn);
      if (!mbar_wait(&acc_full[acc], acc_phase)) {
        fail();
        break;
      }
      tc_fence_after();
      const int m = tm * BM + quarter * 32 + lane;
      T* cz = static_cast<T*>(p.c) + static_cast<long long>(z) * p.stride_c;
      const std::uint32_t t_row = tmem_base + (static_cast<std::uint32_t>(quarter * 32) << 16) +
                                  static_cast<std::uint32_t>(acc * BN);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_load_32cols(t_row + static_cast<std::uint32_t>(c0), v);
        const int n0 = tn * BN + c0;
        if (m < p.m) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = n0 + j;
            if (n < p.n) {
              T* cp = cz + m + static_cast<long long>(n) * p.ldc;
              const float prev = (beta == 0.0f) ? 0.0f : beta * cvt_in(*cp);
              *cp = cvt_out<T>(fmaf(alpha, v[j], prev));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == ACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// K-major operand: element (k, row) of batch z at base + k + row*ld + z*stride.
bool make_map(CUtensorMap* map, const void* base, int fmt, int k, int rows, long long ld,
              long long stride, int batch, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(batch)};
  long long zs = stride;
  if (batch == 1 || zs == 0) zs = ((ld * rows * 2 + 15) / 16) * 8;  // unused: z is always 0
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(zs * 2)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r =
      fn(map, fmt == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool tc_supported(const GemmArgs& g) {
  if (g.type == Elem::kF32) return false;
  if (!g.trans_a || g.trans_b) return false;  // both operands K-major
  if (g.k <= 0 || g.m <= 0 || g.n <= 0) return false;
  if ((g.lda * 2) % 16 != 0 || (g.ldb * 2) % 16 != 0) return false;
  if (g.batch > 1 && ((g.stride_a * 2) % 16 != 0 || (g.stride_b * 2) % 16 != 0)) return false;
  if (g.stride_a < 0 || g.stride_b < 0) return false;
  if (!aligned_to(g.a, 16) || !aligned_to(g.b, 16)) return false;
  // small problems are faster on the FFMA kernel than one persistent wave
  if (static_cast<double>(g.m) * g.n * g.k < double(1 << 21)) return false;
  return true;
}

}  // namespace

const char* gemm_path_name(const GemmArgs& g) noexcept {
  return tc_supported(g) ? "tcgen05" : "simt";
}

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t stream) noexcept {
  if (!tc_supported(g)) return cudaErrorNotSupported;
  const int fmt = (g.type == Elem::kBF16) ? 1 : 0;
  CUtensorMap ma, mb;
  if (!make_map(&ma, g.a, fmt, g.k, g.m, g.lda, g.stride_a, g.batch, BM) ||
      !make_map(&mb, g.b, fmt, g.k, g.n, g.ldb, g.stride_b, g.batch, BN))
    return cudaErrorNotSupported;
  TcParams p{};
  p.m = g.m;
  p.n = g.n;
  p.k = g.k;
  p.tiles_m = (g.m + BM - 1) / BM;
  p.tiles_n = (g.n + BN - 1) / BN;
  p.tiles_total = static_cast<long long>(p.tiles_m) * p.tiles_n * g.batch;
  p.a_batched = (g.batch > 1 && g.stride_a != 0) ? 1 : 0;
  p.b_batched = (g.batch > 1 && g.stride_b != 0) ? 1 : 0;
  p.c = g.c;
  p.ldc = g.ldc;
  p.stride_c = g.stride_c;
  p.alpha = g.alpha;
  p.beta = g.beta;
  p.alpha_dev = g.alpha_dev;
  p.beta_dev = g.beta_dev;
  const int sms = sm_count(current_device());
  const long long grid = p.tiles_total < sms ? p.tiles_total : sms;
  cudaError_t e;
  if (fmt == 1) {
    auto kern = gemm_tc_kernel<__nv_bfloat16, 1>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(grid), THREADS, SMEM_BYTES, stream>>>(ma, mb, p);
  } else {
    auto kern = gemm_tc_kernel<__half, 0>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(grid), THREADS, SMEM_BYTES, stream>>>(ma, mb, p);
  }
  return cudaGetLastError();
}

}  // namespace mb200::blas
