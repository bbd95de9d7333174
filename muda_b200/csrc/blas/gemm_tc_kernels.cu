// gemm_tc_kernels.cu — tcgen05 tensor-core GEMM for bf16 / fp16 operands (sm_100a).
//
// Semantics are those of the reference's 16-bit GEMM (libraries/blas/shaders/
// cublas_kernels.metal:1008-1045): fp32 accumulation of op(A)*op(B), then
// C = alpha*acc + beta*C (beta == 0: C not read), rounded to the 16-bit type.
//
// The main loop is the persistent warp-specialized kernel of tc_gemm_core.cuh
// with 128 x 256 output tiles and a 4-stage TMA ring.  Tiles are visited in
// groups of 16 tile-rows so the CTAs in flight share A and B panels in L2.  A and
// B must be K-major (cublas transa = T, transb = N) with 16-byte aligned leading
// dimensions; other layouts use the FFMA kernel.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <mutex>

#include "blas/gemm.hpp"
#include "blas/tc_gemm_core.cuh"
#include "common/device.hpp"

namespace mb200::blas {
namespace {

constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int GROUP_M = 16;

__device__ unsigned int g_gemm_tc_timeouts;

template <typename T>
struct GemmProblem {
  CUtensorMap ma;  // K-major A: dims (k, m, batch)
  CUtensorMap mb;  // K-major B: dims (k, n, batch)
  long long tiles_total;
  int num_kb;
  int m, n, tiles_m, tiles_n;
  int a_batched, b_batched;
  T* c;
  long long ldc, stride_c;
  float alpha, beta;
  const float* alpha_dev;
  const float* beta_dev;

  __device__ void prefetch() const {
    tc::prefetch_tensormap(&ma);
    tc::prefetch_tensormap(&mb);
  }

  // (batch, tile row, tile column), grouped GROUP_M tile-rows at a time.
  __device__ void coords(long long t, int (&c3)[3]) const {
    const long long per = static_cast<long long>(tiles_m) * tiles_n;
    const int r = static_cast<int>(t % per);
    const int in_group = GROUP_M * tiles_n;
    const int first = (r / in_group) * GROUP_M;
    const int gsz = min(tiles_m - first, GROUP_M);
    c3[0] = static_cast<int>(t / per);
    c3[1] = first + (r % in_group) % gsz;
    c3[2] = (r % in_group) / gsz;
  }

  __device__ void load(const int (&c3)[3], int kb, void* sa, void* sb, std::uint64_t* bar) const {
    tc::tma_load_3d(sa, &ma, kb * tc::kBK, c3[1] * tc::kBM, a_batched ? c3[0] : 0, bar);
    tc::tma_load_3d(sb, &mb, kb * tc::kBK, c3[2] * BN, b_batched ? c3[0] : 0, bar);
  }

  __device__ void scalars(float& a, float& b) const {
    a = alpha_dev ? *alpha_dev : alpha;
    b = beta_dev ? *beta_dev : beta;
  }

  // Row `row` of the tile is output row m; columns col0..col0+31 are output columns.
  __device__ void store(const int (&c3)[3], int row, int col0, const float (&v)[32], float a,
                        float b) const {
    const int mm = c3[1] * tc::kBM + row;
    if (mm >= m) return;
    T* cz = c + static_cast<long long>(c3[0]) * stride_c + mm;
    const int n0 = c3[2] * BN + col0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int nn = n0 + j;
      if (nn < n) {
        T* cp = cz + static_cast<long long>(nn) * ldc;
        const float prev = (b == 0.0f) ? 0.0f : b * to_float(*cp);
        *cp = from_float(fmaf(a, v[j], prev));
      }
    }
  }

  __device__ static float to_float(T v) {
    if constexpr (std::is_same_v<T, __half>) {
      return __half2float(v);
    } else {
      return __bfloat162float(v);
    }
  }
  __device__ static T from_float(float v) {
    if constexpr (std::is_same_v<T, __half>) {
      return __float2half_rn(v);
    } else {
      return __float2bfloat16_rn(v);
    }
  }
};

// K-major operand: element (k, row) of batch z at base + k + row*ld + z*stride.
bool make_map(CUtensorMap* map, const void* base, int fmt, int k, int rows, long long ld,
              long long stride, int batch, int box_rows) {
  long long zs = stride;
  if (batch == 1 || zs == 0) zs = ((ld * rows * 2 + 15) / 16) * 8;  // z is always 0 then
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(zs * 2)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(tc::kBK), static_cast<cuuint32_t>(box_rows),
                             1u};
  return tc::encode_tiled(map, fmt, base, 3, dims, strides, box);
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

unsigned int* timeout_counter() {
  static std::mutex mu;
  static std::array<unsigned int*, 64> addr{};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_tc_timeouts) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    addr[dev] = static_cast<unsigned int*>(p);
  }
  return addr[dev];
}

template <typename T, int FMT>
cudaError_t run(const GemmArgs& g, cudaStream_t stream) {
  GemmProblem<T> p{};
  if (!make_map(&p.ma, g.a, FMT, g.k, g.m, g.lda, g.stride_a, g.batch, tc::kBM) ||
      !make_map(&p.mb, g.b, FMT, g.k, g.n, g.ldb, g.stride_b, g.batch, BN))
    return cudaErrorNotSupported;
  p.m = g.m;
  p.n = g.n;
  p.tiles_m = (g.m + tc::kBM - 1) / tc::kBM;
  p.tiles_n = (g.n + BN - 1) / BN;
  p.tiles_total = static_cast<long long>(p.tiles_m) * p.tiles_n * g.batch;
  p.num_kb = (g.k + tc::kBK - 1) / tc::kBK;
  p.a_batched = (g.batch > 1 && g.stride_a != 0) ? 1 : 0;
  p.b_batched = (g.batch > 1 && g.stride_b != 0) ? 1 : 0;
  p.c = static_cast<T*>(g.c);
  p.ldc = g.ldc;
  p.stride_c = g.stride_c;
  p.alpha = g.alpha;
  p.beta = g.beta;
  p.alpha_dev = g.alpha_dev;
  p.beta_dev = g.beta_dev;
  unsigned int* to = timeout_counter();
  if (to == nullptr) return cudaErrorNotSupported;
  return tc::launch_tc_gemm<GemmProblem<T>, BN, STAGES, FMT>(p, sm_count(current_device()), to,
                                                             stream);
}

}  // namespace

const char* gemm_path_name(const GemmArgs& g) noexcept {
  return tc_supported(g) ? "tcgen05" : "simt";
}

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t stream) noexcept {
  if (!tc_supported(g)) return cudaErrorNotSupported;
  return g.type == Elem::kBF16 ? run<__nv_bfloat16, 1>(g, stream) : run<__half, 0>(g, stream);
}

}  // namespace mb200::blas
