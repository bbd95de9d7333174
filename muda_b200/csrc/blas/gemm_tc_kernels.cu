// gemm_tc_kernels.cu — tcgen05 tensor-core GEMM for bf16 / fp16 operands (sm_100a).
//
// Semantics are those of the reference's 16-bit GEMM (libraries/blas/shaders/
// cublas_kernels.metal:1008-1045): fp32 accumulation of op(A)*op(B), then
// C = alpha*acc + beta*C (beta == 0: C not read), rounded to the 16-bit type.
//
// The main loop is the persistent warp-specialized kernel of tc_gemm_core.cuh
// with 128 x 256 output tiles and a 4-stage TMA ring.  Tiles are visited in
// groups of 16 tile-rows so the CTAs in flight share A and B panels in L2.  Every
// transpose combination runs on it: a K-major operand (A with transa = T, B with
// transb = N) arrives as one 128-byte-wide box per k-block, an MN-major operand
// (A with transa = N, B with transb = T: M or N is the contiguous dimension) as
// 64 x 64 boxes that the MMA reads through MN-major descriptors.  Leading
// dimensions and batch strides must be multiples of 8 elements (16 bytes) and the
// operands 16-byte aligned; other layouts and small problems use the FFMA kernel.
//
// fp32 GEMM (the reference's cublasSgemm arithmetic, cublas_kernels.metal:969-1006:
// fp32 products accumulated in fp32, then C = alpha*acc + beta*C) runs on the same
// loop in split-tf32 form: one pass writes both operands, in any transpose and
// layout, as K-major hi/lo tf32 planes into the handle's workspace, and the
// tensor cores accumulate lo*hi + hi*lo + hi*hi with the chunked fp32 accumulation
// of tc_gemm_split_kernel (fp32-class accuracy).  Problems with fewer output
// tiles than half the SMs split K across CTAs; each split writes raw sums to the
// workspace and one pass over all SMs adds them in split order (deterministic)
// and applies alpha and beta.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <mutex>

#include "blas/gemm.hpp"
#include "blas/tc_gemm_core.cuh"
#include "blas/tf32_split.hpp"
#include "common/device.hpp"

namespace mb200::blas {
namespace {

constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int GROUP_M = 16;

__device__ unsigned int g_gemm_tc_timeouts;

// TOUT: the problem computes C^T = op(B)^T op(A)^T (its M is C's n, its N is C's m), so
// tile row r is column r of C and a thread's 32 accumulator columns are 32 consecutive
// rows of that column: one 64-byte run of C, written as 16-byte stores.  It turns op
// T,T (B MN-major, the slower operand form) into the A-MN-major / B-K-major form.
template <typename T, bool AMN, bool BMN, bool TOUT = false>
struct GemmProblem {
  static constexpr bool kAMn = AMN, kBMn = BMN;
  CUtensorMap ma;  // A: dims (k, m, batch) K-major, (m, k, batch) MN-major
  CUtensorMap mb;  // B: dims (k, n, batch) K-major, (n, k, batch) MN-major
  long long tiles_total;
  int num_kb;
  int m, n, tiles_m, tiles_n;
  int a_batched, b_batched;
  T* c;
  long long ldc, stride_c;
  float alpha, beta;
  const float* alpha_dev;
  const float* beta_dev;
  int vec_out;  // TOUT: C, ldc and stride_c keep 16-byte alignment of every 8-element run

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

  // K-major: one box of (64 K) x (rows of the tile).  MN-major: boxes of 64 rows of
  // the tile (128 bytes) x 64 K, one after another every 8 KB.
  __device__ void load(const int (&c3)[3], int kb, void* sa, void* sb, std::uint64_t* bar) const {
    const int za = a_batched ? c3[0] : 0, zb = b_batched ? c3[0] : 0;
    if constexpr (AMN) {
#pragma unroll
      for (int j = 0; j < tc::kBM / 64; ++j)
        tc::tma_load_3d(static_cast<std::uint8_t*>(sa) + j * tc::kMnBoxBytes, &ma,
                        c3[1] * tc::kBM + 64 * j, kb * tc::kBK, za, bar);
    } else {
      tc::tma_load_3d(sa, &ma, kb * tc::kBK, c3[1] * tc::kBM, za, bar);
    }
    if constexpr (BMN) {
#pragma unroll
      for (int j = 0; j < BN / 64; ++j)
        tc::tma_load_3d(static_cast<std::uint8_t*>(sb) + j * tc::kMnBoxBytes, &mb,
                        c3[2] * BN + 64 * j, kb * tc::kBK, zb, bar);
    } else {
      tc::tma_load_3d(sb, &mb, kb * tc::kBK, c3[2] * BN, zb, bar);
    }
  }

  __device__ void scalars(float& a, float& b) const {
    a = alpha_dev ? *alpha_dev : alpha;
    b = beta_dev ? *beta_dev : beta;
  }

  // Row `row` of the tile is output row m; columns col0..col0+31 are output columns.
  __device__ void store(const int (&c3)[3], int row, int col0, const float (&v)[32], float a,
                        float b) const {
    if constexpr (TOUT) {
      const int nn = c3[1] * tc::kBM + row;  // column of C
      if (nn >= m) return;
      const int m0 = c3[2] * BN + col0;      // first of 32 consecutive rows of C
      T* cp = c + static_cast<long long>(c3[0]) * stride_c + static_cast<long long>(nn) * ldc + m0;
      if (vec_out && b == 0.0f && m0 + 32 <= n) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          T h[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) h[j] = from_float(a * v[g * 8 + j]);
          *reinterpret_cast<uint4*>(cp + g * 8) = *reinterpret_cast<const uint4*>(h);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (m0 + j < n) {
            const float prev = (b == 0.0f) ? 0.0f : b * to_float(cp[j]);
            cp[j] = from_float(fmaf(a, v[j], prev));
          }
        }
      }
      return;
    }
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

// Operand of `rows` rows (M or N) by k, element (k, row) of batch z at
// base + k + row*ld + z*stride when K-major, base + row + k*ld + z*stride when
// MN-major.  K-major boxes are 64 K x box_rows rows; MN-major boxes 64 rows x 64 K.
bool make_map(CUtensorMap* map, const void* base, int fmt, bool mn_major, int k, int rows,
              long long ld, long long stride, int batch, int box_rows) {
  const long long inner = mn_major ? rows : k, outer = mn_major ? k : rows;
  long long zs = stride;
  if (batch == 1 || zs == 0) zs = ((ld * outer * 2 + 15) / 16) * 8;  // z is always 0 then
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(zs * 2)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(mn_major ? 64 : tc::kBK),
                             static_cast<cuuint32_t>(mn_major ? tc::kBK : box_rows), 1u};
  return tc::encode_tiled(map, fmt, base, 3, dims, strides, box);
}

bool tc_supported(const GemmArgs& g) {
  if (g.type == Elem::kF32) return false;
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

template <typename T, int FMT, bool AMN, bool BMN, bool TOUT = false>
cudaError_t run(const GemmArgs& g, cudaStream_t stream) {
  GemmProblem<T, AMN, BMN, TOUT> p{};
  if (!make_map(&p.ma, g.a, FMT, AMN, g.k, g.m, g.lda, g.stride_a, g.batch, tc::kBM) ||
      !make_map(&p.mb, g.b, FMT, BMN, g.k, g.n, g.ldb, g.stride_b, g.batch, BN))
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
  p.vec_out = (aligned_to(g.c, 16) && g.ldc % 8 == 0 && (g.batch == 1 || g.stride_c % 8 == 0))
                  ? 1 : 0;
  unsigned int* to = timeout_counter();
  if (to == nullptr) return cudaErrorNotSupported;
  return tc::launch_tc_gemm<GemmProblem<T, AMN, BMN, TOUT>, BN, STAGES, FMT>(
      p, sm_count(current_device()), to, stream);
}

// A is MN-major when not transposed (column-major m x k), B when transposed.
template <typename T, int FMT>
cudaError_t run_layout(const GemmArgs& g, cudaStream_t stream) {
  const bool amn = !g.trans_a, bmn = g.trans_b;
  if (amn && bmn) return run<T, FMT, true, true>(g, stream);
  if (amn) return run<T, FMT, true, false>(g, stream);
  if (bmn) {
    // T,T as C^T = op(B)^T op(A)^T: op(B)^T (n x k) is MN-major in B, op(A)^T (k x m)
    // K-major in A, the operand forms of N,N; C is written back transposed
    GemmArgs s = g;
    s.m = g.n;
    s.n = g.m;
    s.a = g.b;
    s.lda = g.ldb;
    s.stride_a = g.stride_b;
    s.b = g.a;
    s.ldb = g.lda;
    s.stride_b = g.stride_a;
    return run<T, FMT, true, false, true>(s, stream);
  }
  return run<T, FMT, false, false>(g, stream);
}

// ---------------------------------------------------------------- split tf32 (fp32)

// Tile width by output columns (n <= 64: 64, <= 128: 128, else 256) and the ring
// depth that fills about 192 KB: stages of 32 KB (A) + TBN * 256 B (B).
template <int TBN>
constexpr int kSplitStages = TBN == 64 ? 4 : TBN == 128 ? 3 : 2;
int split_bn(int n) { return n <= 64 ? 64 : n <= 128 ? 128 : 256; }
constexpr int kMaxSplitK = 32;
constexpr std::size_t kWorkspaceCap = std::size_t{2} << 30;

template <int TBN>
struct SplitGemmProblem {
  CUtensorMap ma;  // A planes: dims (k, m, batch, plane), box {32, 128, 1, 2}
  CUtensorMap mb;  // B planes: dims (k, n, batch, plane), box {32, TBN, 1, 2}
  long long tiles_total;
  int num_kb;  // k-blocks per split
  int ksplit;
  int m, n, tiles_m, tiles_n;
  float* c;
  long long ldc, stride_c;
  float* partial;  // ksplit > 1: [batch][ksplit] m x n column-major raw sums
  float alpha, beta;
  const float* alpha_dev;
  const float* beta_dev;

  __device__ void prefetch() const {
    tc::prefetch_tensormap(&ma);
    tc::prefetch_tensormap(&mb);
  }

  // (batch * ksplit + split, tile row, tile column), GROUP_M tile-rows at a time.
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
    const int z = c3[0] / ksplit;
    const int k = ((c3[0] % ksplit) * num_kb + kb) * tc::kBK32;  // past K reads as zeros
    tc::tma_load_4d(sa, &ma, k, c3[1] * tc::kBM, z, 0, bar);
    tc::tma_load_4d(sb, &mb, k, c3[2] * TBN, z, 0, bar);
  }

  __device__ void scalars(float& a, float& b) const {
    a = alpha_dev ? *alpha_dev : alpha;
    b = beta_dev ? *beta_dev : beta;
  }

  __device__ void store(const int (&c3)[3], int row, int col0, const float (&v)[32], float a,
                        float b) const {
    const int mm = c3[1] * tc::kBM + row;
    if (mm >= m) return;
    const int n0 = c3[2] * TBN + col0;
    if (ksplit > 1) {
      float* pz = partial + static_cast<long long>(c3[0]) * m * n + mm;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < n) pz[static_cast<long long>(n0 + j) * m] = v[j];
      return;
    }
    float* cz = c + static_cast<long long>(c3[0]) * stride_c + mm;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int nn = n0 + j;
      if (nn < n) {
        float* cp = cz + static_cast<long long>(nn) * ldc;
        const float prev = (b == 0.0f) ? 0.0f : b * *cp;
        *cp = fmaf(a, v[j], prev);
      }
    }
  }
};

// C = alpha * (sum of the ksplit partial sums, in split order) + beta * C; one
// column of one batch entry per blockIdx.y step, rows across threads (four rows
// per thread with Vec: m % 4 == 0, ldc % 4 == 0, C 16-byte aligned).
template <bool Vec>
__global__ void __launch_bounds__(256)
    reduce_splits(const float* __restrict__ partial, int ksplit, int m, int n, int batch,
                  float* c, long long ldc, long long stride_c, float alpha, float beta,
                  const float* alpha_dev, const float* beta_dev) {
  const float a = alpha_dev ? *alpha_dev : alpha;
  const float b = beta_dev ? *beta_dev : beta;
  const long long mn = static_cast<long long>(m) * n;
  const int per = Vec ? m / 4 : m;
  const long long cols = static_cast<long long>(n) * batch;
  for (long long cz = blockIdx.y; cz < cols; cz += gridDim.y) {
    const long long z = cz / n, col = cz % n;
    const float* pz = partial + z * ksplit * mn + col * m;
    float* cp = c + z * stride_c + col * ldc;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < per; i += gridDim.x * blockDim.x) {
      if constexpr (Vec) {
        float4 acc = __ldcs(reinterpret_cast<const float4*>(pz) + i);
        for (int sp = 1; sp < ksplit; ++sp) {
          const float4 v = __ldcs(reinterpret_cast<const float4*>(pz + sp * mn) + i);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        float4* cv = reinterpret_cast<float4*>(cp) + i;
        float4 prev = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (b != 0.0f) {
          prev = *cv;
          prev = make_float4(b * prev.x, b * prev.y, b * prev.z, b * prev.w);
        }
        *cv = make_float4(fmaf(a, acc.x, prev.x), fmaf(a, acc.y, prev.y), fmaf(a, acc.z, prev.z),
                          fmaf(a, acc.w, prev.w));
      } else {
        float acc = __ldcs(pz + i);
        for (int sp = 1; sp < ksplit; ++sp) acc += __ldcs(pz + sp * mn + i);
        const float prev = (b == 0.0f) ? 0.0f : b * cp[i];
        cp[i] = fmaf(a, acc, prev);
      }
    }
  }
}

long long round_up4(long long v) { return (v + 3) / 4 * 4; }

struct SplitPlan {
  int nb;      // batch entries per chunk
  int bn;      // tile width (64, 128 or 256)
  int ksplit;  // K splits
  int kb_per;  // k-blocks per split
  std::size_t a_floats, b_floats, p_floats;
  std::size_t bytes() const { return (a_floats + b_floats + p_floats) * 4; }
};

SplitPlan plan_split(const GemmArgs& g, int sms, int nb) {
  SplitPlan pl{};
  pl.nb = nb;
  const long long ldk = round_up4(g.k);
  // the tile width follows n only: a narrower tile to raise the tile count re-reads
  // the A panel once per tile column (1024^3 at 64 columns: 28.8 us for the GEMM
  // alone, against 19.5 + 7 us for 256 columns split four ways plus the reduction)
  const int bn = split_bn(g.n);
  pl.bn = bn;
  const int tiles = ((g.m + tc::kBM - 1) / tc::kBM) * ((g.n + bn - 1) / bn) * nb;
  const int total_kb = (g.k + tc::kBK32 - 1) / tc::kBK32;
  int ks = 1;
  if (2 * tiles < sms) {
    ks = sms / tiles;
    if (ks > total_kb / 4) ks = total_kb / 4;
    if (ks > kMaxSplitK) ks = kMaxSplitK;
    if (ks < 1) ks = 1;
  }
  pl.kb_per = (total_kb + ks - 1) / ks;
  pl.ksplit = (total_kb + pl.kb_per - 1) / pl.kb_per;
  pl.a_floats = 2ull * nb * g.m * ldk;
  pl.b_floats = 2ull * nb * g.n * ldk;
  pl.p_floats = pl.ksplit > 1 ? static_cast<std::size_t>(pl.ksplit) * nb * g.m * g.n : 0;
  return pl;
}

// Largest batch chunk whose workspace fits the cap (0 if one entry does not).
SplitPlan plan_for(const GemmArgs& g, int sms) {
  int nb = g.batch;
  SplitPlan pl = plan_split(g, sms, nb);
  while (pl.bytes() > kWorkspaceCap && nb > 1) {
    nb = (nb + 1) / 2;
    pl = plan_split(g, sms, nb);
  }
  if (pl.bytes() > kWorkspaceCap) pl.nb = 0;
  return pl;
}

bool tf32x3_supported(const GemmArgs& g) {
  if (g.type != Elem::kF32) return false;
  if (g.k <= 0 || g.m <= 0 || g.n <= 0 || g.batch <= 0) return false;
  if (g.stride_a < 0 || g.stride_b < 0) return false;
  // small problems are faster on the FFMA kernel than split + tensor cores
  if (static_cast<double>(g.m) * g.n * g.k < double(1 << 24)) return false;
  return true;
}

bool make_plane_map(CUtensorMap* map, const float* planes, long long k, long long rows,
                    int batch, long long ldk, int box_rows) {
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(batch), 2u};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ldk * 4),
                                 static_cast<cuuint64_t>(rows * ldk * 4),
                                 static_cast<cuuint64_t>(batch * rows * ldk * 4)};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(tc::kBK32),
                             static_cast<cuuint32_t>(box_rows), 1u, 2u};
  return tc::encode_tiled(map, 2, planes, 4, dims, strides, box);
}

template <int TBN>
cudaError_t run_split_gemm(const GemmArgs& g, const SplitPlan& pl, int nb, const float* pa,
                           const float* pb, float* pp, float* c, int sms, unsigned int* to,
                           cudaStream_t stream) {
  const long long ldk = round_up4(g.k);
  SplitGemmProblem<TBN> p{};
  if (!make_plane_map(&p.ma, pa, g.k, g.m, nb, ldk, tc::kBM) ||
      !make_plane_map(&p.mb, pb, g.k, g.n, nb, ldk, TBN))
    return cudaErrorNotSupported;
  p.m = g.m;
  p.n = g.n;
  p.tiles_m = (g.m + tc::kBM - 1) / tc::kBM;
  p.tiles_n = (g.n + TBN - 1) / TBN;
  p.ksplit = pl.ksplit;
  p.num_kb = pl.kb_per;
  p.tiles_total = static_cast<long long>(p.tiles_m) * p.tiles_n * nb * pl.ksplit;
  p.c = c;
  p.ldc = g.ldc;
  p.stride_c = g.stride_c;
  p.partial = pp;
  p.alpha = g.alpha;
  p.beta = g.beta;
  p.alpha_dev = g.alpha_dev;
  p.beta_dev = g.beta_dev;
  return tc::launch_tc_gemm<SplitGemmProblem<TBN>, TBN, kSplitStages<TBN>, tc::kFmtTf32x3>(
      p, sms, to, stream);
}

// a_planes: op(A) already split (batch 1), else nullptr and A is split here.
cudaError_t run_chunk(const GemmArgs& g, const SplitPlan& pl, int z0, int nb, float* ws,
                      int sms, unsigned int* to, cudaStream_t stream,
                      const float* a_planes = nullptr) {
  const long long ldk = round_up4(g.k);
  float* pa = a_planes != nullptr ? const_cast<float*>(a_planes) : ws;
  float* pb = a_planes != nullptr ? ws : ws + pl.a_floats;
  float* pp = pb + pl.b_floats;
  // op(A) is m x k: element (i, p) at A[i + p*lda] (N) or A[p + i*lda] (T);
  // op(B) is k x n: element (p, j) at B[p + j*ldb] (N) or B[j + p*ldb] (T), rows j
  const float* b = static_cast<const float*>(g.b) + z0 * g.stride_b;
  const tc::SplitJob jb{b, g.n, g.k, nb, g.trans_b ? 1 : g.ldb, g.trans_b ? g.ldb : 1,
                        g.stride_b, pb, ldk};
  cudaError_t e;
  if (a_planes != nullptr) {
    e = tc::launch_tf32_split(jb.src, jb.rows, jb.cols, jb.batch, jb.rs, jb.ks, jb.zs, jb.dst,
                              jb.ldk, stream);
  } else {
    const float* a = static_cast<const float*>(g.a) + z0 * g.stride_a;
    const tc::SplitJob ja{a, g.m, g.k, nb, g.trans_a ? g.lda : 1, g.trans_a ? 1 : g.lda,
                          g.stride_a, pa, ldk};
    e = tc::launch_tf32_split_pair(ja, jb, stream);
  }
  if (e != cudaSuccess) return e;
  float* c = static_cast<float*>(g.c) + z0 * g.stride_c;
  switch (pl.bn) {
    case 64: e = run_split_gemm<64>(g, pl, nb, pa, pb, pp, c, sms, to, stream); break;
    case 128: e = run_split_gemm<128>(g, pl, nb, pa, pb, pp, c, sms, to, stream); break;
    default: e = run_split_gemm<256>(g, pl, nb, pa, pb, pp, c, sms, to, stream); break;
  }
  if (e != cudaSuccess || pl.ksplit == 1) return e;
  const bool vec = g.m % 4 == 0 && g.ldc % 4 == 0 && (nb == 1 || g.stride_c % 4 == 0) &&
                   aligned_to(c, 16);
  const int per = vec ? g.m / 4 : g.m;
  const long long cols = static_cast<long long>(g.n) * nb;
  const dim3 grid(static_cast<unsigned>((per + 255) / 256 < 64 ? (per + 255) / 256 : 64),
                  static_cast<unsigned>(cols < 65535 ? cols : 65535));
  if (vec)
    reduce_splits<true><<<grid, 256, 0, stream>>>(pp, pl.ksplit, g.m, g.n, nb, c, g.ldc,
                                                  g.stride_c, g.alpha, g.beta, g.alpha_dev,
                                                  g.beta_dev);
  else
    reduce_splits<false><<<grid, 256, 0, stream>>>(pp, pl.ksplit, g.m, g.n, nb, c, g.ldc,
                                                   g.stride_c, g.alpha, g.beta, g.alpha_dev,
                                                   g.beta_dev);
  return cudaGetLastError();
}

}  // namespace

std::size_t gemm_tf32x3_workspace(const GemmArgs& g) noexcept {
  if (!tf32x3_supported(g)) return 0;
  const SplitPlan pl = plan_for(g, sm_count(current_device()));
  return pl.nb == 0 ? 0 : pl.bytes();
}

cudaError_t launch_gemm_tf32x3(const GemmArgs& g, void* workspace, std::size_t ws_bytes,
                               cudaStream_t stream) noexcept {
  if (!tf32x3_supported(g)) return cudaErrorNotSupported;
  const int sms = sm_count(current_device());
  const SplitPlan pl = plan_for(g, sms);
  if (pl.nb == 0 || workspace == nullptr || ws_bytes < pl.bytes() ||
      !aligned_to(workspace, 16))
    return cudaErrorNotSupported;
  unsigned int* to = timeout_counter();
  if (to == nullptr) return cudaErrorNotSupported;
  for (int z0 = 0; z0 < g.batch; z0 += pl.nb) {
    const int nb = g.batch - z0 < pl.nb ? g.batch - z0 : pl.nb;
    const SplitPlan cur = nb == pl.nb ? pl : plan_split(g, sms, nb);
    const cudaError_t e =
        run_chunk(g, cur, z0, nb, static_cast<float*>(workspace), sms, to, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

std::size_t gemm_tf32x3_aplanes_workspace(const GemmArgs& g) noexcept {
  if (!tf32x3_supported(g) || g.batch != 1) return 0;
  const SplitPlan pl = plan_for(g, sm_count(current_device()));
  return pl.nb == 0 ? 0 : pl.bytes() - pl.a_floats * 4;
}

cudaError_t launch_gemm_tf32x3_aplanes(const GemmArgs& g, const float* a_planes, void* workspace,
                                       std::size_t ws_bytes, cudaStream_t stream) noexcept {
  if (!tf32x3_supported(g) || g.batch != 1 || a_planes == nullptr ||
      !aligned_to(a_planes, 16))
    return cudaErrorNotSupported;
  const int sms = sm_count(current_device());
  const SplitPlan pl = plan_for(g, sms);
  if (pl.nb == 0 || workspace == nullptr || ws_bytes < pl.bytes() - pl.a_floats * 4 ||
      !aligned_to(workspace, 16))
    return cudaErrorNotSupported;
  unsigned int* to = timeout_counter();
  if (to == nullptr) return cudaErrorNotSupported;
  return run_chunk(g, pl, 0, 1, static_cast<float*>(workspace), sms, to, stream, a_planes);
}

const char* gemm_path_name(const GemmArgs& g) noexcept {
  if (tc_supported(g)) return "tcgen05";
  if (gemm_tf32x3_workspace(g) != 0) return "tcgen05-tf32x3";
  return "simt";
}

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t stream) noexcept {
  if (!tc_supported(g)) return cudaErrorNotSupported;
  return g.type == Elem::kBF16 ? run_layout<__nv_bfloat16, 1>(g, stream)
                               : run_layout<__half, 0>(g, stream);
}

}  // namespace mb200::blas
