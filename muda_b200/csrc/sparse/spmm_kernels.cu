// spmm_kernels.cu — transposed CSR SpMV and CSR SpMM for sm_100a.
//
// Transposed SpMV, y = alpha * A^T * x + beta * y.  The reference's fp32 path
// (libraries/sparse/src/cusparse_ops.mm:166-191, cusparse_kernels.metal:21-52)
// scales y by beta and then adds alpha*x[r]*a_rk into y[col] with a CAS loop per
// stored entry, one thread per row; its fp16 path is the generic kernel (:116-132),
// one thread per output scanning the whole matrix.  Here both are one pass over the
// matrix in the forward kernel's warp tiles (S lanes per row, long rows on the
// whole warp), each entry a fire-and-forget `red.global.add.f32` into y (fp32) or
// into an fp32 scratch vector that a last pass rounds to half (fp16).
//
// SpMM, C = alpha * op(A) * op(B) + beta * C (fp32; cusparse_kernels.metal:201-281).
// Non-transposed A: one warp per row of A, lanes over output columns (4 per lane
// with float4 loads when B and C are row-contiguous and 16-byte aligned); the row's
// entries are read 32 at a time, coalesced, and broadcast by shuffle, so every
// output is sum = fma(a_k, B(col_k, c), sum) in entry order followed by
// fma(alpha, sum, beta*C) — the reference's per-output arithmetic, bit for bit.
// Transposed A: C is scaled by beta, then each row r of A adds alpha*a_rk*B(r, c)
// into C(col_k, c) with `red.global.add.f32` (B's row is loaded once per row).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common/device.hpp"
#include "sparse/csr_device.cuh"
#include "sparse/spmv.hpp"

namespace mb200::sparse {
namespace {

constexpr int kWarps = 8;
constexpr unsigned kFull = 0xffffffffu;

unsigned grid_for(std::int64_t units, std::int64_t per_cta, int waves) {
  const std::int64_t want = (units + per_cta - 1) / per_cta;
  const int sms = sm_count(current_device());
  const std::int64_t cap = static_cast<std::int64_t>(sms > 0 ? sms : 148) * waves;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

// ---------------------------------------------------------------- SpMV^T --

// fp32: y = beta == 0 ? 0 : beta * y.  fp16: scratch = 0.
template <class T>
__global__ void __launch_bounds__(256)
    spmv_t_prepare(T* __restrict__ y, float* __restrict__ scratch, std::int64_t n, float beta) {
  for (std::int64_t i = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    if constexpr (sizeof(T) == 4) {
      y[i] = (beta == 0.0f) ? 0.0f : beta * y[i];
    } else {
      scratch[i] = 0.0f;
    }
  }
}

// fp16: y = half(fma(alpha, scratch, beta == 0 ? 0 : beta * y)).
__global__ void __launch_bounds__(256)
    spmv_t_finish(__half* __restrict__ y, const float* __restrict__ scratch, std::int64_t n,
                  float alpha, float beta) {
  for (std::int64_t i = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const float prev = (beta == 0.0f) ? 0.0f : beta * __half2float(y[i]);
    y[i] = __float2half_rn(fmaf(alpha, scratch[i], prev));
  }
}

// Adds the entries k in [s, e) of row r, lanes gl, gl + S, ...: fp32 adds
// ax * a_k (ax = alpha * x[r]; rows with ax == 0 and zero products skipped, as the
// reference does); fp16 adds a_k * x[r] into the fp32 scratch.
template <class T>
__device__ __forceinline__ void scatter_row(const CsrView& a, float xr, float alpha, int s, int e,
                                            int gl, int step, float* __restrict__ target) {
  const T* vals = static_cast<const T*>(a.values);
  const float ax = (sizeof(T) == 4) ? alpha * xr : xr;
  if (sizeof(T) == 4 && ax == 0.0f) return;
  int k = s + gl;
  // four entries at a time: all eight loads are in flight before the first reduction
  for (; k + 3 * step < e; k += 4 * step) {
    int c[4];
    T v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      c[u] = __ldcs(a.col_ind + k + u * step) - a.base;
      v[u] = __ldcs(vals + k + u * step);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (static_cast<unsigned>(c[u]) >= static_cast<unsigned long long>(a.cols)) continue;
      const float p = (sizeof(T) == 4) ? ax * widen(v[u]) : widen(v[u]) * ax;
      if (sizeof(T) == 4 && p == 0.0f) continue;
      atomicAdd(target + c[u], p);
    }
  }
  for (; k < e; k += step) {
    const int c = __ldcs(a.col_ind + k) - a.base;
    if (static_cast<unsigned>(c) >= static_cast<unsigned long long>(a.cols)) continue;
    const float p = (sizeof(T) == 4) ? ax * widen(__ldcs(vals + k)) : widen(__ldcs(vals + k)) * ax;
    if (sizeof(T) == 4 && p == 0.0f) continue;
    atomicAdd(target + c, p);
  }
}

template <int S, class T>
__global__ void __launch_bounds__(kWarps * 32)
    spmv_t_scatter(const CsrView a, const T* __restrict__ x, float* __restrict__ target,
                   float alpha) {
  constexpr int G = 32 / S;
  constexpr int kLong = 8 * S;
  const int lane = threadIdx.x & 31;
  const int grp = lane / S;
  const int gl = lane % S;
  const std::int64_t tiles = (a.rows + 31) / 32;
  const std::int64_t warp0 = static_cast<std::int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const std::int64_t nwarps = static_cast<std::int64_t>(gridDim.x) * kWarps;
  for (std::int64_t tile = warp0; tile < tiles; tile += nwarps) {
    const std::int64_t r0 = tile * 32;
    int s_i = 0, e_i = 0;
    float x_i = 0.0f;
    if (r0 + lane < a.rows) {
      s_i = clamp_off(a.row_offsets[r0 + lane], a.base, a.nnz);
      e_i = clamp_off(a.row_offsets[r0 + lane + 1], a.base, a.nnz);
      if (e_i < s_i) e_i = s_i;
      x_i = widen(x[r0 + lane]);
    }
    unsigned long_rows = __ballot_sync(kFull, e_i - s_i > kLong);
#pragma unroll 1
    for (int q = 0; q < S; ++q) {
      const int rl = q * G + grp;
      const int s = __shfl_sync(kFull, s_i, rl);
      const int e = __shfl_sync(kFull, e_i, rl);
      const float xr = __shfl_sync(kFull, x_i, rl);
      if (!((long_rows >> rl) & 1u)) scatter_row<T>(a, xr, alpha, s, e, gl, S, target);
    }
    while (long_rows != 0u) {
      const int rl = __ffs(long_rows) - 1;
      long_rows &= long_rows - 1u;
      const int s = __shfl_sync(kFull, s_i, rl);
      const int e = __shfl_sync(kFull, e_i, rl);
      const float xr = __shfl_sync(kFull, x_i, rl);
      scatter_row<T>(a, xr, alpha, s, e, lane, 32, target);
    }
  }
}

template <int S, class T>
cudaError_t scatter_width(const CsrView& a, const T* x, float* target, float alpha,
                          cudaStream_t st) {
  spmv_t_scatter<S, T><<<grid_for((a.rows + 31) / 32, kWarps, 32), kWarps * 32, 0, st>>>(
      a, x, target, alpha);
  return cudaGetLastError();
}

template <class T>
cudaError_t spmv_t_typed(const CsrView& a, const void* xv, void* yv, float alpha, float beta,
                         float* scratch, cudaStream_t st) {
  const T* x = static_cast<const T*>(xv);
  T* y = static_cast<T*>(yv);
  float* target = (sizeof(T) == 4) ? reinterpret_cast<float*>(y) : scratch;
  spmv_t_prepare<T><<<grid_for(a.cols, 256, 8), 256, 0, st>>>(y, scratch, a.cols, beta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (a.rows > 0) {
    switch (spmv_group_width(a.rows, a.nnz)) {
      case 2: e = scatter_width<2, T>(a, x, target, alpha, st); break;
      case 4: e = scatter_width<4, T>(a, x, target, alpha, st); break;
      case 8: e = scatter_width<8, T>(a, x, target, alpha, st); break;
      case 16: e = scatter_width<16, T>(a, x, target, alpha, st); break;
      default: e = scatter_width<32, T>(a, x, target, alpha, st); break;
    }
    if (e != cudaSuccess) return e;
  }
  if constexpr (sizeof(T) == 2) {
    spmv_t_finish<<<grid_for(a.cols, 256, 8), 256, 0, st>>>(y, scratch, a.cols, alpha, beta);
    e = cudaGetLastError();
  }
  return e;
}

// ------------------------------------------------------------------ SpMM --

// Element (r, c) of a dense operand; ROW: known at compile time to be
// row-contiguous (m[r * ld + c]).
template <bool ROW>
__device__ __forceinline__ std::int64_t dense_index(const DenseView& d, std::int64_t r,
                                                    std::int64_t c) {
  if constexpr (ROW) {
    return r * d.ld + c;
  } else {
    const std::int64_t er = d.trans ? c : r;
    const std::int64_t ec = d.trans ? r : c;
    return d.col_major ? er + ec * d.ld : er * d.ld + ec;
  }
}

template <int VEC>
struct Vec {
  float v[VEC];
};

template <int VEC, bool ROW>
__device__ __forceinline__ Vec<VEC> load_b(const DenseView& b, std::int64_t r, std::int64_t c) {
  Vec<VEC> out;
  if constexpr (VEC == 4) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(b.m + dense_index<true>(b, r, c)));
    out.v[0] = q.x;
    out.v[1] = q.y;
    out.v[2] = q.z;
    out.v[3] = q.w;
  } else {
    out.v[0] = __ldg(b.m + dense_index<ROW>(b, r, c));
  }
  return out;
}

// acc[v] = fma(a_k, B(col_k, col + v), acc[v]) over the entries k in [s, e), in
// order.  The G lanes of a group (shuffle mask `mask`) read the entries G at a time
// (coalesced) and broadcast them; the B rows of kDepth entries are loaded before
// their fmas, so kDepth gathers are in flight per lane (a power-law row of
// thousands of entries is one sequential chain: its latency, not bandwidth, is the
// limit).
constexpr int kDepth = 4;

template <int VEC, int G, bool BROW>
__device__ __forceinline__ void accumulate_range(const CsrView& a, const DenseView& b, int s, int e,
                                                 int gl, unsigned mask, std::int64_t col,
                                                 bool live, float (&acc)[VEC]) {
  constexpr int D = kDepth < G ? kDepth : G;
  const float* vals = static_cast<const float*>(a.values);
  for (int k0 = s; k0 < e; k0 += G) {
    int kk = -1;
    float vv = 0.0f;
    if (k0 + gl < e) {
      kk = __ldg(a.col_ind + k0 + gl) - a.base;
      vv = __ldg(vals + k0 + gl);
    }
    const int cnt = (e - k0 < G) ? e - k0 : G;
    int j = 0;
    for (; j + D <= cnt; j += D) {
      int k[D];
      float av[D];
      Vec<VEC> bv[D];
#pragma unroll
      for (int u = 0; u < D; ++u) {
        k[u] = __shfl_sync(mask, kk, j + u, G);
        av[u] = __shfl_sync(mask, vv, j + u, G);
        if (static_cast<unsigned>(k[u]) < static_cast<unsigned long long>(a.cols) && live)
          bv[u] = load_b<VEC, BROW>(b, k[u], col);
      }
#pragma unroll
      for (int u = 0; u < D; ++u) {
        if (static_cast<unsigned>(k[u]) < static_cast<unsigned long long>(a.cols) && live) {
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[v] = fmaf(av[u], bv[u].v[v], acc[v]);
        }
      }
    }
    for (; j < cnt; ++j) {
      const int k = __shfl_sync(mask, kk, j, G);
      const float av = __shfl_sync(mask, vv, j, G);
      if (static_cast<unsigned>(k) < static_cast<unsigned long long>(a.cols) && live) {
        const Vec<VEC> bv = load_b<VEC, BROW>(b, k, col);
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] = fmaf(av, bv.v[v], acc[v]);
      }
    }
  }
}

// Non-transposed A: groups of G lanes per row (32 / G rows per warp), lane gl of a
// group owning columns cb + gl*VEC .. +VEC of each G*VEC-column block; every output
// is summed in entry order (bit-identical to the reference).
template <int VEC, int G, bool BROW, bool CROW>
__global__ void __launch_bounds__(kWarps * 32)
    spmm_rows(const CsrView a, const DenseView b, const DenseView c, std::int64_t ncols,
              float alpha, float beta) {
  constexpr int RPW = 32 / G;
  const int lane = threadIdx.x & 31;
  const int g = lane / G, gl = lane % G;
  const unsigned mask = (G == 32) ? kFull : (((1u << G) - 1u) << (g * G));
  const std::int64_t warp0 = static_cast<std::int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const std::int64_t nwarps = static_cast<std::int64_t>(gridDim.x) * kWarps;
  for (std::int64_t row0 = warp0 * RPW; row0 < a.rows; row0 += nwarps * RPW) {
    const std::int64_t row = row0 + g;
    if (row >= a.rows) continue;  // the whole group leaves together
    const int s = clamp_off(a.row_offsets[row], a.base, a.nnz);
    const int e0 = clamp_off(a.row_offsets[row + 1], a.base, a.nnz);
    const int e = e0 < s ? s : e0;
    for (std::int64_t cb = 0; cb < ncols; cb += G * VEC) {
      const std::int64_t col = cb + static_cast<std::int64_t>(gl) * VEC;
      const bool live = col < ncols;
      float acc[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = 0.0f;
      accumulate_range<VEC, G, BROW>(a, b, s, e, gl, mask, col, live, acc);
      if (live) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          float* out = c.m + dense_index<CROW>(c, row, col + v);
          const float prev = (beta == 0.0f) ? 0.0f : beta * *out;
          *out = fmaf(alpha, acc[v], prev);
        }
      }
    }
  }
}

// Row-major B and C in 16-byte vectors: the same sums (entry order, bit-identical),
// scheduled for a power-law row-length distribution.
// - Gathers: each lane copies its own 16-byte slice of the B row of entry
//   t + kRing - 1 into a per-lane ring in shared memory with cp.async (L2 only)
//   while it consumes entry t, so kRing - 1 gathers per lane are in flight without
//   holding registers.  A lane reads only the slots it wrote (cp.async.wait_group
//   orders its own copies), so no barrier is needed.  A bit per slot records
//   entries whose column is out of range; they are skipped, as in spmm_rows.
// - Lockstep: the 32 / G rows of a warp advance together up to the longest one, so
//   the warp never splits (a split warp issues each row's instructions separately).
// - Order: a first pass (spmm_find_long) lists the rows of more than kLongRow
//   entries in half-octave length buckets; warps take those first, longest bucket
//   first, then chunks of 32 rows from a counter, so the long sequential chains start
//   at once and overlap the short rows instead of trailing at the end.  If a bucket
//   overflows, every row is taken in the second phase instead.
// - Pairing: the rows a warp runs together come from one length bucket (first phase)
//   or are neighbours after the warp sorts its 32-row chunk by length (second phase),
//   so the lockstep runs to a partner of about the same length.  On the power-law
//   generator at 1M rows this cuts the warp's steps from 13.1 M to 9.7 M (lanes busy
//   61 % -> 84 % of the steps on short rows, 71 % -> 94 % on long ones).
constexpr int kRing = 16;
constexpr int kLongRow = 256;
constexpr int kRowsPerGrab = 32;  // one row per lane, sorted by length

// Bucket of a long row (len > kLongRow): half-octaves, [257, 384) -> 0, [384, 512) -> 1,
// [512, 768) -> 2, ..., the last bucket open-ended.
__device__ __forceinline__ int long_bucket(int len) {
  const int lg = 31 - __clz(len);  // >= 8
  const int b = 2 * (lg - 8) + ((len >> (lg - 1)) & 1);
  return b < kSpmmLongBuckets - 1 ? b : kSpmmLongBuckets - 1;
}

// Ascending bitonic sort of one unsigned per lane across the warp.
__device__ __forceinline__ unsigned warp_sort_ascending(unsigned v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned o = __shfl_xor_sync(kFull, v, j);
      const bool keep_min = ((lane & j) == 0) == ((lane & k) == 0);
      v = keep_min ? (v < o ? v : o) : (v > o ? v : o);
    }
  }
  return v;
}
constexpr std::size_t kRingBytes = static_cast<std::size_t>(kRing) * kWarps * 32 * 16;

// The B gathers carry an L2 evict-last policy, so that L2 keeps the rows of B that
// later entries gather again ahead of the once-read CSR arrays and once-written C
// (1M power-law x 64: 0.632 -> 0.624 ms; also streaming the CSR arrays and C with
// evict-first hints made it slower, 0.677 ms).
__device__ __forceinline__ std::uint64_t l2_evict_last() {
  std::uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void cp_async16_keep(unsigned dst, const void* src,
                                                std::uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(dst),
               "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_wait_ring() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kRing - 1) : "memory");
}

__global__ void __launch_bounds__(256) spmm_find_long(const CsrView a, SpmmSched sc) {
  for (std::int64_t r = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       r < a.rows; r += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    const int s = clamp_off(a.row_offsets[r], a.base, a.nnz);
    const int e = clamp_off(a.row_offsets[r + 1], a.base, a.nnz);
    if (e - s > kLongRow) {
      const int b = long_bucket(e - s);
      const unsigned per = sc.long_cap / kSpmmLongBuckets;
      const unsigned i = atomicAdd(sc.counters + 2 + b, 1u);
      if (i < per) sc.long_rows[b * per + i] = static_cast<int>(r);
    }
  }
}

template <int G>
struct RingRows {
  static constexpr int RPW = 32 / G;
  static constexpr unsigned kSlotBytes = kWarps * 32 * 16;
  const CsrView& a;
  const DenseView& b;
  const DenseView& c;
  std::int64_t ncols;
  float alpha, beta;
  const float4* ring;  // this thread's slot 0
  unsigned mine;       // its shared-memory address
  int gl;
  std::uint64_t keep;  // L2 evict-last policy of the B gathers

  // G >= 16 lanes: the row's column indices and values come G at a time, one per
  // lane (coalesced), and are handed out by shuffles; the lookahead of kRing - 1
  // entries stays within the current and next chunk, the loop is unrolled by G so
  // every ring slot is a constant, and B offsets are 32-bit bytes (the launch checks
  // cols * ld * 4 < 2^32).
  __device__ void chunked(int s, int len, int steps, bool own, std::int64_t row) const {
    static_assert(G % kRing == 0 && G > kRing - 1, "two chunks cover the lookahead");
    const float* vals = static_cast<const float*>(a.values) + s;
    const int* cols = a.col_ind + s;
    const unsigned ldb = static_cast<unsigned>(b.ld) * 4u;
    const unsigned ncol = static_cast<unsigned>(a.cols);
    for (std::int64_t cb = 0; cb < ncols; cb += G * 4) {
      const std::int64_t col = cb + static_cast<std::int64_t>(gl) * 4;
      const bool live = own && col < ncols;
      const char* bcol = reinterpret_cast<const char*>(b.m + col);
      auto ldcol = [&](int i) { return i < len ? __ldg(cols + i) - a.base : -1; };
      int col_c = ldcol(gl), col_n = ldcol(G + gl);
      float val_c = gl < len ? __ldg(vals + gl) : 0.0f;
      auto issue = [&](int k, unsigned slot, bool on) {
        if (on && live && static_cast<unsigned>(k) < ncol)
          cp_async16_keep(mine + slot * kSlotBytes, bcol + static_cast<unsigned>(k) * ldb, keep);
        cp_commit();  // one group per entry (empty when nothing was copied)
      };
#pragma unroll
      for (int u = 0; u < kRing - 1; ++u)
        issue(__shfl_sync(kFull, col_c, u, G), static_cast<unsigned>(u), u < len);
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int j0 = 0; j0 < steps; j0 += G) {
#pragma unroll
        for (int u = 0; u < G; ++u) {
          if (j0 + u >= steps) break;  // warp-uniform
          constexpr int kAhead = kRing - 1;
          const int q = u + kAhead;  // entry j0 + q is issued now
          const int kq = q < G ? __shfl_sync(kFull, col_c, q % G, G)
                               : __shfl_sync(kFull, col_n, (q - G) % G, G);
          issue(kq, static_cast<unsigned>(q % kRing), j0 + q < len);
          const int ku = __shfl_sync(kFull, col_c, u, G);
          const float au = __shfl_sync(kFull, val_c, u, G);
          cp_wait_ring();  // entry j0 + u's copy has landed
          if (j0 + u < len && live && static_cast<unsigned>(ku) < ncol) {
            const float4 v = ring[(u % kRing) * (kWarps * 32)];
            acc.x = fmaf(au, v.x, acc.x);
            acc.y = fmaf(au, v.y, acc.y);
            acc.z = fmaf(au, v.z, acc.z);
            acc.w = fmaf(au, v.w, acc.w);
          }
        }
        col_c = col_n;
        col_n = ldcol(j0 + 2 * G + gl);
        val_c = j0 + G + gl < len ? __ldg(vals + j0 + G + gl) : 0.0f;
      }
      if (live) {
        float* out = c.m + row * c.ld + col;
        const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float prev = (beta == 0.0f) ? 0.0f : beta * out[i];
          out[i] = fmaf(alpha, v[i], prev);
        }
      }
    }
  }

  // Rows `row` of the warp's groups (-1: none); skip_long drops rows of more than
  // kLongRow entries (they were taken in the first phase).
  __device__ void run(std::int64_t row, bool skip_long) const {
    int s = 0, len = 0;
    bool own = row >= 0;
    if (own) {
      s = clamp_off(a.row_offsets[row], a.base, a.nnz);
      const int e = clamp_off(a.row_offsets[row + 1], a.base, a.nnz);
      len = e > s ? e - s : 0;
      if (skip_long && len > kLongRow) {
        own = false;
        len = 0;
      }
    }
    const int steps = static_cast<int>(__reduce_max_sync(kFull, static_cast<unsigned>(len)));
    if (__all_sync(kFull, !own)) return;
    if constexpr (G >= 16) {
      chunked(s, len, steps, own, row);
      return;
    }
    const float* vals = static_cast<const float*>(a.values);
    const int* cols = a.col_ind + s;
    for (std::int64_t cb = 0; cb < ncols; cb += G * 4) {
      const std::int64_t col = cb + static_cast<std::int64_t>(gl) * 4;
      const bool live = own && col < ncols;
      const float* bcol = b.m + col;
      unsigned valid = 0;
      int kpre = len > 0 ? __ldg(cols) - a.base : -1;
      auto issue = [&](int q) {
        const int k = kpre;
        kpre = q + 1 < len ? __ldg(cols + q + 1) - a.base : -1;
        const unsigned slot = static_cast<unsigned>(q) & (kRing - 1);
        if (q < len && live) {
          if (static_cast<unsigned>(k) < static_cast<unsigned long long>(a.cols)) {
            cp_async16_keep(mine + slot * kSlotBytes, bcol + static_cast<std::int64_t>(k) * b.ld,
                            keep);
            valid |= 1u << slot;
          } else {
            valid &= ~(1u << slot);
          }
        }
        cp_commit();  // one group per entry (empty past the row's end)
      };
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int q = 0; q < kRing - 1; ++q) issue(q);
      float vpre = len > 0 ? __ldg(vals + s) : 0.0f;
      for (int j = 0; j < steps; ++j) {
        issue(j + kRing - 1);
        const float av = vpre;
        vpre = j + 1 < len ? __ldg(vals + s + j + 1) : 0.0f;
        cp_wait_ring();  // entry j's copy has landed
        const unsigned slot = static_cast<unsigned>(j) & (kRing - 1);
        if (j < len && live && ((valid >> slot) & 1u)) {
          const float4 q = ring[slot * (kWarps * 32)];
          acc.x = fmaf(av, q.x, acc.x);
          acc.y = fmaf(av, q.y, acc.y);
          acc.z = fmaf(av, q.z, acc.z);
          acc.w = fmaf(av, q.w, acc.w);
        }
      }
      if (live) {
        float* out = c.m + row * c.ld + col;
        const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float prev = (beta == 0.0f) ? 0.0f : beta * out[i];
          out[i] = fmaf(alpha, v[i], prev);
        }
      }
    }
  }
};

template <int G>
__global__ void __launch_bounds__(kWarps * 32)
    spmm_rows_ring(const CsrView a, const DenseView b, const DenseView c, std::int64_t ncols,
                   float alpha, float beta, SpmmSched sc) {
  extern __shared__ float4 ring[];  // [kRing][kWarps * 32]
  constexpr int RPW = RingRows<G>::RPW;
  const int lane = threadIdx.x & 31;
  const int g = lane / G;
  const RingRows<G> rr{a, b, c, ncols, alpha, beta, ring + threadIdx.x,
                       static_cast<unsigned>(__cvta_generic_to_shared(ring + threadIdx.x)),
                       lane % G, l2_evict_last()};
  const unsigned per = sc.long_cap / kSpmmLongBuckets;
  unsigned cnt[kSpmmLongBuckets];
  unsigned nlong = 0;
  bool listed = true;
#pragma unroll
  for (int b = 0; b < kSpmmLongBuckets; ++b) {
    cnt[b] = sc.counters[2 + b];
    nlong += cnt[b];
    listed = listed && cnt[b] <= per;
  }
  if (listed) {
    for (;;) {
      unsigned i0 = 0;
      if (lane == 0) i0 = atomicAdd(sc.counters, static_cast<unsigned>(RPW));
      i0 = __shfl_sync(kFull, i0, 0);
      if (i0 >= nlong) break;
      // position i of the buckets laid end to end, longest bucket first
      unsigned rem = i0 + g;
      int row = -1;
#pragma unroll
      for (int b = kSpmmLongBuckets - 1; b >= 0; --b) {
        if (row < 0 && rem < cnt[b]) row = sc.long_rows[b * per + rem];
        if (row < 0) rem -= rem < cnt[b] ? 0u : cnt[b];
      }
      rr.run(row, false);
    }
  }
  for (;;) {
    unsigned ch = 0;
    if (lane == 0) ch = atomicAdd(sc.counters + 1, 1u);
    ch = __shfl_sync(kFull, ch, 0);
    const std::int64_t r0 = static_cast<std::int64_t>(ch) * kRowsPerGrab;
    if (r0 >= a.rows) break;
    // lane l's key: length (capped) << 6 | owned << 5 | l; rows past the end and, when
    // listed, the long rows are not owned and sort first
    unsigned key = static_cast<unsigned>(lane);
    if (r0 + lane < a.rows) {
      const std::int64_t row = r0 + lane;
      const int s0 = clamp_off(a.row_offsets[row], a.base, a.nnz);
      const int e0 = clamp_off(a.row_offsets[row + 1], a.base, a.nnz);
      const int len = e0 > s0 ? e0 - s0 : 0;
      if (!(listed && len > kLongRow))
        key = (static_cast<unsigned>(len < (1 << 25) ? len : (1 << 25) - 1) << 6) | 32u |
              static_cast<unsigned>(lane);
    }
    key = warp_sort_ascending(key);
#pragma unroll 1
    for (int p = 0; p < 32 / RPW; ++p) {
      const unsigned k = __shfl_sync(kFull, key, p * RPW + g);
      rr.run((k & 32u) ? r0 + static_cast<std::int64_t>(k & 31u) : -1, listed);
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}

// C = beta == 0 ? 0 : beta * C over out_rows x ncols.
__global__ void __launch_bounds__(256)
    spmm_scale(const DenseView c, std::int64_t out_rows, std::int64_t ncols, float beta) {
  const std::int64_t total = out_rows * ncols;
  for (std::int64_t i = blockIdx.x * static_cast<std::int64_t>(blockDim.x) + threadIdx.x;
       i < total; i += static_cast<std::int64_t>(gridDim.x) * blockDim.x) {
    // walk C in its storage order so that consecutive threads touch consecutive words
    const std::int64_t r = c.col_major ? i % out_rows : i / ncols;
    const std::int64_t col = c.col_major ? i / out_rows : i % ncols;
    float* p = c.m + dense_index<false>(c, r, col);
    *p = (beta == 0.0f) ? 0.0f : beta * *p;
  }
}

// Transposed A: warp per row r of A; every entry (k, a) adds alpha * a * B(r, col)
// into C(k, col).
template <bool BROW, bool CROW>
__global__ void __launch_bounds__(kWarps * 32)
    spmm_t_scatter(const CsrView a, const DenseView b, const DenseView c, std::int64_t ncols,
                   float alpha) {
  const int lane = threadIdx.x & 31;
  const float* vals = static_cast<const float*>(a.values);
  const std::int64_t warp0 = static_cast<std::int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const std::int64_t nwarps = static_cast<std::int64_t>(gridDim.x) * kWarps;
  for (std::int64_t row = warp0; row < a.rows; row += nwarps) {
    const int s = clamp_off(a.row_offsets[row], a.base, a.nnz);
    const int e0 = clamp_off(a.row_offsets[row + 1], a.base, a.nnz);
    const int e = e0 < s ? s : e0;
    if (e == s) continue;
    for (std::int64_t cb = 0; cb < ncols; cb += 32) {
      const std::int64_t col = cb + lane;
      const bool live = col < ncols;
      const float br = live ? alpha * __ldg(b.m + dense_index<BROW>(b, row, col)) : 0.0f;
      for (int k0 = s; k0 < e; k0 += 32) {
        int kk = -1;
        float vv = 0.0f;
        if (k0 + lane < e) {
          kk = __ldg(a.col_ind + k0 + lane) - a.base;
          vv = __ldg(vals + k0 + lane);
        }
        const int cnt = (e - k0 < 32) ? e - k0 : 32;
        for (int j = 0; j < cnt; ++j) {
          const int k = __shfl_sync(kFull, kk, j);
          const float av = __shfl_sync(kFull, vv, j);
          if (static_cast<unsigned>(k) < static_cast<unsigned long long>(a.cols) && live)
            atomicAdd(c.m + dense_index<CROW>(c, k, col), av * br);
        }
      }
    }
  }
}

template <int VEC, bool BROW, bool CROW>
cudaError_t spmm_rows_group(const CsrView& a, const DenseView& b, const DenseView& c,
                            std::int64_t ncols, float alpha, float beta, cudaStream_t st) {
  // lanes per row: enough for one pass over the columns, at least 4
  const std::int64_t lanes = (ncols + VEC - 1) / VEC;
  const int G = lanes > 16 ? 32 : (lanes > 8 ? 16 : (lanes > 4 ? 8 : 4));
  const unsigned grid = grid_for((a.rows + 32 / G - 1) / (32 / G), kWarps, 16);
  switch (G) {
    case 4: spmm_rows<VEC, 4, BROW, CROW><<<grid, kWarps * 32, 0, st>>>(a, b, c, ncols, alpha, beta); break;
    case 8: spmm_rows<VEC, 8, BROW, CROW><<<grid, kWarps * 32, 0, st>>>(a, b, c, ncols, alpha, beta); break;
    case 16: spmm_rows<VEC, 16, BROW, CROW><<<grid, kWarps * 32, 0, st>>>(a, b, c, ncols, alpha, beta); break;
    default: spmm_rows<VEC, 32, BROW, CROW><<<grid, kWarps * 32, 0, st>>>(a, b, c, ncols, alpha, beta); break;
  }
  return cudaGetLastError();
}

cudaError_t spmm_ring_launch(const CsrView& a, const DenseView& b, const DenseView& c,
                             std::int64_t ncols, float alpha, float beta, const SpmmSched& sc,
                             cudaStream_t st) {
  const std::int64_t lanes = (ncols + 3) / 4;
  const int G = lanes > 16 ? 32 : (lanes > 8 ? 16 : (lanes > 4 ? 8 : 4));
  // 32-bit byte offsets into B on the chunked (G >= 16) path
  if (G >= 16 && static_cast<double>(a.cols) * static_cast<double>(b.ld) * 4.0 >= 4294967296.0)
    return spmm_rows_group<4, true, true>(a, b, c, ncols, alpha, beta, st);
  cudaError_t e = cudaMemsetAsync(sc.counters, 0, (2 + kSpmmLongBuckets) * sizeof(unsigned), st);
  if (e != cudaSuccess) return e;
  spmm_find_long<<<grid_for(a.rows, 256, 8), 256, 0, st>>>(a, sc);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const unsigned grid = grid_for((a.rows + 32 / G - 1) / (32 / G), kWarps, 3);
  auto go = [&](auto kern) {
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kRingBytes));
    if (r != cudaSuccess) return r;
    kern<<<grid, kWarps * 32, kRingBytes, st>>>(a, b, c, ncols, alpha, beta, sc);
    return cudaGetLastError();
  };
  switch (G) {
    case 4: return go(spmm_rows_ring<4>);
    case 8: return go(spmm_rows_ring<8>);
    case 16: return go(spmm_rows_ring<16>);
    default: return go(spmm_rows_ring<32>);
  }
}

template <bool BROW, bool CROW>
cudaError_t spmm_rows_launch(const CsrView& a, const DenseView& b, const DenseView& c,
                             std::int64_t ncols, float alpha, float beta, bool vec4,
                             const SpmmSched* sc, cudaStream_t st) {
  if constexpr (BROW && CROW) {
    if (vec4 && sc != nullptr) return spmm_ring_launch(a, b, c, ncols, alpha, beta, *sc, st);
  }
  return spmm_rows_group<1, BROW, CROW>(a, b, c, ncols, alpha, beta, st);
}

bool row_contiguous(const DenseView& d) { return d.col_major == d.trans; }

}  // namespace

cudaError_t launch_spmm_csr(const CsrView& a, bool trans_a, const DenseView& b,
                            const DenseView& c, std::int64_t ncols, float alpha, float beta,
                            const SpmmSched* sched, cudaStream_t stream) noexcept {
  const std::int64_t out_rows = trans_a ? a.cols : a.rows;
  if (out_rows <= 0 || ncols <= 0) return cudaSuccess;
  const bool brow = row_contiguous(b);
  const bool crow = !c.col_major;
  DenseView bb = b, cc = c;
  if (brow) {  // normalise: B(r, col) = m[r * ld + col]
    bb.col_major = false;
    bb.trans = false;
  }
  cc.trans = false;
  if (!trans_a) {
    const bool vec4 = brow && crow && ncols % 4 == 0 && b.ld % 4 == 0 && c.ld % 4 == 0 &&
                      aligned_to(b.m, 16) && aligned_to(c.m, 16);
    if (brow && crow)
      return spmm_rows_launch<true, true>(a, bb, cc, ncols, alpha, beta, vec4, sched, stream);
    if (brow)
      return spmm_rows_launch<true, false>(a, bb, cc, ncols, alpha, beta, false, nullptr, stream);
    if (crow)
      return spmm_rows_launch<false, true>(a, bb, cc, ncols, alpha, beta, false, nullptr, stream);
    return spmm_rows_launch<false, false>(a, bb, cc, ncols, alpha, beta, false, nullptr, stream);
  }
  spmm_scale<<<grid_for(out_rows * ncols, 256, 8), 256, 0, stream>>>(cc, out_rows, ncols, beta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || a.rows <= 0) return e;
  const unsigned grid = grid_for(a.rows, kWarps, 16);
  if (brow && crow)
    spmm_t_scatter<true, true><<<grid, kWarps * 32, 0, stream>>>(a, bb, cc, ncols, alpha);
  else if (brow)
    spmm_t_scatter<true, false><<<grid, kWarps * 32, 0, stream>>>(a, bb, cc, ncols, alpha);
  else if (crow)
    spmm_t_scatter<false, true><<<grid, kWarps * 32, 0, stream>>>(a, bb, cc, ncols, alpha);
  else
    spmm_t_scatter<false, false><<<grid, kWarps * 32, 0, stream>>>(a, bb, cc, ncols, alpha);
  return cudaGetLastError();
}

cudaError_t launch_spmv_csr_t(const CsrView& a, Value t, const void* x, void* y, float alpha,
                              float beta, float* scratch, cudaStream_t stream) noexcept {
  if (a.cols <= 0) return cudaSuccess;
  if (t == Value::kF16) {
    if (scratch == nullptr) return cudaErrorInvalidValue;
    return spmv_t_typed<__half>(a, x, y, alpha, beta, scratch, stream);
  }
  return spmv_t_typed<float>(a, x, y, alpha, beta, nullptr, stream);
}

}  // namespace mb200::sparse
