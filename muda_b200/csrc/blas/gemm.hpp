// gemm.hpp — launch interface of the GEMM kernels (column-major, cuBLAS semantics).
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

namespace mb200::blas {

enum class Elem : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// C = alpha * op(A) * op(B) + beta * C for `batch` matrices, column-major.
// alpha/beta are taken from *alpha_dev / *beta_dev when those are non-null
// (device pointer mode), else from alpha / beta.  beta == 0 means C is not read.
struct GemmArgs {
  Elem type;             // A, B and C element type
  bool trans_a, trans_b; // op = transpose (CUBLAS_OP_T and CUBLAS_OP_C are the same for reals)
  int m, n, k;
  const void* a;
  std::int64_t lda, stride_a;
  const void* b;
  std::int64_t ldb, stride_b;
  void* c;
  std::int64_t ldc, stride_c;
  int batch;
  float alpha, beta;
  const float* alpha_dev;
  const float* beta_dev;
};

// Register-blocked FFMA kernel: any type, transposes, leading dimensions and
// strides (fp32 accumulate).  The fp32 path of cublasSgemm.
cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t stream) noexcept;
// The same kernel with K split across CTAs for batch-1 problems whose tiles cannot fill
// the GPU: raw per-split sums in `workspace` (gemm_simt_workspace(g) bytes, 0 when no
// split is used), added in split order by one more pass (deterministic).  Without
// enough workspace it runs launch_gemm_simt.
std::size_t gemm_simt_workspace(const GemmArgs& g) noexcept;
cudaError_t launch_gemm_simt_split(const GemmArgs& g, void* workspace, std::size_t ws_bytes,
                                   cudaStream_t stream) noexcept;

// tcgen05 tensor-core kernel for 16-bit A/B (bf16 or fp16) with fp32 accumulation
// in tensor memory.  Returns cudaErrorNotSupported when the shape or layout is not
// covered (the caller then uses launch_gemm_simt).
cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t stream) noexcept;

// fp32 GEMM on the tensor cores in split-tf32 form (hi/lo tf32 planes, three
// MMAs per K step, within 1.5 * 2^-20 relative per product).  Needs a device
// workspace of gemm_tf32x3_workspace(g) bytes (16-byte aligned) that no other
// stream touches while the call runs; returns 0 bytes / cudaErrorNotSupported
// when the problem is too small or the workspace would exceed 2 GiB per batch
// entry (the caller then uses launch_gemm_simt).
std::size_t gemm_tf32x3_workspace(const GemmArgs& g) noexcept;
cudaError_t launch_gemm_tf32x3(const GemmArgs& g, void* workspace, std::size_t ws_bytes,
                               cudaStream_t stream) noexcept;

// The same with op(A) already split by the caller: a_planes holds the hi plane and
// then the lo plane of op(A), each m rows of tf32_plane_ldk(k) floats, element (i, p)
// of op(A) at a_planes[i * ldk + p] (k contiguous; the padding columns are not read).
// g.a / g.lda / g.trans_a are ignored; batch 1.  Only B is split, into the workspace.
std::size_t gemm_tf32x3_aplanes_workspace(const GemmArgs& g) noexcept;
cudaError_t launch_gemm_tf32x3_aplanes(const GemmArgs& g, const float* a_planes, void* workspace,
                                       std::size_t ws_bytes, cudaStream_t stream) noexcept;
inline std::int64_t tf32_plane_ldk(std::int64_t k) { return (k + 3) / 4 * 4; }

// Name of the kernel family that would serve `g` (for tests and benchmarks).
const char* gemm_path_name(const GemmArgs& g) noexcept;

}  // namespace mb200::blas
