// gemm_tc_kernels.cu — tcgen05 tensor-core GEMM for 16-bit operands.
#include "blas/gemm.hpp"

namespace mb200::blas {

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t stream) noexcept {
  (void)g;
  (void)stream;
  return cudaErrorNotSupported;
}

const char* gemm_path_name(const GemmArgs& g) noexcept {
  (void)g;
  return "simt";
}

}  // namespace mb200::blas
