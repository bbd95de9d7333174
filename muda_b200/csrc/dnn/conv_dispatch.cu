// conv_dispatch.cu — selects the convolution kernel for a geometry.
//
// The reference picks its implicit-GEMM kernel for ungrouped KCRS filters and its
// direct kernel otherwise (libraries/dnn/src/cudnn_ops.mm:172-192).  Here the
// tcgen05 implicit GEMM serves bf16 NHWC tensors with KRSC filters and, in
// split-tf32 form, fp32 NHWC tensors with KRSC or KCRS filters (the layouts of the
// benchmark configuration); every other geometry runs the direct kernel.
#include "dnn/dnn.hpp"

namespace mb200::dnn {

const char* conv_path_name(const ConvShape& s, ConvDtype dt) noexcept {
  if (conv_tc_supported(s, dt, nullptr, nullptr, nullptr)) return "tcgen05";
  if (dt == ConvDtype::kF32 && conv_tf32x3_workspace(s) != 0) return "tcgen05-tf32x3";
  return "direct";
}

cudaError_t launch_conv(const void* x, const void* w, void* y, const ConvShape& s, ConvDtype dt,
                        float alpha, float beta, void* workspace, std::size_t ws_bytes,
                        cudaStream_t stream) noexcept {
  if (conv_tc_supported(s, dt, x, w, y)) {
    const cudaError_t e = launch_conv_tc(x, w, y, s, dt, alpha, beta, stream);
    if (e != cudaErrorNotSupported) return e;
    (void)cudaGetLastError();
  }
  if (dt == ConvDtype::kF32 && workspace != nullptr) {
    const cudaError_t e =
        launch_conv_tf32x3(x, w, y, s, alpha, beta, workspace, ws_bytes, stream);
    if (e != cudaErrorNotSupported) return e;
    (void)cudaGetLastError();
  }
  return launch_conv_direct(x, w, y, s, dt, alpha, beta, stream);
}

}  // namespace mb200::dnn
