// dnn.hpp — launch interface of the convolution and softmax kernels.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

namespace mb200::dnn {

// Element-strided 4-D view (n, c, h, w) — the reference's tensor descriptor
// strides (libraries/dnn/src/cudnn_descriptors.hpp:19-43).
struct View4 {
  int n, c, h, w;
  std::int64_t ns, cs, hs, ws;
};

enum class SoftmaxAlgo : int { kFast = 0, kAccurate = 1, kLog = 2 };

// Softmax over rows of `len` contiguous floats, rows `len` apart:
// y = alpha * softmax(x) + beta * y (beta == 0: y is not read).
cudaError_t launch_softmax_rows(const float* x, float* y, std::int64_t rows, std::int64_t len,
                                SoftmaxAlgo algo, float alpha, float beta,
                                cudaStream_t stream) noexcept;

// Softmax over the channel axis of an arbitrary strided tensor (one reduction per
// (n, h, w) position), or over whole (c, h, w) instances when `instance` is true.
cudaError_t launch_softmax_strided(const float* x, const View4& xv, float* y, const View4& yv,
                                   bool instance, SoftmaxAlgo algo, float alpha, float beta,
                                   cudaStream_t stream) noexcept;

// Convolution geometry shared by every conv kernel; mirrors the parameter block
// the reference packs in BuildConvParams (libraries/dnn/src/cudnn_ops.mm:26-83).
struct ConvShape {
  View4 x;        // input  (n, c_in, h_in, w_in)
  View4 y;        // output (n, c_out, h_out, w_out)
  int kh, kw;     // filter spatial size
  int pad_h, pad_w, stride_h, stride_w, dil_h, dil_w;
  int groups;
  bool filter_krsc;   // true: filter laid out (k, r, s, c) — NHWC; false: (k, c, r, s)
  bool convolution;   // true: CUDNN_CONVOLUTION (filter flipped); false: cross-correlation
};

enum class ConvDtype : int { kF32 = 0, kBF16 = 1 };

// Direct convolution, any geometry: one thread per output element, fp32 accumulate.
cudaError_t launch_conv_direct(const void* x, const void* w, void* y, const ConvShape& s,
                               ConvDtype dt, float alpha, float beta, cudaStream_t stream) noexcept;

// tcgen05 implicit-GEMM kernel: 16-bit NHWC input/output, KRSC filter, groups 1,
// stride 1, C a multiple of 64.  cudaErrorNotSupported for other geometries.
bool conv_tc_supported(const ConvShape& s, ConvDtype dt, const void* x, const void* w,
                       const void* y) noexcept;
cudaError_t launch_conv_tc(const void* x, const void* w, void* y, const ConvShape& s,
                           ConvDtype dt, float alpha, float beta, cudaStream_t stream) noexcept;

// tcgen05 implicit-GEMM kernel for fp32 tensors in split-tf32 form: NHWC input and
// output, KRSC or KCRS filter, groups 1, stride 1, C a multiple of 32, K of 4.
// Needs conv_tf32x3_workspace(s) bytes of device workspace (16-byte aligned) that
// no other stream touches during the call (0: geometry not covered).
std::size_t conv_tf32x3_workspace(const ConvShape& s) noexcept;
cudaError_t launch_conv_tf32x3(const void* x, const void* w, void* y, const ConvShape& s,
                               float alpha, float beta, void* workspace, std::size_t ws_bytes,
                               cudaStream_t stream) noexcept;

// Picks the fastest kernel that supports the geometry and launches it; fp32
// tensors use the tensor cores when `workspace` holds conv_tf32x3_workspace(s)
// bytes, else the direct kernel.
cudaError_t launch_conv(const void* x, const void* w, void* y, const ConvShape& s, ConvDtype dt,
                        float alpha, float beta, void* workspace, std::size_t ws_bytes,
                        cudaStream_t stream) noexcept;

// Name of the kernel family launch_conv would use (for tests and benchmarks).
const char* conv_path_name(const ConvShape& s, ConvDtype dt) noexcept;

// ---- neighbours of the convolution (fp32; dnn_ops_kernels.cu) ----
// Backward data: dx = alpha * conv^T(dy, w) + beta * dx, with s.x the dx view and
// s.y the dy view.
cudaError_t launch_conv_bwd_data(const float* w, const float* dy, float* dx, const ConvShape& s,
                                 float alpha, float beta, cudaStream_t stream) noexcept;
// Backward filter: dw = alpha * sum_(b,p,q) x * dy + beta * dw, through
// conv_bwd_filter_workspace(s) bytes of device workspace (4-byte aligned).
std::size_t conv_bwd_filter_workspace(const ConvShape& s) noexcept;
int conv_bwd_filter_chunks(const ConvShape& s) noexcept;
cudaError_t launch_conv_bwd_filter(const float* x, const float* dy, float* dw, const ConvShape& s,
                                   float alpha, float beta, float* workspace,
                                   cudaStream_t stream) noexcept;
// Tensor-core forms (split tf32, groups 1; conv_bwd_tc.cu): backward data for
// stride 1 with NHWC dx / dy as a forward convolution of dy with the transposed
// filter; backward filter as an im2col GEMM.  Workspace 0: geometry not covered.
std::size_t conv_bwd_data_tc_workspace(const ConvShape& s) noexcept;
cudaError_t launch_conv_bwd_data_tc(const float* w, const float* dy, float* dx,
                                    const ConvShape& s, float alpha, float beta, void* workspace,
                                    std::size_t ws_bytes, cudaStream_t stream) noexcept;
std::size_t conv_bwd_filter_tc_workspace(const ConvShape& s) noexcept;
cudaError_t launch_conv_bwd_filter_tc(const float* x, const float* dy, float* dw,
                                      const ConvShape& s, float alpha, float beta,
                                      void* workspace, std::size_t ws_bytes,
                                      cudaStream_t stream) noexcept;
// Backward bias: db[c] = alpha * sum over (n, h, w) of dy + beta * db[c].
cudaError_t launch_conv_bwd_bias(const float* dy, const View4& v, float* db, float alpha,
                                 float beta, cudaStream_t stream) noexcept;
// c = alpha * a + beta * c, a broadcast along its size-1 dimensions.
cudaError_t launch_add_tensor(const float* a, const View4& av, float* c, const View4& cv,
                              float alpha, float beta, cudaStream_t stream) noexcept;
// y = alpha * act(x) + beta * y; mode = cudnnActivationMode_t.
cudaError_t launch_activation(const float* x, const View4& xv, float* y, const View4& yv,
                              int mode, float coef, float alpha, float beta,
                              cudaStream_t stream) noexcept;

struct PoolShape {
  View4 x, y;
  int win_h, win_w, pad_h, pad_w, stride_h, stride_w;
  int mode;  // cudnnPoolingMode_t
};
cudaError_t launch_pooling(const float* x, float* y, const PoolShape& p, float alpha, float beta,
                           cudaStream_t stream) noexcept;

cudaError_t launch_bn_inference(const float* x, const View4& xv, float* y, const View4& yv,
                                const float* scale, const float* bias, const float* mean,
                                const float* var, bool per_activation, float eps, float alpha,
                                float beta, cudaStream_t stream) noexcept;
// running_* and save_* may be null (skipped).  With bn_training_workspace(xv) > 0
// bytes of workspace each channel is split across several CTAs (three launches);
// a null workspace runs one CTA per channel.
std::size_t bn_training_workspace(const View4& xv) noexcept;
cudaError_t launch_bn_training(const float* x, const View4& xv, float* y, const View4& yv,
                               const float* scale, const float* bias, float* running_mean,
                               float* running_var, float* save_mean, float* save_inv_var,
                               float factor, float eps, float alpha, float beta, float* workspace,
                               cudaStream_t stream) noexcept;

}  // namespace mb200::dnn
