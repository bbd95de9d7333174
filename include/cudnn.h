/*
 * cudnn.h — C ABI of the B200-native convolution-forward and softmax-forward.
 *
 * Drop-in for the MUDA cuDNN shim's hot path: names, argument lists and numeric
 * enum values follow libraries/dnn/include/cudnn.h of the reference (enums
 * cudnn.h:25-128, declarations cudnn.h:150-276).  Enums are int-width.
 * CUDNN_DATA_BFLOAT16 (= 9, NVIDIA's value) is an extension the reference lacks:
 * the reference convolution is fp32-only (cudnn_ops.mm:134-137).
 *
 * Conventions kept from the reference (libraries/dnn/src/cudnn_ops.mm):
 *   - alpha and beta are host float* (cudnn_ops.mm:140-141); beta == 0 means y is not read;
 *   - the convolution workspace is 0 bytes and the algo argument is advisory;
 *   - a KRSC filter is declared with format CUDNN_TENSOR_NHWC, a KCRS filter with NCHW.
 */
#ifndef MUDA_B200_CUDNN_H_
#define MUDA_B200_CUDNN_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CUDNN_MAJOR 8
#define CUDNN_MINOR 9
#define CUDNN_PATCHLEVEL 0
#define CUDNN_VERSION (CUDNN_MAJOR * 1000 + CUDNN_MINOR * 100 + CUDNN_PATCHLEVEL)

typedef enum {
  CUDNN_STATUS_SUCCESS = 0,
  CUDNN_STATUS_NOT_INITIALIZED = 1,
  CUDNN_STATUS_ALLOC_FAILED = 2,
  CUDNN_STATUS_BAD_PARAM = 3,
  CUDNN_STATUS_INTERNAL_ERROR = 4,
  CUDNN_STATUS_INVALID_VALUE = 5,
  CUDNN_STATUS_ARCH_MISMATCH = 6,
  CUDNN_STATUS_MAPPING_ERROR = 7,
  CUDNN_STATUS_EXECUTION_FAILED = 8,
  CUDNN_STATUS_NOT_SUPPORTED = 9
} cudnnStatus_t;

typedef enum {
  CUDNN_DATA_FLOAT = 0,
  CUDNN_DATA_DOUBLE = 1,
  CUDNN_DATA_HALF = 2,
  CUDNN_DATA_INT8 = 3,
  CUDNN_DATA_INT32 = 4,
  CUDNN_DATA_BFLOAT16 = 9 /* extension: not in the reference enum */
} cudnnDataType_t;

typedef enum { CUDNN_TENSOR_NCHW = 0, CUDNN_TENSOR_NHWC = 1 } cudnnTensorFormat_t;

typedef enum { CUDNN_CONVOLUTION = 0, CUDNN_CROSS_CORRELATION = 1 } cudnnConvolutionMode_t;

typedef enum {
  CUDNN_CONVOLUTION_FWD_ALGO_IMPLICIT_GEMM = 0,
  CUDNN_CONVOLUTION_FWD_ALGO_IMPLICIT_PRECOMP_GEMM = 1,
  CUDNN_CONVOLUTION_FWD_ALGO_GEMM = 2,
  CUDNN_CONVOLUTION_FWD_ALGO_DIRECT = 3
} cudnnConvolutionFwdAlgo_t;

typedef enum {
  CUDNN_SOFTMAX_FAST = 0,
  CUDNN_SOFTMAX_ACCURATE = 1,
  CUDNN_SOFTMAX_LOG = 2
} cudnnSoftmaxAlgorithm_t;

typedef enum { CUDNN_SOFTMAX_MODE_INSTANCE = 0, CUDNN_SOFTMAX_MODE_CHANNEL = 1 } cudnnSoftmaxMode_t;

/* reference cudnn.h:72-136 */
typedef enum {
  CUDNN_CONVOLUTION_BWD_DATA_ALGO_0 = 0,
  CUDNN_CONVOLUTION_BWD_DATA_ALGO_1 = 1
} cudnnConvolutionBwdDataAlgo_t;

typedef enum {
  CUDNN_CONVOLUTION_BWD_FILTER_ALGO_0 = 0,
  CUDNN_CONVOLUTION_BWD_FILTER_ALGO_1 = 1
} cudnnConvolutionBwdFilterAlgo_t;

typedef enum {
  CUDNN_ACTIVATION_SIGMOID = 0,
  CUDNN_ACTIVATION_RELU = 1,
  CUDNN_ACTIVATION_TANH = 2,
  CUDNN_ACTIVATION_CLIPPED_RELU = 3,
  CUDNN_ACTIVATION_ELU = 4,
  CUDNN_ACTIVATION_IDENTITY = 5,
  CUDNN_ACTIVATION_SWISH = 6
} cudnnActivationMode_t;

typedef enum { CUDNN_NOT_PROPAGATE_NAN = 0, CUDNN_PROPAGATE_NAN = 1 } cudnnNanPropagation_t;

typedef enum {
  CUDNN_POOLING_MAX = 0,
  CUDNN_POOLING_AVERAGE_COUNT_INCLUDE_PADDING = 1,
  CUDNN_POOLING_AVERAGE_COUNT_EXCLUDE_PADDING = 2,
  CUDNN_POOLING_MAX_DETERMINISTIC = 3
} cudnnPoolingMode_t;

typedef enum {
  CUDNN_BATCHNORM_PER_ACTIVATION = 0,
  CUDNN_BATCHNORM_SPATIAL = 1,
  CUDNN_BATCHNORM_SPATIAL_PERSISTENT = 2
} cudnnBatchNormMode_t;

struct cudnnContext;
struct cudnnTensorStruct;
struct cudnnFilterStruct;
struct cudnnConvolutionStruct;
struct cudnnActivationStruct;
struct cudnnPoolingStruct;
typedef struct cudnnActivationStruct* cudnnActivationDescriptor_t;
typedef struct cudnnPoolingStruct* cudnnPoolingDescriptor_t;
typedef struct cudnnContext* cudnnHandle_t;
typedef struct cudnnTensorStruct* cudnnTensorDescriptor_t;
typedef struct cudnnFilterStruct* cudnnFilterDescriptor_t;
typedef struct cudnnConvolutionStruct* cudnnConvolutionDescriptor_t;

/* Context — reference cudnn_descriptors.mm:46-128 */
size_t cudnnGetVersion(void);
const char* cudnnGetErrorString(cudnnStatus_t status);
cudnnStatus_t cudnnCreate(cudnnHandle_t* handle);
cudnnStatus_t cudnnDestroy(cudnnHandle_t handle);
cudnnStatus_t cudnnSetStream(cudnnHandle_t handle, cudaStream_t streamId);
cudnnStatus_t cudnnGetStream(cudnnHandle_t handle, cudaStream_t* streamId);

/* Tensor descriptors — reference cudnn_descriptors.mm:130-231 */
cudnnStatus_t cudnnCreateTensorDescriptor(cudnnTensorDescriptor_t* tensorDesc);
cudnnStatus_t cudnnSetTensor4dDescriptor(cudnnTensorDescriptor_t tensorDesc,
                                         cudnnTensorFormat_t format, cudnnDataType_t dataType,
                                         int n, int c, int h, int w);
cudnnStatus_t cudnnSetTensor4dDescriptorEx(cudnnTensorDescriptor_t tensorDesc,
                                           cudnnDataType_t dataType, int n, int c, int h, int w,
                                           int nStride, int cStride, int hStride, int wStride);
cudnnStatus_t cudnnGetTensor4dDescriptor(cudnnTensorDescriptor_t tensorDesc,
                                         cudnnDataType_t* dataType, int* n, int* c, int* h, int* w,
                                         int* nStride, int* cStride, int* hStride, int* wStride);
cudnnStatus_t cudnnDestroyTensorDescriptor(cudnnTensorDescriptor_t tensorDesc);

/* Filter descriptors — reference cudnn_descriptors.mm:233-290 */
cudnnStatus_t cudnnCreateFilterDescriptor(cudnnFilterDescriptor_t* filterDesc);
cudnnStatus_t cudnnSetFilter4dDescriptor(cudnnFilterDescriptor_t filterDesc,
                                         cudnnDataType_t dataType, cudnnTensorFormat_t format,
                                         int k, int c, int h, int w);
cudnnStatus_t cudnnGetFilter4dDescriptor(cudnnFilterDescriptor_t filterDesc,
                                         cudnnDataType_t* dataType, cudnnTensorFormat_t* format,
                                         int* k, int* c, int* h, int* w);
cudnnStatus_t cudnnDestroyFilterDescriptor(cudnnFilterDescriptor_t filterDesc);

/* Convolution descriptors — reference cudnn_descriptors.mm:292-385 */
cudnnStatus_t cudnnCreateConvolutionDescriptor(cudnnConvolutionDescriptor_t* convDesc);
cudnnStatus_t cudnnSetConvolution2dDescriptor(cudnnConvolutionDescriptor_t convDesc, int pad_h,
                                              int pad_w, int u, int v, int dilation_h,
                                              int dilation_w, cudnnConvolutionMode_t mode,
                                              cudnnDataType_t computeType);
cudnnStatus_t cudnnSetConvolutionGroupCount(cudnnConvolutionDescriptor_t convDesc, int groupCount);
cudnnStatus_t cudnnGetConvolutionGroupCount(cudnnConvolutionDescriptor_t convDesc, int* groupCount);
cudnnStatus_t cudnnGetConvolution2dForwardOutputDim(cudnnConvolutionDescriptor_t convDesc,
                                                    cudnnTensorDescriptor_t inputTensorDesc,
                                                    cudnnFilterDescriptor_t filterDesc, int* n,
                                                    int* c, int* h, int* w);
cudnnStatus_t cudnnDestroyConvolutionDescriptor(cudnnConvolutionDescriptor_t convDesc);

/* Activation and pooling descriptors — reference cudnn_descriptors.mm:382-484 */
cudnnStatus_t cudnnCreateActivationDescriptor(cudnnActivationDescriptor_t* activationDesc);
cudnnStatus_t cudnnSetActivationDescriptor(cudnnActivationDescriptor_t activationDesc,
                                           cudnnActivationMode_t mode,
                                           cudnnNanPropagation_t reluNanOpt, double coef);
cudnnStatus_t cudnnGetActivationDescriptor(cudnnActivationDescriptor_t activationDesc,
                                           cudnnActivationMode_t* mode,
                                           cudnnNanPropagation_t* reluNanOpt, double* coef);
cudnnStatus_t cudnnDestroyActivationDescriptor(cudnnActivationDescriptor_t activationDesc);
cudnnStatus_t cudnnCreatePoolingDescriptor(cudnnPoolingDescriptor_t* poolingDesc);
cudnnStatus_t cudnnSetPooling2dDescriptor(cudnnPoolingDescriptor_t poolingDesc,
                                          cudnnPoolingMode_t mode,
                                          cudnnNanPropagation_t maxpoolingNanOpt, int windowHeight,
                                          int windowWidth, int verticalPadding,
                                          int horizontalPadding, int verticalStride,
                                          int horizontalStride);
cudnnStatus_t cudnnGetPooling2dForwardOutputDim(cudnnPoolingDescriptor_t poolingDesc,
                                                cudnnTensorDescriptor_t inputTensorDesc, int* n,
                                                int* c, int* h, int* w);
cudnnStatus_t cudnnDestroyPoolingDescriptor(cudnnPoolingDescriptor_t poolingDesc);
/* reference cudnn_descriptors.mm:486-500 */
cudnnStatus_t cudnnDeriveBNTensorDescriptor(cudnnTensorDescriptor_t derivedBnDesc,
                                            cudnnTensorDescriptor_t xDesc,
                                            cudnnBatchNormMode_t mode);

/* Operations — reference cudnn_ops.mm:89-193 (conv) and cudnn_ops.mm:625-720 (softmax) */
cudnnStatus_t cudnnGetConvolutionForwardWorkspaceSize(
    cudnnHandle_t handle, cudnnTensorDescriptor_t xDesc, cudnnFilterDescriptor_t wDesc,
    cudnnConvolutionDescriptor_t convDesc, cudnnTensorDescriptor_t yDesc,
    cudnnConvolutionFwdAlgo_t algo, size_t* sizeInBytes);
cudnnStatus_t cudnnConvolutionForward(cudnnHandle_t handle, const void* alpha,
                                      cudnnTensorDescriptor_t xDesc, const void* x,
                                      cudnnFilterDescriptor_t wDesc, const void* w,
                                      cudnnConvolutionDescriptor_t convDesc,
                                      cudnnConvolutionFwdAlgo_t algo, void* workSpace,
                                      size_t workSpaceSizeInBytes, const void* beta,
                                      cudnnTensorDescriptor_t yDesc, void* y);
cudnnStatus_t cudnnSoftmaxForward(cudnnHandle_t handle, cudnnSoftmaxAlgorithm_t algo,
                                  cudnnSoftmaxMode_t mode, const void* alpha,
                                  cudnnTensorDescriptor_t xDesc, const void* x, const void* beta,
                                  cudnnTensorDescriptor_t yDesc, void* y);

/* Neighbours of the convolution, fp32 — reference cudnn_ops.mm:195-624, 722-902.
 * Backward data, AddTensor, ReLU / clipped ReLU / identity and pooling give the
 * reference's per-output arithmetic exactly; the reductions (backward filter and
 * bias, batch-norm training statistics) are deterministic but summed in a
 * different order than the reference's single sequential loop.  The algo and
 * workspace arguments of the backward calls are ignored: the backward filter's
 * partial sums live in the handle's workspace. */
cudnnStatus_t cudnnConvolutionBackwardData(cudnnHandle_t handle, const void* alpha,
                                           cudnnFilterDescriptor_t wDesc, const void* w,
                                           cudnnTensorDescriptor_t dyDesc, const void* dy,
                                           cudnnConvolutionDescriptor_t convDesc,
                                           cudnnConvolutionBwdDataAlgo_t algo, void* workSpace,
                                           size_t workSpaceSizeInBytes, const void* beta,
                                           cudnnTensorDescriptor_t dxDesc, void* dx);
cudnnStatus_t cudnnConvolutionBackwardFilter(cudnnHandle_t handle, const void* alpha,
                                             cudnnTensorDescriptor_t xDesc, const void* x,
                                             cudnnTensorDescriptor_t dyDesc, const void* dy,
                                             cudnnConvolutionDescriptor_t convDesc,
                                             cudnnConvolutionBwdFilterAlgo_t algo, void* workSpace,
                                             size_t workSpaceSizeInBytes, const void* beta,
                                             cudnnFilterDescriptor_t dwDesc, void* dw);
cudnnStatus_t cudnnConvolutionBackwardBias(cudnnHandle_t handle, const void* alpha,
                                           cudnnTensorDescriptor_t dyDesc, const void* dy,
                                           const void* beta, cudnnTensorDescriptor_t dbDesc,
                                           void* db);
cudnnStatus_t cudnnAddTensor(cudnnHandle_t handle, const void* alpha, cudnnTensorDescriptor_t aDesc,
                             const void* A, const void* beta, cudnnTensorDescriptor_t cDesc,
                             void* C);
cudnnStatus_t cudnnActivationForward(cudnnHandle_t handle,
                                     cudnnActivationDescriptor_t activationDesc, const void* alpha,
                                     cudnnTensorDescriptor_t xDesc, const void* x, const void* beta,
                                     cudnnTensorDescriptor_t yDesc, void* y);
cudnnStatus_t cudnnPoolingForward(cudnnHandle_t handle, cudnnPoolingDescriptor_t poolingDesc,
                                  const void* alpha, cudnnTensorDescriptor_t xDesc, const void* x,
                                  const void* beta, cudnnTensorDescriptor_t yDesc, void* y);
cudnnStatus_t cudnnBatchNormalizationForwardInference(
    cudnnHandle_t handle, cudnnBatchNormMode_t mode, const void* alpha, const void* beta,
    cudnnTensorDescriptor_t xDesc, const void* x, cudnnTensorDescriptor_t yDesc, void* y,
    cudnnTensorDescriptor_t bnScaleBiasMeanVarDesc, const void* bnScale, const void* bnBias,
    const void* estimatedMean, const void* estimatedVariance, double epsilon);
cudnnStatus_t cudnnBatchNormalizationForwardTraining(
    cudnnHandle_t handle, cudnnBatchNormMode_t mode, const void* alpha, const void* beta,
    cudnnTensorDescriptor_t xDesc, const void* x, cudnnTensorDescriptor_t yDesc, void* y,
    cudnnTensorDescriptor_t bnScaleBiasMeanVarDesc, const void* bnScale, const void* bnBias,
    double exponentialAverageFactor, void* resultRunningMean, void* resultRunningVariance,
    double epsilon, void* resultSaveMean, void* resultSaveInvVariance);

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_CUDNN_H_ */
