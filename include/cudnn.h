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

struct cudnnContext;
struct cudnnTensorStruct;
struct cudnnFilterStruct;
struct cudnnConvolutionStruct;
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

#ifdef __cplusplus
}
#endif

#endif /* MUDA_B200_CUDNN_H_ */
