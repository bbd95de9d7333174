"""ctypes bindings of the five C-ABI libraries (libmuda_<name>.so).

These mirror the reference's own Python ABI tests, which drive the library
shims through ctypes (tests/python/test_cuda_libraries_abi.py:55-303): the same
entry points, argument types and integer status codes.  Pointers are passed as
plain integers (e.g. ``tensor.data_ptr()``) and streams as raw ``cudaStream_t``
values (e.g. ``torch.cuda.current_stream().cuda_stream``).

Loading fails loudly when a library has not been built: there is no fallback.
"""

from __future__ import annotations

import ctypes as C
from functools import lru_cache

from muda_b200.build import lib_path

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
u64 = C.c_uint64
sz = C.c_size_t
f32 = C.c_float
P = C.POINTER


class LibraryMissing(RuntimeError):
    pass


def _load(name: str) -> C.CDLL:
    path = lib_path(name)
    if not path.exists():
        raise LibraryMissing(f"{path} is not built; run `python -m muda_b200.build`")
    return C.CDLL(str(path))


def _declare(lib: C.CDLL, protos: dict[str, tuple[list, object]]) -> C.CDLL:
    for name, (argtypes, restype) in protos.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


# ------------------------------------------------------------------ cuRAND --
CURAND_STATUS_SUCCESS = 0
CURAND_STATUS_NOT_INITIALIZED = 101
CURAND_STATUS_ALLOCATION_FAILED = 102
CURAND_STATUS_INVALID_VALUE = 104
CURAND_STATUS_LAUNCH_FAILURE = 201
CURAND_RNG_PSEUDO_DEFAULT = 100
CURAND_RNG_PSEUDO_PHILOX4_32_10 = 161

CURAND_PROTOS = {
    "curandCreateGenerator": ([P(vp), i32], i32),
    "curandCreateGeneratorHost": ([P(vp), i32], i32),
    "curandDestroyGenerator": ([vp], i32),
    "curandSetStream": ([vp, vp], i32),
    "curandGetStream": ([vp, P(vp)], i32),
    "curandSetPseudoRandomGeneratorSeed": ([vp, C.c_ulonglong], i32),
    "curandSetGeneratorOffset": ([vp, C.c_ulonglong], i32),
    "curandSetGeneratorOrdering": ([vp, i32], i32),
    "curandGetVersion": ([P(i32)], i32),
    "curandGetProperty": ([i32, P(i32)], i32),
    "curandGenerate": ([vp, vp, sz], i32),
    "curandGenerateUniform": ([vp, vp, sz], i32),
    "curandGenerateNormal": ([vp, vp, sz, f32, f32], i32),
    "curandGenerateLogNormal": ([vp, vp, sz, f32, f32], i32),
    "curandGenerateUniformDouble": ([vp, vp, sz], i32),
    "curandGenerateNormalDouble": ([vp, vp, sz, C.c_double, C.c_double], i32),
    "curandGenerateLogNormalDouble": ([vp, vp, sz, C.c_double, C.c_double], i32),
    "curandGeneratePoisson": ([vp, vp, sz, C.c_double], i32),
    "curandSetQuasiRandomGeneratorDimensions": ([vp, C.c_uint], i32),
    "curandGetDirectionVectors32": ([P(vp), i32], i32),
    "curandGetScrambleConstants32": ([P(vp)], i32),
}


@lru_cache(maxsize=None)
def curand() -> C.CDLL:
    return _declare(_load("curand"), CURAND_PROTOS)


# ------------------------------------------------------------------- cuDNN --
CUDNN_STATUS_SUCCESS = 0
CUDNN_STATUS_BAD_PARAM = 3
CUDNN_STATUS_EXECUTION_FAILED = 8
CUDNN_STATUS_NOT_SUPPORTED = 9
CUDNN_DATA_FLOAT = 0
CUDNN_DATA_DOUBLE = 1
CUDNN_DATA_HALF = 2
CUDNN_DATA_BFLOAT16 = 9
CUDNN_TENSOR_NCHW = 0
CUDNN_TENSOR_NHWC = 1
CUDNN_CONVOLUTION = 0
CUDNN_CROSS_CORRELATION = 1
CUDNN_SOFTMAX_FAST = 0
CUDNN_SOFTMAX_ACCURATE = 1
CUDNN_SOFTMAX_LOG = 2
CUDNN_SOFTMAX_MODE_INSTANCE = 0
CUDNN_SOFTMAX_MODE_CHANNEL = 1
CUDNN_ACTIVATION_SIGMOID, CUDNN_ACTIVATION_RELU, CUDNN_ACTIVATION_TANH = 0, 1, 2
CUDNN_ACTIVATION_CLIPPED_RELU, CUDNN_ACTIVATION_ELU, CUDNN_ACTIVATION_IDENTITY = 3, 4, 5
CUDNN_ACTIVATION_SWISH = 6
CUDNN_POOLING_MAX, CUDNN_POOLING_AVERAGE_COUNT_INCLUDE_PADDING = 0, 1
CUDNN_POOLING_AVERAGE_COUNT_EXCLUDE_PADDING, CUDNN_POOLING_MAX_DETERMINISTIC = 2, 3
CUDNN_BATCHNORM_PER_ACTIVATION, CUDNN_BATCHNORM_SPATIAL = 0, 1

_ip = P(i32)
CUDNN_PROTOS = {
    "cudnnGetVersion": ([], sz),
    "cudnnGetErrorString": ([i32], C.c_char_p),
    "cudnnCreate": ([P(vp)], i32),
    "cudnnDestroy": ([vp], i32),
    "cudnnSetStream": ([vp, vp], i32),
    "cudnnGetStream": ([vp, P(vp)], i32),
    "cudnnCreateTensorDescriptor": ([P(vp)], i32),
    "cudnnSetTensor4dDescriptor": ([vp, i32, i32, i32, i32, i32, i32], i32),
    "cudnnSetTensor4dDescriptorEx": ([vp, i32, i32, i32, i32, i32, i32, i32, i32, i32], i32),
    "cudnnGetTensor4dDescriptor": ([vp, _ip, _ip, _ip, _ip, _ip, _ip, _ip, _ip, _ip], i32),
    "cudnnDestroyTensorDescriptor": ([vp], i32),
    "cudnnCreateFilterDescriptor": ([P(vp)], i32),
    "cudnnSetFilter4dDescriptor": ([vp, i32, i32, i32, i32, i32, i32], i32),
    "cudnnGetFilter4dDescriptor": ([vp, _ip, _ip, _ip, _ip, _ip, _ip], i32),
    "cudnnDestroyFilterDescriptor": ([vp], i32),
    "cudnnCreateConvolutionDescriptor": ([P(vp)], i32),
    "cudnnSetConvolution2dDescriptor": ([vp, i32, i32, i32, i32, i32, i32, i32, i32], i32),
    "cudnnSetConvolutionGroupCount": ([vp, i32], i32),
    "cudnnGetConvolutionGroupCount": ([vp, _ip], i32),
    "cudnnGetConvolution2dForwardOutputDim": ([vp, vp, vp, _ip, _ip, _ip, _ip], i32),
    "cudnnDestroyConvolutionDescriptor": ([vp], i32),
    "cudnnGetConvolutionForwardWorkspaceSize": ([vp, vp, vp, vp, vp, i32, P(sz)], i32),
    "cudnnConvolutionForward": ([vp, vp, vp, vp, vp, vp, vp, i32, vp, sz, vp, vp, vp], i32),
    "cudnnSoftmaxForward": ([vp, i32, i32, vp, vp, vp, vp, vp, vp], i32),
    "cudnnCreateActivationDescriptor": ([P(vp)], i32),
    "cudnnSetActivationDescriptor": ([vp, i32, i32, C.c_double], i32),
    "cudnnGetActivationDescriptor": ([vp, P(i32), P(i32), P(C.c_double)], i32),
    "cudnnDestroyActivationDescriptor": ([vp], i32),
    "cudnnCreatePoolingDescriptor": ([P(vp)], i32),
    "cudnnSetPooling2dDescriptor": ([vp, i32, i32, i32, i32, i32, i32, i32, i32], i32),
    "cudnnGetPooling2dForwardOutputDim": ([vp, vp, P(i32), P(i32), P(i32), P(i32)], i32),
    "cudnnDestroyPoolingDescriptor": ([vp], i32),
    "cudnnDeriveBNTensorDescriptor": ([vp, vp, i32], i32),
    "cudnnConvolutionBackwardData": ([vp, vp, vp, vp, vp, vp, vp, i32, vp, sz, vp, vp, vp], i32),
    "cudnnConvolutionBackwardFilter": ([vp, vp, vp, vp, vp, vp, vp, i32, vp, sz, vp, vp, vp], i32),
    "cudnnConvolutionBackwardBias": ([vp, vp, vp, vp, vp, vp, vp], i32),
    "cudnnAddTensor": ([vp, vp, vp, vp, vp, vp, vp], i32),
    "cudnnActivationForward": ([vp, vp, vp, vp, vp, vp, vp, vp], i32),
    "cudnnPoolingForward": ([vp, vp, vp, vp, vp, vp, vp, vp], i32),
    "cudnnBatchNormalizationForwardInference": ([vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                                 vp, C.c_double], i32),
    "cudnnBatchNormalizationForwardTraining": ([vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                                C.c_double, vp, vp, C.c_double, vp, vp], i32),
}


@lru_cache(maxsize=None)
def cudnn() -> C.CDLL:
    return _declare(_load("cudnn"), CUDNN_PROTOS)


# ---------------------------------------------------------------- cuSPARSE --
CUSPARSE_STATUS_SUCCESS = 0
CUSPARSE_STATUS_NOT_INITIALIZED = 1
CUSPARSE_STATUS_INVALID_VALUE = 3
CUSPARSE_STATUS_NOT_SUPPORTED = 10
CUSPARSE_OPERATION_NON_TRANSPOSE = 0
CUSPARSE_OPERATION_TRANSPOSE = 1
CUSPARSE_INDEX_32I = 2
CUSPARSE_INDEX_64I = 3
CUSPARSE_INDEX_BASE_ZERO = 0
CUSPARSE_INDEX_BASE_ONE = 1
CUSPARSE_ORDER_COL = 1
CUSPARSE_ORDER_ROW = 2
CUDA_R_32F = 0
CUDA_R_16F = 2
CUDA_R_16BF = 14

CUSPARSE_PROTOS = {
    "cusparseCreate": ([P(vp)], i32),
    "cusparseDestroy": ([vp], i32),
    "cusparseGetVersion": ([vp, P(i32)], i32),
    "cusparseSetStream": ([vp, vp], i32),
    "cusparseGetStream": ([vp, P(vp)], i32),
    "cusparseGetErrorName": ([i32], C.c_char_p),
    "cusparseGetErrorString": ([i32], C.c_char_p),
    "cusparseCreateCsr": ([P(vp), i64, i64, i64, vp, vp, vp, i32, i32, i32, i32], i32),
    "cusparseDestroySpMat": ([vp], i32),
    "cusparseCreateDnVec": ([P(vp), i64, vp, i32], i32),
    "cusparseDestroyDnVec": ([vp], i32),
    "cusparseSpMV_bufferSize": ([vp, i32, vp, vp, vp, vp, vp, i32, i32, P(sz)], i32),
    "cusparseSpMV": ([vp, i32, vp, vp, vp, vp, vp, i32, i32, vp], i32),
    "cusparseCreateDnMat": ([P(vp), i64, i64, i64, vp, i32, i32], i32),
    "cusparseDestroyDnMat": ([vp], i32),
    "cusparseSpMM_bufferSize": ([vp, i32, i32, vp, vp, vp, vp, vp, i32, i32, P(sz)], i32),
    "cusparseSpMM": ([vp, i32, i32, vp, vp, vp, vp, vp, i32, i32, vp], i32),
}


@lru_cache(maxsize=None)
def cusparse() -> C.CDLL:
    return _declare(_load("cusparse"), CUSPARSE_PROTOS)


# ------------------------------------------------------------------- cuFFT --
CUFFT_SUCCESS = 0
CUFFT_INVALID_PLAN = 1
CUFFT_INVALID_TYPE = 3
CUFFT_INVALID_VALUE = 4
CUFFT_EXEC_FAILED = 6
CUFFT_INVALID_SIZE = 8
CUFFT_NOT_SUPPORTED = 16
CUFFT_FORWARD = -1
CUFFT_INVERSE = 1
CUFFT_R2C = 0x2A
CUFFT_C2R = 0x2C
CUFFT_C2C = 0x29
CUFFT_Z2Z = 0x69

CUFFT_PROTOS = {
    "cufftCreate": ([P(vp)], i32),
    "cufftPlan1d": ([P(vp), i32, i32, i32], i32),
    "cufftPlanMany": ([P(vp), i32, P(i32), P(i32), i32, i32, P(i32), i32, i32, i32, i32], i32),
    "cufftMakePlan1d": ([vp, i32, i32, i32, P(sz)], i32),
    "cufftPlan2d": ([P(vp), i32, i32, i32], i32),
    "cufftPlan3d": ([P(vp), i32, i32, i32, i32], i32),
    "cufftMakePlan2d": ([vp, i32, i32, i32, P(sz)], i32),
    "cufftMakePlan3d": ([vp, i32, i32, i32, i32, P(sz)], i32),
    "cufftMakePlanMany": ([vp, i32, P(i32), P(i32), i32, i32, P(i32), i32, i32, i32, i32, P(sz)],
                          i32),
    "cufftSetStream": ([vp, vp], i32),
    "cufftGetSize": ([vp, P(sz)], i32),
    "cufftDestroy": ([vp], i32),
    "cufftExecC2C": ([vp, vp, vp, i32], i32),
    "cufftExecR2C": ([vp, vp, vp], i32),
    "cufftExecC2R": ([vp, vp, vp], i32),
    "cufftExecC2CNoAlloc": ([vp, vp, C.c_longlong, C.c_longlong, i32, vp], i32),
}


@lru_cache(maxsize=None)
def cufft() -> C.CDLL:
    return _declare(_load("cufft"), CUFFT_PROTOS)


# ------------------------------------------------------------------ cuBLAS --
CUBLAS_STATUS_SUCCESS = 0
CUBLAS_STATUS_NOT_INITIALIZED = 1
CUBLAS_STATUS_INVALID_VALUE = 7
CUBLAS_STATUS_EXECUTION_FAILED = 13
CUBLAS_STATUS_NOT_SUPPORTED = 15
CUBLAS_OP_N = 0
CUBLAS_OP_T = 1
CUBLAS_OP_C = 2
CUBLAS_POINTER_MODE_HOST = 0
CUBLAS_POINTER_MODE_DEVICE = 1
CUBLAS_DEFAULT_MATH = 0
CUBLAS_TENSOR_OP_MATH = 1
CUBLAS_PEDANTIC_MATH = 2
CUBLAS_TF32_TENSOR_OP_MATH = 3
CUBLAS_COMPUTE_16F = 64
CUBLAS_COMPUTE_32F = 68
CUBLAS_GEMM_DEFAULT = -1

ll = C.c_longlong
CUBLAS_PROTOS = {
    "cublasCreate_v2": ([P(vp)], i32),
    "cublasDestroy_v2": ([vp], i32),
    "cublasGetVersion_v2": ([vp, P(i32)], i32),
    "cublasSetStream_v2": ([vp, vp], i32),
    "cublasGetStream_v2": ([vp, P(vp)], i32),
    "cublasSetPointerMode_v2": ([vp, i32], i32),
    "cublasGetPointerMode_v2": ([vp, P(i32)], i32),
    "cublasSetMathMode": ([vp, i32], i32),
    "cublasGetMathMode": ([vp, P(i32)], i32),
    "cublasGetStatusName": ([i32], C.c_char_p),
    "cublasGetStatusString": ([i32], C.c_char_p),
    "cublasSgemm_v2": ([vp, i32, i32, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32], i32),
    "cublasHgemm": ([vp, i32, i32, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32], i32),
    "cublasGemmEx": ([vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp, i32, i32, vp, vp, i32,
                      i32, i32, i32], i32),
    "cublasSgemmStridedBatched": ([vp, i32, i32, i32, i32, i32, vp, vp, i32, ll, vp, i32, ll,
                                   vp, vp, i32, ll, i32], i32),
    "cublasGemmStridedBatchedEx": ([vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, ll, vp, i32,
                                    i32, ll, vp, vp, i32, i32, ll, i32, i32, i32], i32),
    "cublasSaxpy_v2": ([vp, i32, vp, vp, i32, vp, i32], i32),
    "cublasScopy_v2": ([vp, i32, vp, i32, vp, i32], i32),
    "cublasSscal_v2": ([vp, i32, vp, vp, i32], i32),
    "cublasSswap_v2": ([vp, i32, vp, i32, vp, i32], i32),
    "cublasSdot_v2": ([vp, i32, vp, i32, vp, i32, vp], i32),
    "cublasSnrm2_v2": ([vp, i32, vp, i32, vp], i32),
    "cublasSasum_v2": ([vp, i32, vp, i32, vp], i32),
    "cublasIsamax_v2": ([vp, i32, vp, i32, vp], i32),
    "cublasSgemv_v2": ([vp, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32], i32),
    "cublasSgeam": ([vp, i32, i32, i32, i32, vp, vp, i32, vp, vp, i32, vp, i32], i32),
    "cublasDgeam": ([vp, i32, i32, i32, i32, vp, vp, i32, vp, vp, i32, vp, i32], i32),
    "cublasDaxpy_v2": ([vp, i32, vp, vp, i32, vp, i32], i32),
    "cublasDcopy_v2": ([vp, i32, vp, i32, vp, i32], i32),
    "cublasDscal_v2": ([vp, i32, vp, vp, i32], i32),
    "cublasDswap_v2": ([vp, i32, vp, i32, vp, i32], i32),
    "cublasDdot_v2": ([vp, i32, vp, i32, vp, i32, vp], i32),
    "cublasDnrm2_v2": ([vp, i32, vp, i32, vp], i32),
    "cublasDasum_v2": ([vp, i32, vp, i32, vp], i32),
    "cublasIdamax_v2": ([vp, i32, vp, i32, vp], i32),
    "cublasDgemv_v2": ([vp, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32], i32),
    "cublasDgemm_v2": ([vp, i32, i32, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32], i32),
    "cublasDgemmStridedBatched": ([vp, i32, i32, i32, i32, i32, vp, vp, i32, ll, vp, i32, ll,
                                   vp, vp, i32, ll, i32], i32),
}


@lru_cache(maxsize=None)
def cublas() -> C.CDLL:
    return _declare(_load("cublas"), CUBLAS_PROTOS)


# ---------------------------------------------------------- peer exchange --
MB200_PEER_SUCCESS = 0
MB200_PEER_INVALID_VALUE = 1
MB200_PEER_CUDA_ERROR = 2
MB200_PEER_HANDLE_BYTES = 64
MB200_PEER_MAX_RANKS = 32
MB200_PEER_STATUS_WORD = 48
MB200_PEER_HEADER_BYTES = 256

PEER_PROTOS = {
    "mb200PeerAlloc": ([C.c_size_t, P(C.c_void_p), C.c_void_p], C.c_int),
    "mb200PeerOpen": ([C.c_void_p, P(C.c_void_p)], C.c_int),
    "mb200PeerClose": ([C.c_void_p], C.c_int),
    "mb200PeerFree": ([C.c_void_p], C.c_int),
    "mb200PeerBuffer": ([C.c_void_p, C.c_size_t, C.c_uint], C.c_void_p),
    "mb200PeerAllgather": ([P(C.c_void_p), C.c_int, C.c_int, C.c_size_t, C.c_size_t, C.c_uint,
                            C.c_void_p, C.c_void_p], C.c_int),
    "mb200PeerTakeStatus": ([C.c_void_p, P(C.c_uint)], C.c_int),
}


@lru_cache(maxsize=None)
def peer() -> C.CDLL:
    return _declare(_load("peer"), PEER_PROTOS)


PROBE_PROTOS = {
    "mb200ProbeGather": ([C.c_void_p, C.c_void_p, C.c_longlong, C.c_int, C.c_void_p, C.c_uint,
                          C.c_void_p], C.c_int),
    "mb200ProbeScatter": ([C.c_void_p, C.c_void_p, C.c_longlong, C.c_int, C.c_uint,
                           C.c_void_p], C.c_int),
    "mb200ProbeRowGather": ([C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p, C.c_uint,
                             C.c_void_p], C.c_int),
    "mb200ProbeNormalError": ([C.c_void_p, C.c_void_p], C.c_int),
}


@lru_cache(maxsize=None)
def probe() -> C.CDLL:
    """Benchmark probes (not part of the drop-in API)."""
    return _declare(_load("probe"), PROBE_PROTOS)


ALL_PROTOS: dict[str, dict[str, tuple[list, object]]] = {
    "curand": CURAND_PROTOS,
    "cudnn": CUDNN_PROTOS,
    "cusparse": CUSPARSE_PROTOS,
    "cufft": CUFFT_PROTOS,
    "cublas": CUBLAS_PROTOS,
    "peer": PEER_PROTOS,
    "probe": PROBE_PROTOS,
}

LOADERS = {
    "curand": curand,
    "cudnn": cudnn,
    "cusparse": cusparse,
    "cufft": cufft,
    "cublas": cublas,
    "peer": peer,
    "probe": probe,
}
