"""Shared helpers for the GPU tests: thin wrappers over the C ABI via ctypes."""

from __future__ import annotations

import ctypes as C
import contextlib

import numpy as np

from muda_b200 import capi


def stream_ptr(torch) -> int:
    return int(torch.cuda.current_stream().cuda_stream)


@contextlib.contextmanager
def curand_generator(seed: int, torch=None, host: bool = False, offset: int | None = None):
    L = capi.curand()
    g = C.c_void_p()
    create = L.curandCreateGeneratorHost if host else L.curandCreateGenerator
    assert create(C.byref(g), capi.CURAND_RNG_PSEUDO_PHILOX4_32_10) == 0
    try:
        assert L.curandSetPseudoRandomGeneratorSeed(g, seed) == 0
        if offset is not None:
            assert L.curandSetGeneratorOffset(g, offset) == 0
        if torch is not None:
            assert L.curandSetStream(g, C.c_void_p(stream_ptr(torch))) == 0
        yield g
    finally:
        assert L.curandDestroyGenerator(g) == 0


def ulp_distance_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in units of least precision between two float32 arrays."""
    ia = a.astype(np.float32).view(np.int32).astype(np.int64)
    ib = b.astype(np.float32).view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, np.int64(-0x80000000) - ia, ia)
    ib = np.where(ib < 0, np.int64(-0x80000000) - ib, ib)
    return np.abs(ia - ib)


# ------------------------------------------------------------------- cuDNN --
class Dnn:
    """Owns a cuDNN handle plus the descriptors a test creates; destroys them on exit."""

    def __init__(self, torch=None):
        self.L = capi.cudnn()
        self.h = C.c_void_p()
        assert self.L.cudnnCreate(C.byref(self.h)) == 0
        if torch is not None:
            assert self.L.cudnnSetStream(self.h, C.c_void_p(stream_ptr(torch))) == 0
        self._owned = []

    def tensor(self, n, c, h, w, fmt=capi.CUDNN_TENSOR_NCHW, dtype=capi.CUDNN_DATA_FLOAT,
               strides=None):
        d = C.c_void_p()
        assert self.L.cudnnCreateTensorDescriptor(C.byref(d)) == 0
        if strides is None:
            assert self.L.cudnnSetTensor4dDescriptor(d, fmt, dtype, n, c, h, w) == 0
        else:
            assert self.L.cudnnSetTensor4dDescriptorEx(d, dtype, n, c, h, w, *strides) == 0
        self._owned.append(("cudnnDestroyTensorDescriptor", d))
        return d

    def filter(self, k, c, r, s, fmt=capi.CUDNN_TENSOR_NCHW, dtype=capi.CUDNN_DATA_FLOAT):
        d = C.c_void_p()
        assert self.L.cudnnCreateFilterDescriptor(C.byref(d)) == 0
        assert self.L.cudnnSetFilter4dDescriptor(d, dtype, fmt, k, c, r, s) == 0
        self._owned.append(("cudnnDestroyFilterDescriptor", d))
        return d

    def conv(self, pad=(0, 0), stride=(1, 1), dil=(1, 1), mode=capi.CUDNN_CROSS_CORRELATION,
             groups=1, compute=capi.CUDNN_DATA_FLOAT):
        d = C.c_void_p()
        assert self.L.cudnnCreateConvolutionDescriptor(C.byref(d)) == 0
        assert self.L.cudnnSetConvolution2dDescriptor(d, pad[0], pad[1], stride[0], stride[1],
                                                      dil[0], dil[1], mode, compute) == 0
        if groups != 1:
            assert self.L.cudnnSetConvolutionGroupCount(d, groups) == 0
        self._owned.append(("cudnnDestroyConvolutionDescriptor", d))
        return d

    def close(self):
        for fn, d in reversed(self._owned):
            assert getattr(self.L, fn)(d) == 0
        assert self.L.cudnnDestroy(self.h) == 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


def fptr(v: float):
    return C.byref(C.c_float(v))
