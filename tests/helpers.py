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
