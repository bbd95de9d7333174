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
}


@lru_cache(maxsize=None)
def curand() -> C.CDLL:
    return _declare(_load("curand"), CURAND_PROTOS)


ALL_PROTOS: dict[str, dict[str, tuple[list, object]]] = {
    "curand": CURAND_PROTOS,
}

LOADERS = {
    "curand": curand,
}
