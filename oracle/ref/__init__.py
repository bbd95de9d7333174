"""The reference's own host Philox generator, compiled — TEST INFRASTRUCTURE ONLY.

``oracle/_ref/libcurand_ref.so`` (built by ``oracle/ref/build.py`` from the
reference's unmodified ``libraries/rand/src/curand_context.mm``) pins both the
oracle restatement and the GPU kernels to the reference's real code.  Only
``tests/`` and the CPU legs of ``bench.py`` use it.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from oracle.ref.build import OUT as LIB_PATH

UINT, UNIFORM, NORMAL, LOGNORMAL, UNIFORM_DOUBLE, NORMAL_DOUBLE, LOGNORMAL_DOUBLE, POISSON = range(8)
_DTYPE = {UINT: np.uint32, UNIFORM: np.float32, NORMAL: np.float32, LOGNORMAL: np.float32,
          UNIFORM_DOUBLE: np.float64, NORMAL_DOUBLE: np.float64, LOGNORMAL_DOUBLE: np.float64,
          POISSON: np.uint32}

_lib: C.CDLL | None = None


def available() -> bool:
    return Path(LIB_PATH).exists()


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{LIB_PATH} is not built (oracle/ref/build.py needs the "
                                    "reference tree)")
        L = C.CDLL(str(LIB_PATH))
        L.ref_philox_step.argtypes = [C.c_uint64, C.c_uint64, C.POINTER(C.c_uint32)]
        L.ref_philox_step.restype = None
        L.ref_generate.argtypes = [C.c_int, C.c_uint64, C.c_uint64, C.c_void_p, C.c_size_t,
                                   C.c_double, C.c_double, C.c_double, C.POINTER(C.c_uint64)]
        L.ref_generate.restype = C.c_int
        L.ref_generate_at.argtypes = [C.c_int, C.c_uint64, C.POINTER(C.c_uint64), C.c_size_t,
                                      C.c_size_t, C.c_void_p, C.c_double, C.c_double]
        L.ref_generate_at.restype = C.c_int
        L.ref_generate_parallel.argtypes = [C.c_int, C.c_uint64, C.c_uint64, C.c_void_p,
                                            C.c_size_t, C.c_double, C.c_double, C.c_int]
        L.ref_generate_parallel.restype = C.c_uint64
        _lib = L
    return _lib


def philox_step(ctr: int, seed: int) -> np.ndarray:
    out = np.zeros(4, dtype=np.uint32)
    lib().ref_philox_step(ctr, seed, out.ctypes.data_as(C.POINTER(C.c_uint32)))
    return out


def generate(kind: int, seed: int, offset: int, n: int, mean: float = 0.0, stddev: float = 1.0,
             lam: float = 0.0) -> tuple[np.ndarray, int]:
    """One GenerateHost* call of the reference on a generator at (seed, offset);
    returns the outputs and the generator offset after the call."""
    out = np.zeros(max(n, 1), dtype=_DTYPE[kind])
    new = C.c_uint64()
    st = lib().ref_generate(kind, seed, offset, out.ctypes.data_as(C.c_void_p), n, mean, stddev,
                            lam, C.byref(new))
    assert st == 0, f"reference GenerateHost kind {kind} returned {st}"
    return out[:n], new.value


def generate_at(kind: int, seed: int, offsets: np.ndarray, words: int, mean: float = 0.0,
                stddev: float = 1.0) -> np.ndarray:
    """len(offsets) separate calls of `words` outputs, call i at offsets[i]; returns an
    array of shape (len(offsets), words)."""
    offs = np.ascontiguousarray(offsets, dtype=np.uint64)
    out = np.zeros((len(offs), words), dtype=_DTYPE[kind])
    st = lib().ref_generate_at(kind, seed, offs.ctypes.data_as(C.POINTER(C.c_uint64)), len(offs),
                               words, out.ctypes.data_as(C.c_void_p), mean, stddev)
    assert st == 0, f"reference GenerateHost kind {kind} returned {st}"
    return out


def generate_parallel(kind: int, seed: int, offset: int, n: int, mean: float = 0.0,
                      stddev: float = 1.0, threads: int = 1,
                      out: np.ndarray | None = None) -> tuple[np.ndarray, int]:
    """One logical GenerateHost* call of n outputs, run as `threads` reference calls on
    consecutive slices of whole Philox blocks (identical output; offset must be a
    multiple of the block's word count)."""
    if out is None:
        out = np.empty(max(n, 1), dtype=_DTYPE[kind])
    nxt = lib().ref_generate_parallel(kind, seed, offset, out.ctypes.data_as(C.c_void_p), n,
                                      mean, stddev, threads)
    return out[:n], int(nxt)
