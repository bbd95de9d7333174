"""CPU oracle for the hot path — TEST INFRASTRUCTURE ONLY.

Restatements of the reference's host code and kernel arithmetic (see
``oracle/oracle.h``), compiled into ``oracle/_build/liboracle.so`` by
``oracle/build.py``.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` may import this package, as the checker or as the timed
CPU baseline; the product under ``muda_b200/`` never does.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lib: C.CDLL | None = None

_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)


def lib() -> C.CDLL:
    """Loads (building first if needed) the oracle shared library."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from oracle.build import build
            build()
        L = C.CDLL(str(LIB_PATH))
        L.oracle_philox_block.argtypes = [C.c_uint64, C.c_uint64, _u32p]
        L.oracle_philox_block.restype = None
        L.oracle_generate_uint.argtypes = [C.c_uint64, C.c_uint64, _u32p, C.c_size_t, C.c_int]
        L.oracle_generate_uint.restype = C.c_uint64
        L.oracle_generate_uniform.argtypes = [C.c_uint64, C.c_uint64, _f32p, C.c_size_t, C.c_int]
        L.oracle_generate_uniform.restype = C.c_uint64
        L.oracle_generate_normal.argtypes = [C.c_uint64, C.c_uint64, _f32p, C.c_size_t,
                                             C.c_float, C.c_float, C.c_int]
        L.oracle_generate_normal.restype = C.c_uint64
        L.oracle_philox_gather.argtypes = [C.POINTER(C.c_uint64), C.c_size_t, C.c_uint64, _u32p,
                                           C.c_int]
        L.oracle_philox_gather.restype = None
        _register_extra(L)
        _lib = L
    return _lib


def _register_extra(L: C.CDLL) -> None:
    """Declares the prototypes of the non-RNG oracles present in the library."""
    from oracle import protos
    protos.declare(L)


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


# ---------------------------------------------------------------- Philox --
def philox_block(ctr: int, seed: int) -> np.ndarray:
    out = np.zeros(4, dtype=np.uint32)
    lib().oracle_philox_block(ctr, seed, _ptr(out, C.c_uint32))
    return out


def generate_uint(seed: int, offset: int, n: int, threads: int = 1) -> tuple[np.ndarray, int]:
    out = np.empty(n, dtype=np.uint32)
    nxt = lib().oracle_generate_uint(seed, offset, _ptr(out, C.c_uint32), n, threads)
    return out, int(nxt)


def generate_uniform(seed: int, offset: int, n: int, threads: int = 1) -> tuple[np.ndarray, int]:
    out = np.empty(n, dtype=np.float32)
    nxt = lib().oracle_generate_uniform(seed, offset, _ptr(out, C.c_float), n, threads)
    return out, int(nxt)


def generate_normal(seed: int, offset: int, n: int, mean: float = 0.0, stddev: float = 1.0,
                    threads: int = 1) -> tuple[np.ndarray, int]:
    out = np.empty(n, dtype=np.float32)
    nxt = lib().oracle_generate_normal(seed, offset, _ptr(out, C.c_float), n, mean, stddev,
                                       threads)
    return out, int(nxt)


def philox_gather(ctrs: np.ndarray, seed: int, threads: int = 8) -> np.ndarray:
    """Philox blocks at the given counters, shape (len(ctrs), 4)."""
    ctrs = np.ascontiguousarray(ctrs, dtype=np.uint64)
    out = np.empty((len(ctrs), 4), dtype=np.uint32)
    lib().oracle_philox_gather(_ptr(ctrs, C.c_uint64), len(ctrs), seed, _ptr(out, C.c_uint32),
                               threads)
    return out
