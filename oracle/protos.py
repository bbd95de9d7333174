"""ctypes prototypes of the non-RNG oracle functions (test infrastructure only)."""

from __future__ import annotations

import ctypes as C


def declare(L: C.CDLL) -> None:
    for name, argtypes, restype in _PROTOS:
        fn = getattr(L, name, None)
        if fn is None:
            continue
        fn.argtypes = argtypes
        fn.restype = restype


_PROTOS: list[tuple[str, list, object]] = []
