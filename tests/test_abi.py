"""C-ABI checks that need no GPU: every library loads and exports every entry
point its header declares, and the host-side argument / handle logic returns the
reference's status codes."""

import ctypes as C
import re
from pathlib import Path

import pytest

from muda_b200 import capi
from muda_b200.build import LIBS, lib_path

INCLUDE = Path(__file__).resolve().parent.parent / "include"

HEADER_LIB = {
    "curand.h": "curand",
    "cudnn.h": "cudnn",
    "cusparse.h": "cusparse",
    "cufft.h": "cufft",
    "cublas_v2.h": "cublas",
    "mb200_peer.h": "peer",
    "mb200_probe.h": "probe",
}


def declared_functions(header: Path) -> list[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s+\*?([A-Za-z_][A-Za-z0-9_]*)\s*\(",
                       text, flags=re.M)
    return sorted(set(n for n in names if not n.startswith("MUDA")))


def test_every_header_has_a_library():
    for h in INCLUDE.glob("*.h"):
        assert h.name in HEADER_LIB, f"{h.name} has no library mapping"


@pytest.mark.parametrize("header", sorted(HEADER_LIB))
def test_library_exports_every_declared_symbol(built, header):
    lib = C.CDLL(str(lib_path(HEADER_LIB[header])))
    names = declared_functions(INCLUDE / header)
    assert names, header
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"{header}: missing exports {missing}"


def test_bindings_cover_headers(built):
    for header, name in HEADER_LIB.items():
        declared = set(declared_functions(INCLUDE / header))
        bound = set(capi.ALL_PROTOS[name])
        assert declared == bound, f"{header}: declared-but-unbound {declared - bound}, " \
                                  f"bound-but-undeclared {bound - declared}"


# ---------------------------------------------------------------- cuRAND --
def test_curand_handle_logic(built):
    L = capi.curand()
    gen = C.c_void_p()
    assert L.curandCreateGenerator(C.byref(gen), capi.CURAND_RNG_PSEUDO_PHILOX4_32_10) == 0
    assert gen.value
    assert L.curandCreateGenerator(None, 100) == capi.CURAND_STATUS_ALLOCATION_FAILED
    assert L.curandSetPseudoRandomGeneratorSeed(gen, 1234) == 0
    assert L.curandSetGeneratorOffset(gen, 16) == 0
    s = C.c_void_p(123)
    assert L.curandSetStream(gen, C.c_void_p(0)) == 0
    assert L.curandGetStream(gen, C.byref(s)) == 0 and not s.value
    assert L.curandGetStream(gen, None) == capi.CURAND_STATUS_INVALID_VALUE
    # num == 0 succeeds without touching the device; null output with num > 0 fails first
    assert L.curandGenerateUniform(gen, None, 0) == 0
    assert L.curandGenerateUniform(gen, None, 16) == capi.CURAND_STATUS_INVALID_VALUE
    assert L.curandDestroyGenerator(gen) == 0
    # stale handle
    assert L.curandDestroyGenerator(gen) == capi.CURAND_STATUS_NOT_INITIALIZED
    assert L.curandSetPseudoRandomGeneratorSeed(gen, 1) == capi.CURAND_STATUS_NOT_INITIALIZED
    assert L.curandGenerateUniform(gen, C.c_void_p(64), 16) == capi.CURAND_STATUS_NOT_INITIALIZED
    # forged handles: null, wrong kind bits, random value
    for bad in (0, 0x1, 0xDEADBEEF, (7 << 32) | (0x11 << 24) | 1):
        assert L.curandSetStream(C.c_void_p(bad), None) == capi.CURAND_STATUS_NOT_INITIALIZED


def test_curand_slot_reuse_rejects_old_handle(built):
    L = capi.curand()
    a = C.c_void_p()
    assert L.curandCreateGenerator(C.byref(a), 100) == 0
    assert L.curandDestroyGenerator(a) == 0
    b = C.c_void_p()
    assert L.curandCreateGenerator(C.byref(b), 100) == 0
    assert a.value != b.value
    assert L.curandSetPseudoRandomGeneratorSeed(a, 1) == capi.CURAND_STATUS_NOT_INITIALIZED
    assert L.curandSetPseudoRandomGeneratorSeed(b, 1) == 0
    assert L.curandDestroyGenerator(b) == 0


def test_curand_version_and_property(built):
    L = capi.curand()
    v = C.c_int()
    assert L.curandGetVersion(C.byref(v)) == 0 and v.value == 10200
    for prop, expect in ((0, 10), (1, 2), (2, 0)):
        assert L.curandGetProperty(prop, C.byref(v)) == 0 and v.value == expect
    assert L.curandGetProperty(7, C.byref(v)) == capi.CURAND_STATUS_INVALID_VALUE
    assert L.curandGetVersion(None) == capi.CURAND_STATUS_INVALID_VALUE
