"""cufftExecC2CNoAlloc: the allocation-free FFT entry point.

It exists for callers that cannot allocate device memory when they need a
transform (inside an allocator or memory-pool callback, real-time paths that
forbid allocation after start-up, processes under a hard memory cap); it keeps
its tables and workspace in a fixed device array owned by the library.  This
test calls it through the C ABI twice in a row, with different lengths so the
second call runs over the first call's leftover tables and workspace, and checks
each result against the planned cufftExecC2C path within the FFT tolerance used
everywhere else (relative L2 error <= 1e-5 per transform).  Because both paths
run the same Stockham kernels, results are also checked against numpy's
double-precision FFT (sign -1 forward, no scaling on either direction), including
a two-pass length whose batch is larger than one chunk of the fixed workspace, so
that the chunk loop runs more than once.

The file is named to be collected last, so a run that stops at the first failure
has already run every other test.
"""

import ctypes as C

import numpy as np
import pytest

from muda_b200 import capi
from tests.helpers import stream_ptr

pytestmark = pytest.mark.gpu

TOL = 1e-5


def planned(torch, x, n, batch, direction):
    L = capi.cufft()
    p = C.c_void_p()
    assert L.cufftPlan1d(C.byref(p), n, capi.CUFFT_C2C, batch) == 0
    try:
        assert L.cufftSetStream(p, C.c_void_p(stream_ptr(torch))) == 0
        out = torch.empty_like(x)
        assert L.cufftExecC2C(p, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                              direction) == 0
        torch.cuda.synchronize()
        return out
    finally:
        assert L.cufftDestroy(p) == 0


def no_alloc(torch, x, n, batch, direction):
    L = capi.cufft()
    out = torch.empty_like(x)
    st = L.cufftExecC2CNoAlloc(C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), n, batch,
                               direction, C.c_void_p(stream_ptr(torch)))
    torch.cuda.synchronize()
    assert st == 0
    return out


def worst_rel_l2(got, want, n, batch):
    g = got.view(batch, 2 * n).double()
    w = want.view(batch, 2 * n).double()
    return float(((g - w).norm(dim=1) / w.norm(dim=1)).max())


def test_no_alloc_matches_planned_path_twice(cuda, built):
    torch = cuda
    gen = torch.Generator(device="cuda").manual_seed(1234)
    calls = [(1 << 15, 6, capi.CUFFT_FORWARD), (1 << 20, 2, capi.CUFFT_INVERSE)]
    for n, batch, direction in calls:
        x = torch.randn(2 * n * batch, generator=gen, device="cuda", dtype=torch.float32)
        got = no_alloc(torch, x, n, batch, direction)
        want = planned(torch, x, n, batch, direction)
        assert worst_rel_l2(got, want, n, batch) <= TOL, (n, batch)


def numpy_fft(x, n, batch, direction):
    """numpy's float64 transform with the library's conventions (no 1/N on the inverse)."""
    z = x.cpu().numpy().astype(np.float64).view(np.complex128).reshape(batch, n)
    if direction == capi.CUFFT_FORWARD:
        return np.fft.fft(z, axis=1)
    return np.fft.ifft(z, axis=1) * n


def worst_rel_l2_f64(got, want, n, batch):
    g = got.cpu().numpy().astype(np.float64).view(np.complex128).reshape(batch, n)
    return float((np.linalg.norm(g - want, axis=1) / np.linalg.norm(want, axis=1)).max())


@pytest.mark.parametrize("n,batch,direction", [
    (1 << 10, 33, capi.CUFFT_FORWARD),          # one pass
    (1 << 14, 5, capi.CUFFT_INVERSE),           # largest single-pass length
    (1 << 17, 9, capi.CUFFT_FORWARD),           # two passes; chunk of 8: the loop runs twice
    (1 << 20, 3, capi.CUFFT_INVERSE),           # largest length; chunk of 1: three chunks
])
def test_no_alloc_matches_float64_fft(cuda, built, n, batch, direction):
    torch = cuda
    gen = torch.Generator(device="cuda").manual_seed(n + batch)
    x = torch.randn(2 * n * batch, generator=gen, device="cuda", dtype=torch.float32)
    got = no_alloc(torch, x, n, batch, direction)
    assert worst_rel_l2_f64(got, numpy_fft(x, n, batch, direction), n, batch) <= TOL
    # a second call in place on the same buffer, the other direction
    y = got.clone()
    L = capi.cufft()
    other = capi.CUFFT_INVERSE if direction == capi.CUFFT_FORWARD else capi.CUFFT_FORWARD
    ptr = C.c_void_p(y.data_ptr())
    assert L.cufftExecC2CNoAlloc(ptr, ptr, n, batch, other, C.c_void_p(stream_ptr(torch))) == 0
    torch.cuda.synchronize()
    assert worst_rel_l2_f64(y, numpy_fft(got, n, batch, other), n, batch) <= TOL


def test_no_alloc_single_pass_and_in_place(cuda, built):
    torch = cuda
    gen = torch.Generator(device="cuda").manual_seed(7)
    n, batch = 4096, 64
    x = torch.randn(2 * n * batch, generator=gen, device="cuda", dtype=torch.float32)
    want = planned(torch, x, n, batch, capi.CUFFT_FORWARD)
    y = x.clone()
    L = capi.cufft()
    ptr = C.c_void_p(y.data_ptr())
    assert L.cufftExecC2CNoAlloc(ptr, ptr, n, batch, capi.CUFFT_FORWARD,
                                 C.c_void_p(stream_ptr(torch))) == 0
    torch.cuda.synchronize()
    assert worst_rel_l2(y, want, n, batch) <= TOL


def test_no_alloc_rejects_sizes_beyond_its_maximum(cuda, built):
    torch = cuda
    L = capi.cufft()
    x = torch.zeros(2 * 16, dtype=torch.float32, device="cuda")
    p = C.c_void_p(x.data_ptr())
    s = C.c_void_p(stream_ptr(torch))
    assert L.cufftExecC2CNoAlloc(p, p, 1 << 21, 1, capi.CUFFT_FORWARD, s) == \
        capi.CUFFT_INVALID_SIZE
    assert L.cufftExecC2CNoAlloc(p, p, 12, 1, capi.CUFFT_FORWARD, s) == capi.CUFFT_INVALID_SIZE
    assert L.cufftExecC2CNoAlloc(p, p, 16, 1, 0, s) == capi.CUFFT_INVALID_VALUE
