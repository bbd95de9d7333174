"""cuBLAS level 1 / 2 (fp32): saxpy, scopy, sscal, sswap, sdot, snrm2, sasum, isamax, sgemv.

CPU: the oracle against the reference's known answers (tests/cublas_test.cpp:134-297)
and the entry points' argument checks.  GPU (marked): the CUDA kernels through the C
ABI against the oracle.  Bars: axpy / copy / scal / swap and the single-pass gemv N
bit-exact (same per-element formula and order); dot / nrm2 / asum within 1e-5 of the
sum of term magnitudes (float64 ground truth); isamax exact; gemv within 1e-5 of
|alpha| |op(A)| |x| + |beta y| per output.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import stream_ptr


def ref_level1_inputs():
    """tests/cublas_test.cpp:141-148."""
    n = 128
    x = (np.arange(n, dtype=np.float32) + 1) * np.float32(0.25)
    y = (n - np.arange(n, dtype=np.float32)) * np.float32(0.5)
    x[42] = -99.5
    return n, x, y


def test_oracle_reference_level1_pins():
    """cublas_test.cpp:163-229: isamax 43 (1-based), asum/dot against the host loop,
    saxpy with alpha 2."""
    n, x, y = ref_level1_inputs()
    assert oracle.isamax(n, x, 1) == 43
    asum, _, _ = oracle.sreduce("asum", n, x, 1)
    assert abs(asum - float(np.sum(np.abs(x), dtype=np.float32))) < 1e-2
    dot, _, _ = oracle.sreduce("dot", n, x, 1, y, 1)
    assert abs(dot - float(np.sum(x * y, dtype=np.float32))) < 1e-1
    out = oracle.saxpy(n, 2.0, x, 1, y, 1)
    assert np.all(np.abs(out - (2.0 * x + y)) < 1e-4)


def test_oracle_reference_gemv_pin():
    """cublas_test.cpp:239-281: 16 x 12, A[r, c] = (r+1)(c+1)/10, x = (c+1)/2, y = 1,
    alpha 1.5, beta 0.5."""
    m, n = 16, 12
    r, c = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
    A = (((r + 1) * (c + 1)).astype(np.float32) * np.float32(0.1)).T.reshape(-1)  # column-major
    x = (np.arange(n, dtype=np.float32) + 1) * np.float32(0.5)
    y, _, _ = oracle.sgemv(False, m, n, 1.5, A, m, x, 1, 0.5, np.ones(m, np.float32), 1)
    want = 1.5 * (A.reshape(n, m).T.astype(np.float64) @ x) + 0.5
    assert np.all(np.abs(y - want) < 1e-3)


def test_oracle_index_conventions():
    x = np.array([1, -7, 3, 7, np.nan, 2], np.float32)
    assert oracle.isamax(6, x, 1) == 2        # first of the equal magnitudes
    assert oracle.isamax(3, x, 2) == 2        # elements 0, 2, 4: |3| wins, NaN never
    assert oracle.isamax(0, x, 1) == 0 and oracle.isamax(3, x, 0) == 0
    # negative increment walks from the far end: element 0 of the vector is x[4]
    y = oracle.scopy(3, np.array([1, 0, 2, 0, 3], np.float32), -2, np.zeros(3, np.float32), 1)
    assert list(y) == [3, 2, 1]
    # sscal with alpha 0 writes exact zeros even over NaN
    s = oracle.sscal(2, 0.0, np.array([np.nan, np.inf], np.float32), 1)
    assert list(s) == [0.0, 0.0]


def test_argument_checks(built):
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    one = C.byref(C.c_float(1.0))
    p = C.c_void_p(256)
    res = C.c_float(7.0)
    idx = C.c_int(7)
    bad = C.c_void_p(12345)
    # bad handle (cublas_level1.mm:223-225)
    assert L.cublasSaxpy_v2(bad, 4, one, p, 1, p, 1) == capi.CUBLAS_STATUS_NOT_INITIALIZED
    assert L.cublasSdot_v2(bad, 4, p, 1, p, 1, C.byref(res)) == capi.CUBLAS_STATUS_NOT_INITIALIZED
    # null scalar / result
    assert L.cublasSaxpy_v2(h, 4, None, p, 1, p, 1) == capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSscal_v2(h, 4, None, p, 1) == capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSnrm2_v2(h, 4, p, 1, None) == capi.CUBLAS_STATUS_INVALID_VALUE
    # n <= 0 succeeds without touching memory; host-mode reductions return 0
    assert L.cublasSaxpy_v2(h, 0, one, p, 1, p, 1) == 0
    assert L.cublasSscal_v2(h, 4, one, p, -1) == 0
    assert L.cublasSdot_v2(h, 0, p, 1, p, 1, C.byref(res)) == 0 and res.value == 0.0
    assert L.cublasIsamax_v2(h, 5, p, 0, C.byref(idx)) == 0 and idx.value == 0
    # alpha == 0 is a no-op for saxpy even with unaddressable vectors (cublas_level1.mm:239)
    assert L.cublasSaxpy_v2(h, 4, C.byref(C.c_float(0.0)), p, 1, p, 1) == 0
    # unaddressable vectors are rejected before any launch
    assert L.cublasScopy_v2(h, 4, p, 1, p, 1) == capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSasum_v2(h, 4, p, 1, C.byref(res)) == capi.CUBLAS_STATUS_INVALID_VALUE
    # gemv argument checks (cublas_level2.mm:45-48)
    for args in ((3, 4, 4), (0, -1, 4), (0, 4, -1)):
        t, m, n = args
        assert L.cublasSgemv_v2(h, t, m, n, one, p, 4, p, 1, one, p, 1) == \
            capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSgemv_v2(h, 0, 4, 4, one, p, 3, p, 1, one, p, 1) == \
        capi.CUBLAS_STATUS_INVALID_VALUE  # lda < m
    assert L.cublasSgemv_v2(h, 0, 4, 4, one, p, 4, p, 0, one, p, 1) == \
        capi.CUBLAS_STATUS_INVALID_VALUE  # incx == 0
    assert L.cublasSgemv_v2(h, 0, 4, 4, None, p, 4, p, 1, one, p, 1) == \
        capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSgemv_v2(h, 0, 0, 4, one, p, 1, p, 1, one, p, 1) == 0
    assert L.cublasDestroy_v2(h) == 0


# --------------------------------------------------------------------- GPU --
class Blas:
    def __init__(self, torch, device_mode=False):
        self.L = capi.cublas()
        self.h = C.c_void_p()
        assert self.L.cublasCreate_v2(C.byref(self.h)) == 0
        assert self.L.cublasSetStream_v2(self.h, C.c_void_p(stream_ptr(torch))) == 0
        if device_mode:
            assert self.L.cublasSetPointerMode_v2(self.h, capi.CUBLAS_POINTER_MODE_DEVICE) == 0

    def close(self):
        assert self.L.cublasDestroy_v2(self.h) == 0


def span(n, inc):
    return 1 + (n - 1) * abs(inc) if n > 0 else 0


def dev(torch, a, misalign=0):
    """Device copy of a float32 array starting `misalign` floats into its allocation."""
    t = torch.zeros(len(a) + 8, dtype=torch.float32, device="cuda")
    t[misalign:misalign + len(a)] = torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    return t, C.c_void_p(t.data_ptr() + 4 * misalign)


def back(t, misalign, count):
    return t.cpu().numpy()[misalign:misalign + count]


ELT_CASES = [(1, 1, 1, 0), (1000003, 1, 1, 0), (1000003, 1, 1, 1), (4096, 2, 3, 0),
             (777, -1, 1, 0), (513, -3, -2, 1), (300, 0, 1, 0), (5, 1, -1, 0)]


@pytest.mark.gpu
@pytest.mark.parametrize("n,incx,incy,mis", ELT_CASES)
def test_gpu_elementwise_bit_exact(cuda, built, n, incx, incy, mis):
    torch = cuda
    rng = np.random.default_rng(n + 7 * incx + incy)
    x = rng.uniform(-2, 2, span(n, incx)).astype(np.float32)
    y = rng.uniform(-2, 2, span(n, incy)).astype(np.float32)
    b = Blas(torch)
    L = b.L
    for alpha in (1.75, 0.0):
        tx, px = dev(torch, x, mis)
        ty, py = dev(torch, y, mis)
        assert L.cublasSaxpy_v2(b.h, n, C.byref(C.c_float(alpha)), px, incx, py, incy) == 0
        torch.cuda.synchronize()
        assert np.array_equal(back(ty, mis, len(y)), oracle.saxpy(n, alpha, x, incx, y, incy))
    if incy != 0:
        tx, px = dev(torch, x, mis)
        ty, py = dev(torch, y, mis)
        assert L.cublasScopy_v2(b.h, n, px, incx, py, incy) == 0
        torch.cuda.synchronize()
        assert np.array_equal(back(ty, mis, len(y)), oracle.scopy(n, x, incx, y, incy))
    if incx != 0 and incy != 0:
        tx, px = dev(torch, x, mis)
        ty, py = dev(torch, y, mis)
        assert L.cublasSswap_v2(b.h, n, px, incx, py, incy) == 0
        torch.cuda.synchronize()
        wx, wy = oracle.sswap(n, x, incx, y, incy)
        assert np.array_equal(back(tx, mis, len(x)), wx)
        assert np.array_equal(back(ty, mis, len(y)), wy)
    for alpha in (-0.5, 0.0):
        tx, px = dev(torch, x, mis)
        assert L.cublasSscal_v2(b.h, n, C.byref(C.c_float(alpha)), px, incx) == 0
        torch.cuda.synchronize()
        assert np.array_equal(back(tx, mis, len(x)), oracle.sscal(n, alpha, x, incx))
    b.close()


@pytest.mark.gpu
def test_gpu_device_pointer_scalars(cuda, built):
    torch = cuda
    n = 100003
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    y = rng.uniform(-1, 1, n).astype(np.float32)
    b = Blas(torch, device_mode=True)
    scal = torch.tensor([0.5, 0.0], dtype=torch.float32, device="cuda")
    tx, px = dev(torch, x)
    ty, py = dev(torch, y)
    assert b.L.cublasSaxpy_v2(b.h, n, C.c_void_p(scal.data_ptr()), px, 1, py, 1) == 0
    assert b.L.cublasSscal_v2(b.h, n, C.c_void_p(scal.data_ptr() + 4), px, 1) == 0
    out = torch.full((4,), -1.0, device="cuda")
    ridx = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    assert b.L.cublasSdot_v2(b.h, n, py, 1, py, 1, C.c_void_p(out.data_ptr())) == 0
    assert b.L.cublasIsamax_v2(b.h, n, py, 1, C.c_void_p(ridx.data_ptr())) == 0
    assert b.L.cublasSnrm2_v2(b.h, 0, py, 1, C.c_void_p(out.data_ptr() + 4)) == 0
    torch.cuda.synchronize()
    b.close()
    y1 = oracle.saxpy(n, 0.5, x, 1, y, 1)
    assert np.array_equal(back(ty, 0, n), y1)
    assert np.array_equal(back(tx, 0, n), np.zeros(n, np.float32))
    _, d64, mag = oracle.sreduce("dot", n, y1, 1, y1, 1)
    o = out.cpu().numpy()
    assert abs(o[0] - d64) <= 1e-5 * mag and o[1] == 0.0
    assert int(ridx.cpu()[0]) == oracle.isamax(n, y1, 1)


RED_CASES = [(1, 1, 1, 0), (1000, 1, 1, 0), (4097, 1, 1, 1), (1 << 22, 1, 1, 0),
             ((1 << 22) + 3, 1, 1, 1), (100003, 3, -2, 0), (5000, -1, 1, 0), (777, 0, 1, 0)]


@pytest.mark.gpu
@pytest.mark.parametrize("n,incx,incy,mis", RED_CASES)
def test_gpu_reductions(cuda, built, n, incx, incy, mis):
    torch = cuda
    rng = np.random.default_rng(n + incx)
    x = rng.standard_normal(span(n, incx)).astype(np.float32)
    y = rng.standard_normal(span(n, incy)).astype(np.float32)
    tx, px = dev(torch, x, mis)
    ty, py = dev(torch, y, mis)
    b = Blas(torch)
    res = C.c_float()
    idx = C.c_int()
    assert b.L.cublasSdot_v2(b.h, n, px, incx, py, incy, C.byref(res)) == 0
    _, d64, mag = oracle.sreduce("dot", n, x, incx, y, incy)
    assert abs(res.value - d64) <= 1e-5 * mag + 1e-30
    if incx > 0:
        assert b.L.cublasSnrm2_v2(b.h, n, px, incx, C.byref(res)) == 0
        _, d64, mag = oracle.sreduce("nrm2", n, x, incx)
        assert abs(res.value - d64) <= 1e-5 * d64 + 1e-30
        assert b.L.cublasSasum_v2(b.h, n, px, incx, C.byref(res)) == 0
        _, d64, mag = oracle.sreduce("asum", n, x, incx)
        assert abs(res.value - d64) <= 1e-5 * mag + 1e-30
    assert b.L.cublasIsamax_v2(b.h, n, px, incx, C.byref(idx)) == 0
    assert idx.value == oracle.isamax(n, x, incx)
    b.close()


@pytest.mark.gpu
def test_gpu_isamax_ties_nan_and_repeat_determinism(cuda, built):
    torch = cuda
    n = 3_000_017
    x = np.random.default_rng(2).uniform(-1, 1, n).astype(np.float32)
    x[[5, 2_000_000, 2_999_999]] = 7.0   # ties: the first wins
    x[[3, 1_500_000]] = np.nan           # never chosen
    x[2_500_000] = -7.0
    tx, px = dev(torch, x)
    b = Blas(torch)
    idx, res1, res2 = C.c_int(), C.c_float(), C.c_float()
    assert b.L.cublasIsamax_v2(b.h, n, px, 1, C.byref(idx)) == 0
    assert idx.value == 6 == oracle.isamax(n, x, 1)
    x2 = x.copy()
    x2[np.isnan(x2)] = 0.0
    t2, p2 = dev(torch, x2)
    assert b.L.cublasSasum_v2(b.h, n, p2, 1, C.byref(res1)) == 0
    assert b.L.cublasSasum_v2(b.h, n, p2, 1, C.byref(res2)) == 0
    assert res1.value == res2.value  # fixed combination order
    b.close()


GEMV_CASES = [  # trans, m, n, incx, incy, beta
    (False, 16, 12, 1, 1, 0.5), (False, 100000, 64, 1, 1, 0.0), (False, 300, 20000, 1, 1, -1.0),
    (False, 4097, 333, 2, -3, 0.25), (True, 20000, 300, 1, 1, 0.0), (True, 64, 100000, 1, 1, 0.5),
    (True, 3001, 777, -2, 1, 1.0), (True, 4096, 4096, 1, 1, 0.0), (False, 4096, 4096, 1, 1, 0.0)]


@pytest.mark.gpu
@pytest.mark.parametrize("trans,m,n,incx,incy,beta", GEMV_CASES)
def test_gpu_sgemv(cuda, built, trans, m, n, incx, incy, beta):
    torch = cuda
    rng = np.random.default_rng(m + 3 * n + incx)
    lda = m + (3 if m % 2 else 0)
    A = rng.uniform(-1, 1, lda * n).astype(np.float32)
    x_len, y_len = (m, n) if trans else (n, m)
    x = rng.uniform(-1, 1, span(x_len, incx)).astype(np.float32)
    y = rng.uniform(-1, 1, span(y_len, incy)).astype(np.float32)
    alpha = 1.25
    tA = torch.from_numpy(A).cuda()
    tx, px = dev(torch, x)
    ty, py = dev(torch, y)
    b = Blas(torch)
    st = b.L.cublasSgemv_v2(b.h, 1 if trans else 0, m, n, C.byref(C.c_float(alpha)),
                            C.c_void_p(tA.data_ptr()), lda, px, incx,
                            C.byref(C.c_float(beta)), py, incy)
    torch.cuda.synchronize()
    b.close()
    assert st == 0
    got = back(ty, 0, len(y)).astype(np.float64)
    want, exact, absv = oracle.sgemv(trans, m, n, alpha, A, lda, x, incx, beta, y, incy,
                                     threads=16)
    # the outputs in the reference's order of y
    pos = np.array([(i if incy >= 0 else i - y_len + 1) * incy for i in range(y_len)])
    err = np.abs(got[pos] - exact)
    assert np.all(err <= 1e-5 * absv + 1e-30), float((err / np.maximum(absv, 1e-30)).max())
    mask = np.ones(len(y), bool)
    mask[pos] = False
    assert np.array_equal(got[mask], y[mask].astype(np.float64))
    # one pass over the columns (no column chunks): the reference kernel's exact order
    if not trans and (n <= 256 or m >= 151552):
        assert np.array_equal(got[pos].astype(np.float32), want[pos])
