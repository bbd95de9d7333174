"""cuBLAS double precision: Daxpy/Dcopy/Dscal/Dswap/Ddot/Dnrm2/Dasum/Idamax, Dgemv,
Dgemm and DgemmStridedBatched, against the oracle's restatement of the reference-BLAS
definitions the reference's host CBLAS calls compute (oracle/blas64.cpp).

Bars: daxpy / dcopy / dscal / dswap bit-exact (the product and the sum of daxpy are
rounded separately, as written); idamax exact; ddot / dasum within
(n + 64) * 2^-52 of the sum of term magnitudes; dnrm2 within 64 * 2^-52 relative, with
no overflow or underflow for entries near 1e+300 or 1e-300; dgemv / dgemm within
(inner + 2) * 2^-52 of |alpha| (|op(A)| |op(B)|)_ij + |beta C_ij|.  The reference's
own known answers (tests/cublas_test.cpp:462-620) pin the oracle and the GPU path.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import stream_ptr

EPS = 2.0 ** -52
OPS = {False: capi.CUBLAS_OP_N, True: capi.CUBLAS_OP_T}


def dref(v):
    return C.byref(C.c_double(v))


# ------------------------------------------------------------------- CPU ---
def test_oracle_reference_known_answers():
    """tests/cublas_test.cpp:462-620 on the oracle: daxpy 6.5, ddot 1664, dnrm2
    sqrt(512), dasum 256, idamax 1, dscal 1.0, dgemv 67, dgemm 48."""
    x = np.full(128, 2.0)
    y = oracle.daxpy(128, 2.5, x, 1, np.full(128, 1.5), 1)
    assert np.all(y == 6.5)
    assert oracle.dreduce("dot", 128, x, 1, y, 1)[0] == 1664.0
    assert oracle.dreduce("nrm2", 128, x, 1)[0] == pytest.approx(np.sqrt(512.0), rel=1e-15)
    assert oracle.dreduce("asum", 128, x, 1)[0] == 256.0
    assert oracle.idamax(128, y, 1) == 1
    assert np.all(oracle.dscal(128, 0.5, x, 1) == 1.0)
    A = np.ones(256)
    assert np.all(oracle.dgemv(False, 16, 16, 2.0, A, 16, np.full(16, 2.0), 1, 1.0,
                               np.full(16, 3.0), 1)[0] == 67.0)
    assert np.all(oracle.dgemm(False, False, 16, 16, 16, 1.0, A, 16, np.full(256, 3.0), 16, 0.0,
                               np.zeros(256), 16)[0] == 48.0)


def test_oracle_element_rules():
    """Negative increments walk from the far end; idamax keeps the first maximum and a
    leading NaN wins; a zero-stride y accumulates in element order."""
    x = np.arange(1.0, 6.0)
    assert np.array_equal(oracle.dcopy(5, x, -1, np.zeros(5), 1), x[::-1])
    y = oracle.daxpy(5, 1.0, x, 1, np.zeros(1), 0)
    assert y[0] == 15.0
    assert oracle.idamax(4, np.array([1.0, -3.0, 3.0, 2.0]), 1) == 2
    assert oracle.idamax(3, np.array([np.nan, 5.0, 7.0]), 1) == 1
    assert oracle.idamax(3, np.array([1.0, np.nan, 0.5]), 1) == 1
    assert oracle.idamax(0, x, 1) == 0 and oracle.idamax(5, x, 0) == 0


def test_argument_checks(built):
    """Status codes in the reference's order, host-side (no device memory touched)."""
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    bad = C.c_void_p(12345)
    inv, ok, ni = (capi.CUBLAS_STATUS_INVALID_VALUE, capi.CUBLAS_STATUS_SUCCESS,
                   capi.CUBLAS_STATUS_NOT_INITIALIZED)
    assert L.cublasDaxpy_v2(bad, 4, dref(1.0), bad, 1, bad, 1) == ni
    assert L.cublasDaxpy_v2(h, 0, None, bad, 1, bad, 1) == ok        # n <= 0 before alpha
    assert L.cublasDaxpy_v2(h, 4, None, bad, 1, bad, 1) == inv
    assert L.cublasDaxpy_v2(h, 4, dref(0.0), bad, 1, bad, 1) == ok   # alpha 0: nothing read
    assert L.cublasDaxpy_v2(h, 4, dref(1.0), bad, 1, bad, 1) == inv  # unaddressable
    assert L.cublasDscal_v2(h, 4, None, bad, 0) == ok                # incx <= 0 first
    assert L.cublasDscal_v2(h, 4, None, bad, 1) == inv
    assert L.cublasDcopy_v2(h, -1, bad, 1, bad, 1) == ok
    assert L.cublasDswap_v2(h, 3, bad, 1, bad, 1) == inv
    r = C.c_double(7.0)
    assert L.cublasDdot_v2(h, 4, bad, 1, bad, 1, None) == inv
    assert L.cublasDdot_v2(h, 0, bad, 1, bad, 1, C.byref(r)) == ok and r.value == 0.0
    r.value = 7.0
    assert L.cublasDnrm2_v2(h, 5, bad, 0, C.byref(r)) == ok and r.value == 0.0
    r.value = 7.0
    assert L.cublasDasum_v2(h, 5, bad, -1, C.byref(r)) == ok and r.value == 0.0
    i = C.c_int(9)
    assert L.cublasIdamax_v2(h, 0, bad, 1, C.byref(i)) == ok and i.value == 0
    assert L.cublasIdamax_v2(h, 3, bad, 1, None) == inv
    one = dref(1.0)
    assert L.cublasDgemv_v2(h, 7, 4, 4, one, bad, 4, bad, 1, one, bad, 1) == inv   # bad op
    assert L.cublasDgemv_v2(h, 0, 4, 4, one, bad, 3, bad, 1, one, bad, 1) == inv   # lda < m
    assert L.cublasDgemv_v2(h, 0, 4, 4, one, bad, 4, bad, 0, one, bad, 1) == inv   # incx 0
    assert L.cublasDgemv_v2(h, 0, 0, 4, one, bad, 1, bad, 1, one, bad, 1) == ok    # empty
    assert L.cublasDgemm_v2(h, 0, 0, -1, 4, 4, one, bad, 4, bad, 4, one, bad, 4) == inv
    assert L.cublasDgemm_v2(h, 1, 0, 4, 4, 5, one, bad, 4, bad, 5, one, bad, 4) == inv  # lda < k
    assert L.cublasDgemm_v2(h, 0, 0, 4, 4, 4, None, bad, 4, bad, 4, one, bad, 4) == inv
    assert L.cublasDgemm_v2(h, 0, 0, 4, 0, 4, one, bad, 4, bad, 4, one, bad, 4) == ok
    assert L.cublasDgemmStridedBatched(h, 0, 0, 4, 4, 4, one, bad, 4, 16, bad, 4, 16, one, bad,
                                       4, 16, 0) == ok
    assert L.cublasDgemm_v2(h, 0, 0, 4, 4, 4, one, bad, 4, bad, 4, one, bad, 4) == inv
    assert L.cublasDestroy_v2(h) == 0


# ------------------------------------------------------------------- GPU ---
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


def dev(torch, a, offset=0):
    """Device copy of a float64 array starting `offset` elements into its buffer."""
    buf = torch.zeros(len(a) + offset + 2, dtype=torch.float64, device="cuda")
    if len(a):
        buf[offset:offset + len(a)] = torch.from_numpy(np.ascontiguousarray(a, np.float64))
    return buf, C.c_void_p(buf.data_ptr() + 8 * offset)


def span(n, inc):
    return 1 + (n - 1) * abs(inc) if n > 0 else 0


@pytest.mark.gpu
def test_gpu_reference_known_answers(cuda, built):
    """tests/cublas_test.cpp:462-620, the same calls in the same order."""
    torch = cuda
    b = Blas(torch)
    L, h = b.L, b.h
    dx, px = dev(torch, np.full(128, 2.0))
    dy, py = dev(torch, np.full(128, 1.5))
    assert L.cublasDaxpy_v2(h, 128, dref(2.5), px, 1, py, 1) == 0
    torch.cuda.synchronize()
    assert torch.all(dy[:128] == 6.5)
    r = C.c_double()
    assert L.cublasDdot_v2(h, 128, px, 1, py, 1, C.byref(r)) == 0 and r.value == 1664.0
    assert L.cublasDnrm2_v2(h, 128, px, 1, C.byref(r)) == 0
    assert abs(r.value - np.sqrt(512.0)) <= 1e-12
    assert L.cublasDasum_v2(h, 128, px, 1, C.byref(r)) == 0 and r.value == 256.0
    i = C.c_int()
    assert L.cublasIdamax_v2(h, 128, py, 1, C.byref(i)) == 0 and i.value == 1
    assert L.cublasDscal_v2(h, 128, dref(0.5), px, 1) == 0
    torch.cuda.synchronize()
    assert float(dx[0]) == 1.0
    dA, pA = dev(torch, np.ones(256))
    dvx, pvx = dev(torch, np.full(16, 2.0))
    dvy, pvy = dev(torch, np.full(16, 3.0))
    assert L.cublasDgemv_v2(h, 0, 16, 16, dref(2.0), pA, 16, pvx, 1, dref(1.0), pvy, 1) == 0
    torch.cuda.synchronize()
    assert torch.all(dvy[:16] == 67.0)
    dB, pB = dev(torch, np.full(256, 3.0))
    dC, pC = dev(torch, np.zeros(256))
    assert L.cublasDgemm_v2(h, 0, 0, 16, 16, 16, dref(1.0), pA, 16, pB, 16, dref(0.0), pC, 16) == 0
    torch.cuda.synchronize()
    assert torch.all(dC[:256] == 48.0)
    assert L.cublasDgeam(h, 1, 0, 16, 16, dref(2.0), pA, 16, dref(3.0), pB, 16, pC, 16) == 0
    torch.cuda.synchronize()
    assert torch.all(dC[:256] == 11.0)
    b.close()


ELT_CASES = [(1, 1, 1, 0), (7, 1, 1, 1), (1000, 1, 1, 0), (1000, 1, 1, 1), ((1 << 20) + 3, 1, 1, 0),
             (999, 2, 3, 0), (513, -1, 1, 0), (513, -2, -3, 1), (77, 0, 1, 0), (100, 1, 0, 0),
             (64, 0, 0, 0), (300, -1, 0, 1)]


@pytest.mark.gpu
@pytest.mark.parametrize("n,incx,incy,off", ELT_CASES)
def test_gpu_elementwise_bit_exact(cuda, built, n, incx, incy, off):
    torch = cuda
    rng = np.random.default_rng(n + 7 * incx + 13 * incy)
    x = rng.normal(size=span(n, incx))
    y = rng.normal(size=span(n, incy))
    b = Blas(torch)
    L, h = b.L, b.h
    for name in ("axpy", "copy", "scal", "swap"):
        dx, px = dev(torch, x, off)
        dy, py = dev(torch, y, off)
        if name == "axpy":
            assert L.cublasDaxpy_v2(h, n, dref(-1.75), px, incx, py, incy) == 0
            want_y, want_x = oracle.daxpy(n, -1.75, x, incx, y, incy), x
        elif name == "copy":
            assert L.cublasDcopy_v2(h, n, px, incx, py, incy) == 0
            want_y, want_x = oracle.dcopy(n, x, incx, y, incy), x
        elif name == "scal":
            assert L.cublasDscal_v2(h, n, dref(0.3), px, incx) == 0
            want_x, want_y = oracle.dscal(n, 0.3, x, incx), y
        else:
            assert L.cublasDswap_v2(h, n, px, incx, py, incy) == 0
            want_x, want_y = oracle.dswap(n, x, incx, y, incy)
        torch.cuda.synchronize()
        got_x = dx[off:off + len(x)].cpu().numpy()
        got_y = dy[off:off + len(y)].cpu().numpy()
        assert np.array_equal(got_x.view(np.uint64), want_x.view(np.uint64)), name
        assert np.array_equal(got_y.view(np.uint64), want_y.view(np.uint64)), name
    b.close()


RED_CASES = [(1, 1, 1), (2, 1, 1), (1001, 1, 1), ((1 << 22) + 5, 1, 1), (5000, 3, -2),
             (5000, -1, 1), (4097, 1, 0), (12345, 2, 2)]


@pytest.mark.gpu
@pytest.mark.parametrize("n,incx,incy", RED_CASES)
@pytest.mark.parametrize("device_mode", [False, True])
def test_gpu_reductions(cuda, built, n, incx, incy, device_mode):
    torch = cuda
    rng = np.random.default_rng(n + incx)
    x = rng.normal(size=span(n, incx)) * np.exp(rng.uniform(-5, 5, span(n, incx)))
    y = rng.normal(size=span(n, incy))
    dx, px = dev(torch, x, 1)
    dy, py = dev(torch, y)
    b = Blas(torch, device_mode)
    L, h = b.L, b.h
    res = torch.zeros(4, dtype=torch.float64, device="cuda")

    def out(i):
        return C.c_void_p(res.data_ptr() + 8 * i)

    r = [C.c_double() for _ in range(3)]
    ir = C.c_int()
    args = [out(i) for i in range(3)] + [out(3)] if device_mode else \
        [C.byref(v) for v in r] + [C.byref(ir)]
    assert L.cublasDdot_v2(h, n, px, incx, py, incy, args[0]) == 0
    assert L.cublasDnrm2_v2(h, n, px, incx, args[1]) == 0
    assert L.cublasDasum_v2(h, n, px, incx, args[2]) == 0
    assert L.cublasIdamax_v2(h, n, px, incx, args[3]) == 0
    torch.cuda.synchronize()
    if device_mode:
        vals = res.cpu().numpy()
        got = [float(vals[0]), float(vals[1]), float(vals[2])]
        got_i = int(res[3:4].view(torch.int32)[0].item())
    else:
        got = [v.value for v in r]
        got_i = ir.value
    _, dot_ext, dot_mag = oracle.dreduce("dot", n, x, incx, y, incy)
    _, nrm_ext, _ = oracle.dreduce("nrm2", n, x, incx)
    _, asum_ext, asum_mag = oracle.dreduce("asum", n, x, incx)
    assert abs(got[0] - dot_ext) <= (n + 64) * EPS * dot_mag
    assert abs(got[1] - nrm_ext) <= 64 * EPS * nrm_ext
    assert abs(got[2] - asum_ext) <= (n + 64) * EPS * asum_mag
    assert got_i == oracle.idamax(n, x, incx)
    b.close()


@pytest.mark.gpu
def test_gpu_reduction_special_values(cuda, built):
    """dnrm2 without overflow / underflow (entries around 1e+300, 1e-300, mixed),
    NaN and inf propagation, idamax ties and NaN rules."""
    torch = cuda
    b = Blas(torch)
    L, h = b.L, b.h
    r = C.c_double()
    cases = [np.full(1000, 1e300), np.full(1000, 1e-300), np.concatenate(
        [np.full(10, 3e200), np.full(10, 1.0), np.full(10, 2e-200)]),
        np.concatenate([np.full(10, 1.0), np.full(10, 2e-200)])]
    for x in cases:
        dx, px = dev(torch, x)
        assert L.cublasDnrm2_v2(h, len(x), px, 1, C.byref(r)) == 0
        want = oracle.dreduce("nrm2", len(x), x, 1)[1]
        assert np.isfinite(r.value) and abs(r.value - want) <= 64 * EPS * want, (r.value, want)
    for bad, check in ((np.nan, np.isnan), (np.inf, np.isinf)):
        x = np.ones(5000)
        x[4000] = bad
        dx, px = dev(torch, x)
        assert L.cublasDnrm2_v2(h, 5000, px, 1, C.byref(r)) == 0 and check(r.value)
        assert L.cublasDasum_v2(h, 5000, px, 1, C.byref(r)) == 0 and check(r.value)
    i = C.c_int()
    for x in (np.array([1.0, -3.0, 3.0, 2.0]), np.array([np.nan, 5.0, 7.0]),
              np.array([1.0, np.nan, 0.5, np.nan]), np.concatenate([np.ones(70000), [-2.0],
                                                                    np.full(5, 2.0)])):
        dx, px = dev(torch, x)
        assert L.cublasIdamax_v2(h, len(x), px, 1, C.byref(i)) == 0
        assert i.value == oracle.idamax(len(x), x, 1), x[:4]
    b.close()


GEMV_CASES = [(1, 1, 1, 1), (100, 37, 1, 1), (37, 100, 2, -1), (4096, 4096, 1, 1),
              (100000, 37, 1, 1), (37, 100000, 1, 1), (513, 1025, -3, 2)]


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,incx,incy", GEMV_CASES)
@pytest.mark.parametrize("trans", [False, True])
def test_gpu_dgemv(cuda, built, m, n, incx, incy, trans):
    torch = cuda
    rng = np.random.default_rng(m * 3 + n)
    lda = m + 3
    A = rng.normal(size=lda * n)
    xl, yl = (m, n) if trans else (n, m)
    x = rng.normal(size=span(xl, incx))
    y = rng.normal(size=span(yl, incy))
    b = Blas(torch)
    for alpha, beta in ((1.25, -0.5), (0.5, 0.0), (0.0, 2.0)):
        A_in, y_in = A.copy(), y.copy()
        if alpha == 0.0:
            A_in[::7] = np.nan  # not read
        if beta == 0.0:
            y_in[:] = np.nan    # not read
        dA, pA = dev(torch, A_in)
        dx, px = dev(torch, x)
        dy, py = dev(torch, y_in)
        assert b.L.cublasDgemv_v2(b.h, OPS[trans], m, n, dref(alpha), pA, lda, px, incx,
                                  dref(beta), py, incy) == 0
        torch.cuda.synchronize()
        got = dy[:len(y)].cpu().numpy()
        want, bound = oracle.dgemv(trans, m, n, alpha, A_in if alpha else A, lda, x, incx, beta,
                                   y_in, incy)
        idx = np.array([i * incy if incy >= 0 else (i - yl + 1) * incy for i in range(yl)])
        err = np.abs(got[idx] - want[idx])
        assert np.all(err <= (max(m, n) + 2) * EPS * bound + 1e-300), (alpha, beta, err.max())
    b.close()


GEMM_CASES = [(1, 1, 1, 1, 0), (33, 65, 17, 1, 3), (128, 128, 8, 1, 0), (300, 520, 1000, 2, 5),
              (1024, 1024, 1024, 1, 0), (129, 2000, 64, 3, 1), (2048, 2048, 2048, 1, 0)]


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,batch,pad", GEMM_CASES)
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_gpu_dgemm(cuda, built, m, n, k, batch, pad, ta, tb):
    torch = cuda
    rng = np.random.default_rng(m + 3 * n + 7 * k + 11 * ta + 13 * tb)
    lda = (k if ta else m) + pad
    ldb = (n if tb else k) + pad
    ldc = m + pad
    sa = lda * (m if ta else k) + 3
    sb = ldb * (k if tb else n) + 5
    sc = ldc * n + 7
    A = rng.uniform(-1, 1, sa * batch)
    B = rng.uniform(-1, 1, sb * batch)
    C0 = rng.uniform(-1, 1, sc * batch)
    alpha, beta = 1.5, (0.0 if k % 2 else -0.75)
    dA, pA = dev(torch, A)
    dB, pB = dev(torch, B)
    dC, pC = dev(torch, C0)
    b = Blas(torch)
    assert b.L.cublasDgemmStridedBatched(b.h, OPS[ta], OPS[tb], m, n, k, dref(alpha), pA, lda, sa,
                                         pB, ldb, sb, dref(beta), pC, ldc, sc, batch) == 0
    torch.cuda.synchronize()
    b.close()
    got = dC[:len(C0)].cpu().numpy()
    total = m * n * batch
    ne = min(total, 20000)
    pick = rng.choice(total, ne, replace=False) if ne < total else np.arange(total)
    z, rem = pick // (m * n), pick % (m * n)
    rows, cols = (rem % m).astype(np.int32), rem // m
    want, bound = oracle.dgemm(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C0, ldc,
                               stride_a=sa, stride_b=sb, stride_c=sc, batch=batch,
                               entries=(rows, (z * n + cols).astype(np.int32)), threads=16)
    flat = z * sc + cols * ldc + rows
    err = np.abs(got[flat] - want[flat])
    assert np.all(err <= (k + 2) * EPS * bound), float((err / bound).max())
    mask = np.ones(len(got), bool)
    for zz in range(batch):
        mask[(zz * sc + np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).reshape(-1)] = False
    assert np.array_equal(got[mask], C0[mask])


@pytest.mark.gpu
def test_gpu_dgemm_scalar_rules_and_device_mode(cuda, built):
    """alpha == 0 reads neither A nor B (C = beta C), beta == 0 does not read C, k == 0
    gives beta C, and device-pointer scalars give the host-mode result."""
    torch = cuda
    m, n, k = 200, 150, 60
    rng = np.random.default_rng(3)
    A, B, C0 = rng.normal(size=m * k), rng.normal(size=k * n), rng.normal(size=m * n)
    nanA = np.full(m * k, np.nan)
    b = Blas(torch)
    dA, pA = dev(torch, nanA)
    dB, pB = dev(torch, B)
    dC, pC = dev(torch, C0)
    assert b.L.cublasDgemm_v2(b.h, 0, 0, m, n, k, dref(0.0), pA, m, pB, k, dref(2.0), pC, m) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dC[:m * n].cpu().numpy(), 2.0 * C0)
    dA, pA = dev(torch, A)
    dC, pC = dev(torch, np.full(m * n, np.nan))
    assert b.L.cublasDgemm_v2(b.h, 0, 0, m, n, k, dref(1.0), pA, m, pB, k, dref(0.0), pC, m) == 0
    torch.cuda.synchronize()
    got = dC[:m * n].cpu().numpy()
    want, bound = oracle.dgemm(False, False, m, n, k, 1.0, A, m, B, k, 0.0, np.zeros(m * n), m)
    assert np.all(np.abs(got - want) <= (k + 2) * EPS * bound)
    dC, pC = dev(torch, C0)
    assert b.L.cublasDgemm_v2(b.h, 0, 0, m, n, 0, dref(1.0), pA, m, pB, 1, dref(-1.0), pC, m) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dC[:m * n].cpu().numpy(), -C0)
    b.close()
    bd = Blas(torch, device_mode=True)
    sc = torch.tensor([1.5, -0.25], dtype=torch.float64, device="cuda")
    dC, pC = dev(torch, C0)
    assert bd.L.cublasDgemm_v2(bd.h, 1, 1, m, n, k, C.c_void_p(sc.data_ptr()), pA, k, pB, n,
                               C.c_void_p(sc.data_ptr() + 8), pC, m) == 0
    torch.cuda.synchronize()
    bd.close()
    got = dC[:m * n].cpu().numpy()
    want, bound = oracle.dgemm(True, True, m, n, k, 1.5, A, k, B, n, -0.25, C0, m)
    assert np.all(np.abs(got - want) <= (k + 2) * EPS * bound)
