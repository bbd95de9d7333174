"""cuBLAS geam (fp32 Sgeam, fp64 Dgeam): C = alpha * op(A) + beta * op(B).

CPU: the oracle against the reference's known answers (tests/cublas_test.cpp:443-455
for Sgeam, :599-612 for Dgeam) and against numpy's separately rounded products and
sum; the entry points' argument checks (libraries/blas/src/cublas_level3.mm:623-640,
:825-841).  GPU (marked): the CUDA kernel through the C ABI against the oracle,
bit-exact (same per-element formula, each multiply and add rounded on its own).
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import stream_ptr

F32, F64 = np.float32, np.float64


def test_oracle_reference_geam_pins():
    """Sgeam(T, N) 8 x 8, alpha 2, A = 1, beta 3, B = 0.5 gives 3.5; Dgeam(T, N) 16 x 16,
    A = 1, B = 3 gives 11."""
    c = oracle.geam(F32, True, False, 8, 8, 2.0, np.ones(64, F32), 8, 3.0,
                    np.full(64, 0.5, F32), 8, np.zeros(64, F32), 8)
    assert np.all(c == 3.5)
    d = oracle.geam(F64, True, False, 16, 16, 2.0, np.ones(256), 16, 3.0, np.full(256, 3.0),
                    16, np.zeros(256), 16)
    assert np.all(d == 11.0)


def col_major(rng, rows, cols, ld, dtype):
    """A column-major rows x cols matrix with leading dimension ld (padding = NaN)."""
    buf = np.full(ld * (cols - 1) + rows, np.nan, dtype)
    vals = rng.uniform(-1, 1, (cols, rows)).astype(dtype)
    for c in range(cols):
        buf[c * ld:c * ld + rows] = vals[c]
    return buf, vals.T  # vals.T[r, c] = element (r, c)


def numpy_geam(dtype, alpha, opa, beta, opb):
    """Each product rounded to dtype, then the sum rounded (separate operations)."""
    ta = (dtype(alpha) * opa).astype(dtype) if alpha != 0 else np.zeros_like(opb, dtype)
    tb = (dtype(beta) * opb).astype(dtype) if beta != 0 else np.zeros_like(opa, dtype)
    return (ta + tb).astype(dtype)


@pytest.mark.parametrize("dtype", [F32, F64])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_oracle_geam_against_numpy(dtype, ta, tb):
    rng = np.random.default_rng(3)
    m, n = 37, 23
    A, a = col_major(rng, n if ta else m, m if ta else n, (n if ta else m) + 3, dtype)
    B, b = col_major(rng, n if tb else m, m if tb else n, (n if tb else m) + 1, dtype)
    ldc = m + 2
    Cb = np.full(ldc * (n - 1) + m, -7.0, dtype)
    got = oracle.geam(dtype, ta, tb, m, n, 1.5, A, (n if ta else m) + 3, -0.75, B,
                      (n if tb else m) + 1, Cb, ldc)
    want = numpy_geam(dtype, 1.5, a.T if ta else a, -0.75, b.T if tb else b)
    for c in range(n):
        assert np.array_equal(got[c * ldc:c * ldc + m], want[:, c])
        if c < n - 1:
            assert np.all(got[c * ldc + m:(c + 1) * ldc] == -7.0)  # padding untouched


def test_geam_argument_checks(built):
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    one_f, one_d = C.byref(C.c_float(1.0)), C.byref(C.c_double(1.0))
    zero_f = C.byref(C.c_float(0.0))
    p = C.c_void_p(256)
    bad = C.c_void_p(12345)
    inv, ok = capi.CUBLAS_STATUS_INVALID_VALUE, capi.CUBLAS_STATUS_SUCCESS
    for fn, one in ((L.cublasSgeam, one_f), (L.cublasDgeam, one_d)):
        assert fn(bad, 0, 0, 4, 4, one, p, 4, one, p, 4, p, 4) == \
            capi.CUBLAS_STATUS_NOT_INITIALIZED
        assert fn(h, 3, 0, 4, 4, one, p, 4, one, p, 4, p, 4) == inv      # bad op
        assert fn(h, 0, 0, -1, 4, one, p, 4, one, p, 4, p, 4) == inv     # m < 0
        assert fn(h, 0, 0, 4, 4, None, p, 4, one, p, 4, p, 4) == inv     # null alpha
        assert fn(h, 0, 0, 4, 4, one, p, 4, None, p, 4, p, 4) == inv     # null beta
        assert fn(h, 0, 0, 4, 6, one, p, 3, one, p, 4, p, 4) == inv      # lda < m (op N)
        assert fn(h, 1, 0, 4, 6, one, p, 4, one, p, 4, p, 4) == inv      # lda < n (op T)
        assert fn(h, 0, 1, 4, 6, one, p, 4, one, p, 5, p, 4) == inv      # ldb < n (op T)
        assert fn(h, 0, 0, 4, 4, one, p, 4, one, p, 4, p, 3) == inv      # ldc < m
        assert fn(h, 0, 0, 0, 4, one, p, 1, one, p, 1, p, 1) == ok       # empty
        assert fn(h, 0, 0, 4, 4, one, p, 4, one, p, 4, p, 4) == inv      # unaddressable
    # Sgeam with an empty output and null C succeeds; Dgeam rejects a null C first
    assert L.cublasSgeam(h, 0, 0, 0, 4, one_f, p, 1, one_f, p, 1, None, 1) == ok
    assert L.cublasDgeam(h, 0, 0, 0, 4, one_d, p, 1, one_d, p, 1, None, 1) == inv
    # an unaddressable C is refused even when both scalars are 0 (the null A and B
    # are then not examined; tests/test_geam.py::test_geam_zero_scalars_skip_operands
    # shows on the GPU that they are skipped)
    assert L.cublasSgeam(h, 0, 0, 4, 4, zero_f, None, 4, zero_f, None, 4, p, 4) == inv
    assert L.cublasDestroy_v2(h) == 0


# --------------------------------------------------------------------- GPU --
CASES = [
    # m, n, ta, tb, lda pad, ldb pad, ldc pad, alpha, beta
    (1, 1, False, False, 0, 0, 0, 2.0, 3.0),
    (8, 8, True, False, 0, 0, 0, 2.0, 3.0),
    (33, 65, True, True, 1, 2, 3, -1.25, 0.5),
    (1000, 777, False, True, 0, 5, 0, 1.0, 1.0),
    (777, 1000, True, False, 7, 0, 1, 0.3, -2.0),
    (4099, 131, False, False, 3, 0, 0, 0.0, 1.5),     # alpha 0: A not read
    (129, 4099, True, True, 0, 0, 0, -0.7, 0.0),       # beta 0: B not read
    (64, 64, False, False, 0, 0, 0, 0.0, 0.0),         # both 0: C = +0
    # op N,N with 16-byte aligned columns: the vectorised column-streaming kernel
    (1028, 300, False, False, 0, 4, 8, 1.5, -0.25),
    (2048, 33, False, False, 0, 0, 0, 0.0, 2.0),       # alpha 0 on that kernel
    (512, 77, False, False, 4, 0, 0, 1.25, 0.0),       # beta 0 on that kernel
    (1024, 40, False, False, 2, 0, 0, 1.0, 1.0),       # lda not a multiple of 4: tiled kernel
]


def run_case(torch, dtype, case, device_mode=False):
    m, n, ta, tb, pa, pb, pc, alpha, beta = case
    rng = np.random.default_rng(m * 7919 + n)
    lda, ldb, ldc = (n if ta else m) + pa, (n if tb else m) + pb, m + pc
    A, _ = col_major(rng, n if ta else m, m if ta else n, lda, dtype)
    B, _ = col_major(rng, n if tb else m, m if tb else n, ldb, dtype)
    A = np.nan_to_num(A, nan=0.0)
    B = np.nan_to_num(B, nan=0.0)
    if alpha == 0:
        A[:] = np.nan  # an unread operand's NaNs must not reach C
    if beta == 0:
        B[:] = np.nan
    Cb = np.full(ldc * (n - 1) + m, 9.0, dtype)
    want = oracle.geam(dtype, ta, tb, m, n, alpha, A, lda, beta, B, ldb, Cb, ldc)
    tdt = torch.float32 if dtype == F32 else torch.float64
    dA, dB, dC = (torch.from_numpy(x.copy()).to("cuda") for x in (A, B, Cb))
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(stream_ptr(torch))) == 0
    ctype = C.c_float if dtype == F32 else C.c_double
    if device_mode:
        assert L.cublasSetPointerMode_v2(h, capi.CUBLAS_POINTER_MODE_DEVICE) == 0
        sc = torch.tensor([alpha, beta], dtype=tdt, device="cuda")
        pa_, pb_ = C.c_void_p(sc.data_ptr()), C.c_void_p(sc.data_ptr() + sc.element_size())
    else:
        pa_, pb_ = C.byref(ctype(alpha)), C.byref(ctype(beta))
    fn = L.cublasSgeam if dtype == F32 else L.cublasDgeam
    st = fn(h, int(ta), int(tb), m, n, pa_, C.c_void_p(dA.data_ptr()), lda, pb_,
            C.c_void_p(dB.data_ptr()), ldb, C.c_void_p(dC.data_ptr()), ldc)
    assert st == 0
    torch.cuda.synchronize()
    assert L.cublasDestroy_v2(h) == 0
    got = dC.cpu().numpy()
    udt = np.uint32 if dtype == F32 else np.uint64
    assert np.array_equal(got.view(udt), want.view(udt)), f"case {case}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [F32, F64])
@pytest.mark.parametrize("case", CASES)
def test_geam_bit_exact(cuda, built, dtype, case):
    run_case(cuda, dtype, case)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [F32, F64])
def test_geam_device_pointer_mode(cuda, built, dtype):
    run_case(cuda, dtype, (300, 517, True, False, 2, 1, 4, 1.75, -0.5), device_mode=True)
    run_case(cuda, dtype, (300, 517, False, True, 0, 0, 0, 0.0, 2.5), device_mode=True)


@pytest.mark.gpu
def test_sgeam_in_place_and_large_transpose(cuda, built):
    """C = A in place (op N, lda = ldc), then an 8192 x 6144 A^T + B against torch's
    separately rounded elementwise product and sum on the GPU."""
    torch = cuda
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(stream_ptr(torch))) == 0
    g = torch.Generator(device="cuda").manual_seed(5)
    m, n = 1500, 700
    A = torch.rand(n, m, device="cuda", generator=g)  # column-major m x n, ld m
    B = torch.rand(n, m, device="cuda", generator=g)
    want = (A * 2.0) + (B * -3.0)
    st = L.cublasSgeam(h, 0, 0, m, n, C.byref(C.c_float(2.0)), C.c_void_p(A.data_ptr()), m,
                       C.byref(C.c_float(-3.0)), C.c_void_p(B.data_ptr()), m,
                       C.c_void_p(A.data_ptr()), m)
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(A, want)
    m, n = 8192, 6144
    A = torch.rand(m, n, device="cuda", generator=g)   # column-major n x m (op T), ld n
    B = torch.rand(n, m, device="cuda", generator=g)   # column-major m x n, ld m
    Cm = torch.empty(n, m, device="cuda")
    st = L.cublasSgeam(h, 1, 0, m, n, C.byref(C.c_float(0.5)), C.c_void_p(A.data_ptr()), n,
                       C.byref(C.c_float(1.25)), C.c_void_p(B.data_ptr()), m,
                       C.c_void_p(Cm.data_ptr()), m)
    assert st == 0
    torch.cuda.synchronize()
    want = (A.t() * 0.5) + (B * 1.25)
    assert torch.equal(Cm, want)
    assert L.cublasDestroy_v2(h) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [F32, F64])
def test_geam_zero_scalars_skip_operands(cuda, built, dtype):
    """Host pointer mode, alpha = beta = 0, A = B = NULL and a valid C: the operands are
    neither checked nor read (cublas_level3.mm:633-640) and C becomes +0."""
    torch = cuda
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(stream_ptr(torch))) == 0
    tdt = torch.float32 if dtype == F32 else torch.float64
    ctype = C.c_float if dtype == F32 else C.c_double
    fn = L.cublasSgeam if dtype == F32 else L.cublasDgeam
    c = torch.full((37 * 19,), -5.0, dtype=tdt, device="cuda")
    zero = C.byref(ctype(0.0))
    assert fn(h, 0, 1, 37, 19, zero, None, 37, zero, None, 19, C.c_void_p(c.data_ptr()), 37) == 0
    torch.cuda.synchronize()
    got = c.cpu().numpy()
    assert np.all(got == 0.0) and not np.any(np.signbit(got))
    # only alpha 0: A NULL is fine, B is read
    b = torch.full((37 * 19,), 2.0, dtype=tdt, device="cuda")
    assert fn(h, 0, 0, 37, 19, zero, None, 37, C.byref(ctype(0.5)), C.c_void_p(b.data_ptr()),
              37, C.c_void_p(c.data_ptr()), 37) == 0
    torch.cuda.synchronize()
    assert np.all(c.cpu().numpy() == 1.0)
    assert L.cublasDestroy_v2(h) == 0


@pytest.mark.gpu
def test_geam_device_mode_requires_both_operands(cuda, built):
    """Documented difference: in device pointer mode the scalars are read on the GPU
    inside the kernel, so both operands must be addressable even when a scalar is 0.
    The reference synchronises the stream, reads the scalar on the host and skips the
    operand; here a NULL operand is CUBLAS_STATUS_INVALID_VALUE."""
    torch = cuda
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(stream_ptr(torch))) == 0
    assert L.cublasSetPointerMode_v2(h, capi.CUBLAS_POINTER_MODE_DEVICE) == 0
    sc = torch.tensor([0.0, 1.0], dtype=torch.float32, device="cuda")
    b = torch.ones(64, device="cuda")
    c = torch.zeros(64, device="cuda")
    st = L.cublasSgeam(h, 0, 0, 8, 8, C.c_void_p(sc.data_ptr()), None, 8,
                       C.c_void_p(sc.data_ptr() + 4), C.c_void_p(b.data_ptr()), 8,
                       C.c_void_p(c.data_ptr()), 8)
    assert st == capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasDestroy_v2(h) == 0


@pytest.mark.gpu
def test_geam_refuses_racing_overlap(cuda, built):
    """In-place use is supported when C is the operand itself, not transposed, with the
    same leading dimension.  C overlapping a transposed operand, or the same memory at
    a different leading dimension, would race between tiles and is refused."""
    torch = cuda
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(stream_ptr(torch))) == 0
    one = C.byref(C.c_float(1.0))
    zero = C.byref(C.c_float(0.0))
    buf = torch.rand(256 * 256 + 512, device="cuda")
    b = torch.rand(256 * 256, device="cuda")
    p = C.c_void_p(buf.data_ptr())
    pb = C.c_void_p(b.data_ptr())
    inv = capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSgeam(h, 1, 0, 256, 256, one, p, 256, one, pb, 256, p, 256) == inv  # C == A^T
    assert L.cublasSgeam(h, 0, 0, 256, 256, one, p, 257, one, pb, 256, p, 256) == inv  # other ld
    shifted = C.c_void_p(buf.data_ptr() + 4 * 100)
    assert L.cublasSgeam(h, 0, 0, 256, 256, one, p, 256, one, pb, 256, shifted, 256) == inv
    # alpha 0 in host mode: A is not read, so its overlap does not matter
    assert L.cublasSgeam(h, 1, 0, 256, 256, zero, p, 256, one, pb, 256, p, 256) == 0
    # C == B, op N, same ld: supported in place
    want = buf[:256 * 256].clone() * 0 + b  # alpha 0 above wrote C = B
    torch.cuda.synchronize()
    assert torch.equal(buf[:256 * 256], want)
    assert L.cublasSgeam(h, 0, 0, 256, 256, zero, None, 256, C.byref(C.c_float(2.0)), p, 256,
                         p, 256) == 0
    torch.cuda.synchronize()
    assert torch.equal(buf[:256 * 256], want * 2.0)
    assert L.cublasDestroy_v2(h) == 0
