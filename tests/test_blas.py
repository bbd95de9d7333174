"""cublasSgemm / cublasSgemmStridedBatched / cublasGemmEx / cublasGemmStridedBatchedEx /
cublasHgemm.

CPU: the oracle against the reference's known answers, and the handle logic.
GPU (marked): the CUDA paths through the C ABI against the oracle.  Bar: fp32
within 1e-5 normwise relative error of the double-accumulated product; 16-bit
outputs within 1e-2 normwise relative error.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import stream_ptr

OPS = {False: capi.CUBLAS_OP_N, True: capi.CUBLAS_OP_T}


def ref_case_inputs(m, n, k, ta, tb):
    """tests/cublas_test.cpp:299-315."""
    lda = k if ta else m
    ldb = n if tb else k
    A = ((np.arange(lda * (m if ta else k)) % 13) + 1).astype(np.float32) * np.float32(0.1)
    B = ((np.arange(ldb * (k if tb else n)) % 11) + 1).astype(np.float32) * np.float32(0.1)
    C = np.full(m * n, 2.0, np.float32)
    return A, lda, B, ldb, C


def op_matrix(X, ld, rows, cols, trans):
    """op(X) as a dense (rows x cols) float64 array from a column-major buffer."""
    if trans:
        return X.reshape(-1, ld)[:rows, :cols].astype(np.float64)
    return X.reshape(-1, ld).T[:rows, :cols].astype(np.float64)


@pytest.mark.parametrize("m,n,k,ta,tb", [(32, 24, 40, False, False), (32, 24, 40, True, False),
                                         (32, 24, 40, False, True), (32, 24, 40, True, True),
                                         (128, 96, 64, False, False), (96, 128, 64, True, False)])
def test_oracle_reference_sgemm_pin(m, n, k, ta, tb):
    """tests/cublas_test.cpp:299-380 (alpha 1.25, beta 0.5, C = 2, abs tol 1e-2)."""
    A, lda, B, ldb, C = ref_case_inputs(m, n, k, ta, tb)
    oracle.gemm("f32", ta, tb, m, n, k, 1.25, A, lda, B, ldb, 0.5, C, m)
    want = 1.25 * op_matrix(A, lda, m, k, ta) @ op_matrix(B, ldb, k, n, tb) + 1.0
    assert np.max(np.abs(C.reshape(n, m).T - want)) < 1e-2


def test_oracle_reference_hgemm_and_batched_pins():
    """tests/cublas_test.cpp:383-441: 16^3 HGEMM of 0.5 * 0.25 -> 2.0; batch-3 8^3 SGEMM
    of 1 * 0.5 -> 4.0."""
    H = np.zeros(256, np.uint16)
    oracle.gemm("f16", False, False, 16, 16, 16, 1.0, oracle.half_bits(np.full(256, 0.5)), 16,
                oracle.half_bits(np.full(256, 0.25)), 16, 0.0, H, 16)
    assert np.all(np.abs(H.view(np.float16).astype(np.float32) - 2.0) < 1e-2)
    Cb = np.zeros(3 * 64, np.float32)
    oracle.gemm("f32", False, False, 8, 8, 8, 1.0, np.ones(192, np.float32), 8,
                np.full(192, 0.5, np.float32), 8, 0.0, Cb, 8, stride_a=64, stride_b=64,
                stride_c=64, batch=3)
    assert np.all(np.abs(Cb - 4.0) < 1e-4)


def test_handle_logic(built):
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(None) == capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasCreate_v2(C.byref(h)) == 0
    v = C.c_int()
    assert L.cublasGetVersion_v2(h, C.byref(v)) == 0 and v.value == 12000
    assert L.cublasSetPointerMode_v2(h, 1) == 0
    assert L.cublasGetPointerMode_v2(h, C.byref(v)) == 0 and v.value == 1
    assert L.cublasSetPointerMode_v2(h, 2) == capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSetMathMode(h, 3) == 0
    assert L.cublasGetMathMode(h, C.byref(v)) == 0 and v.value == 3
    assert L.cublasSetMathMode(h, 4) == capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSetPointerMode_v2(h, 0) == 0
    assert L.cublasGetStatusName(15) == b"CUBLAS_STATUS_NOT_SUPPORTED"
    one = C.byref(C.c_float(1.0))
    p = C.c_void_p(256)
    # argument checks (cublas_level3.mm:515-531)
    assert L.cublasSgemm_v2(h, 3, 0, 4, 4, 4, one, p, 4, p, 4, one, p, 4) == \
        capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSgemm_v2(h, 0, 0, -1, 4, 4, one, p, 4, p, 4, one, p, 4) == \
        capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSgemm_v2(h, 0, 0, 4, 4, 4, one, p, 3, p, 4, one, p, 4) == \
        capi.CUBLAS_STATUS_INVALID_VALUE
    assert L.cublasSgemm_v2(h, 0, 0, 4, 4, 4, None, p, 4, p, 4, one, p, 4) == \
        capi.CUBLAS_STATUS_INVALID_VALUE
    # zero-size problems succeed without touching memory
    assert L.cublasSgemm_v2(h, 0, 0, 0, 4, 4, one, p, 1, p, 4, one, p, 1) == 0
    # unaddressable operands are rejected before launch
    assert L.cublasSgemm_v2(h, 0, 0, 4, 4, 4, one, p, 4, p, 4, one, p, 4) == \
        capi.CUBLAS_STATUS_INVALID_VALUE
    # unsupported type combinations (cublas_level3.mm:607)
    assert L.cublasGemmEx(h, 0, 0, 4, 4, 4, one, p, 0, 4, p, 2, 4, one, p, 0, 4, 68, -1) == \
        capi.CUBLAS_STATUS_NOT_SUPPORTED
    assert L.cublasDestroy_v2(h) == 0
    assert L.cublasDestroy_v2(h) == capi.CUBLAS_STATUS_NOT_INITIALIZED
    assert L.cublasSgemm_v2(h, 0, 0, 4, 4, 4, one, p, 4, p, 4, one, p, 4) == \
        capi.CUBLAS_STATUS_NOT_INITIALIZED


# --------------------------------------------------------------------- GPU --
class Blas:
    def __init__(self, torch):
        self.L = capi.cublas()
        self.h = C.c_void_p()
        assert self.L.cublasCreate_v2(C.byref(self.h)) == 0
        assert self.L.cublasSetStream_v2(self.h, C.c_void_p(stream_ptr(torch))) == 0

    def close(self):
        assert self.L.cublasDestroy_v2(self.h) == 0


def normwise(got, want):
    return np.linalg.norm(got.astype(np.float64) - want) / max(np.linalg.norm(want), 1e-300)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,ta,tb", [(32, 24, 40, False, False), (32, 24, 40, True, False),
                                         (32, 24, 40, False, True), (32, 24, 40, True, True),
                                         (128, 96, 64, False, False), (96, 128, 64, True, False)])
def test_gpu_reference_sgemm_pin(cuda, built, m, n, k, ta, tb):
    torch = cuda
    A, lda, B, ldb, C0 = ref_case_inputs(m, n, k, ta, tb)
    b = Blas(torch)
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C0))
    al, be = C.c_float(1.25), C.c_float(0.5)
    st = b.L.cublasSgemm_v2(b.h, OPS[ta], OPS[tb], m, n, k, C.byref(al), C.c_void_p(dA.data_ptr()),
                            lda, C.c_void_p(dB.data_ptr()), ldb, C.byref(be),
                            C.c_void_p(dC.data_ptr()), m)
    b.close()
    assert st == 0
    want = 1.25 * op_matrix(A, lda, m, k, ta) @ op_matrix(B, ldb, k, n, tb) + 1.0
    got = dC.cpu().numpy().reshape(n, m).T
    assert np.max(np.abs(got - want)) < 1e-2


def rand_case(rng, m, n, k, ta, tb, batch, pad=3):
    lda = (k if ta else m) + pad
    ldb = (n if tb else k) + pad
    ldc = m + pad
    sa = lda * (m if ta else k) + 5
    sb = ldb * (k if tb else n) + 7
    sc = ldc * n + 11
    A = rng.uniform(-1, 1, sa * batch).astype(np.float32)
    B = rng.uniform(-1, 1, sb * batch).astype(np.float32)
    Cm = rng.uniform(-1, 1, sc * batch).astype(np.float32)
    return A, lda, sa, B, ldb, sb, Cm, ldc, sc


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 3), (33, 65, 17), (128, 128, 8),
                                   (130, 257, 129), (300, 64, 1000), (1024, 1024, 1024)])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_gpu_sgemm_matches_oracle(cuda, built, m, n, k, ta, tb):
    torch = cuda
    rng = np.random.default_rng(m * 31 + n * 7 + k)
    batch = 2 if m * n * k < (1 << 24) else 1
    A, lda, sa, B, ldb, sb, C0, ldc, sc = rand_case(rng, m, n, k, ta, tb, batch)
    alpha, beta = 0.75, (0.0 if k % 2 else -1.5)
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C0))
    b = Blas(torch)
    st = b.L.cublasSgemmStridedBatched(b.h, OPS[ta], OPS[tb], m, n, k,
                                       C.byref(C.c_float(alpha)), C.c_void_p(dA.data_ptr()), lda,
                                       sa, C.c_void_p(dB.data_ptr()), ldb, sb,
                                       C.byref(C.c_float(beta)), C.c_void_p(dC.data_ptr()), ldc,
                                       sc, batch)
    b.close()
    assert st == 0
    got = dC.cpu().numpy()
    want = oracle.gemm("f32", ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C0.copy(), ldc,
                       stride_a=sa, stride_b=sb, stride_c=sc, batch=batch, accum_f64=True)
    for z in range(batch):
        idx = (z * sc + np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).reshape(-1)
        assert normwise(got[idx], want[idx].astype(np.float64)) <= 1e-5
    # entries outside the m x n windows are untouched
    mask = np.ones(len(got), bool)
    for z in range(batch):
        mask[(z * sc + np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).reshape(-1)] = False
    assert np.array_equal(got[mask], C0[mask])


def _op_dense(X, ld, stride, z, rows, cols, trans):
    """op(X) of batch entry z as a dense float64 (rows x cols) array."""
    base = X[z * stride:]
    if trans:
        return base[:ld * rows].reshape(rows, ld)[:, :cols].astype(np.float64)
    return base[:ld * cols].reshape(cols, ld).T[:rows, :].astype(np.float64)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,batch", [(256, 256, 256, 1), (300, 520, 1000, 3),
                                         (1024, 1024, 1024, 1), (2048, 64, 4096, 1),
                                         (129, 1000, 333, 2)])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_gpu_sgemm_split_tf32_tensor_core(cuda, built, m, n, k, batch, ta, tb):
    """fp32 GEMM on the tensor cores (hi/lo tf32 planes, split K for small tile
    counts): every entry within 1e-5 of |alpha| (|op(A)| |op(B)|)_ij + |beta C_ij|
    of the double-accumulated product, normwise 1e-5, padding untouched, and the
    same bar for the FFMA kernel under CUBLAS_PEDANTIC_MATH."""
    torch = cuda
    rng = np.random.default_rng(m + 3 * n + 7 * k + batch)
    A, lda, sa, B, ldb, sb, C0, ldc, sc = rand_case(rng, m, n, k, ta, tb, batch)
    alpha, beta = 1.25, (0.0 if (m + n) % 2 else -0.5)
    results = {}
    for mode in (capi.CUBLAS_DEFAULT_MATH, capi.CUBLAS_PEDANTIC_MATH):
        dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C0))
        b = Blas(torch)
        assert b.L.cublasSetMathMode(b.h, mode) == 0
        st = b.L.cublasSgemmStridedBatched(
            b.h, OPS[ta], OPS[tb], m, n, k, C.byref(C.c_float(alpha)), C.c_void_p(dA.data_ptr()),
            lda, sa, C.c_void_p(dB.data_ptr()), ldb, sb, C.byref(C.c_float(beta)),
            C.c_void_p(dC.data_ptr()), ldc, sc, batch)
        torch.cuda.synchronize()
        b.close()
        assert st == 0
        results[mode] = dC.cpu().numpy()
    for mode, got in results.items():
        mask = np.ones(len(got), bool)
        for z in range(batch):
            a = _op_dense(A, lda, sa, z, m, k, ta)
            bb = _op_dense(B, ldb, sb, z, k, n, tb)
            idx = (z * sc + np.arange(n)[None, :] * ldc + np.arange(m)[:, None])  # m x n
            c0 = C0[idx].astype(np.float64)
            want = alpha * (a @ bb) + beta * c0
            scale = abs(alpha) * (np.abs(a) @ np.abs(bb)) + abs(beta) * np.abs(c0)
            err = np.abs(got[idx].astype(np.float64) - want)
            assert np.all(err <= 1e-5 * scale + 1e-30), (mode, float((err / scale).max()))
            assert normwise(got[idx], want) <= 1e-5
            mask[idx.reshape(-1)] = False
        assert np.array_equal(got[mask], C0[mask])


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,batch,pad_c", [(2048, 1280, 520, 1, 4), (1024, 1024, 1024, 1, 4),
                                               (1028, 516, 2052, 1, 4), (1536, 1024, 256, 2, 4),
                                               (2048, 1280, 96, 1, 3), (512, 512, 4096, 1, 3)])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_gpu_sgemm_ffma_aligned_operands(cuda, built, m, n, k, batch, pad_c, ta, tb):
    """The FFMA kernel for 16-byte aligned fp32 operands (CUBLAS_PEDANTIC_MATH; leading
    dimensions and strides multiples of 4, m, n, k multiples of 4): whole-grid and
    split-K launches, partial tiles in m, n and k, batches, beta != 0, and C with a
    leading dimension that rules out 16-byte stores.  Every entry within 1e-5 of
    |alpha| (|op(A)| |op(B)|)_ij + |beta C_ij| of the float64 product, padding untouched."""
    torch = cuda
    rng = np.random.default_rng(m + 5 * n + 11 * k + batch)
    lda = (k if ta else m) + 4
    ldb = (n if tb else k) + 8
    ldc = m + pad_c
    sa = lda * (m if ta else k) + 4
    sb = ldb * (k if tb else n) + 12
    sc = ldc * n + 5
    A = rng.uniform(-1, 1, sa * batch).astype(np.float32)
    B = rng.uniform(-1, 1, sb * batch).astype(np.float32)
    C0 = rng.uniform(-1, 1, sc * batch).astype(np.float32)
    alpha, beta = 0.75, (-0.5 if k % 8 else 0.0)
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C0))
    b = Blas(torch)
    assert b.L.cublasSetMathMode(b.h, capi.CUBLAS_PEDANTIC_MATH) == 0
    st = b.L.cublasSgemmStridedBatched(
        b.h, OPS[ta], OPS[tb], m, n, k, C.byref(C.c_float(alpha)), C.c_void_p(dA.data_ptr()),
        lda, sa, C.c_void_p(dB.data_ptr()), ldb, sb, C.byref(C.c_float(beta)),
        C.c_void_p(dC.data_ptr()), ldc, sc, batch)
    torch.cuda.synchronize()
    b.close()
    assert st == 0
    got = dC.cpu().numpy()
    mask = np.ones(len(got), bool)
    for z in range(batch):
        a = _op_dense(A, lda, sa, z, m, k, ta)
        bb = _op_dense(B, ldb, sb, z, k, n, tb)
        idx = (z * sc + np.arange(n)[None, :] * ldc + np.arange(m)[:, None])
        c0 = C0[idx].astype(np.float64)
        want = alpha * (a @ bb) + beta * c0
        scale = abs(alpha) * (np.abs(a) @ np.abs(bb)) + abs(beta) * np.abs(c0)
        err = np.abs(got[idx].astype(np.float64) - want)
        assert np.all(err <= 1e-5 * scale + 1e-30), float((err / scale).max())
        mask[idx.reshape(-1)] = False
    assert np.array_equal(got[mask], C0[mask])


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1024, 1024, 1024), (516, 1028, 3076), (128, 128, 4096)])
def test_gpu_sgemm_ffma_stream_k_is_deterministic(cuda, built, m, n, k):
    """Problems with fewer 128 x 128 tiles than SMs run as equal k runs per CTA whose
    pieces are added back in k order: repeated calls give the same bits."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.rand(m * k, device="cuda", generator=g) - 0.5
    bm = torch.rand(k * n, device="cuda", generator=g) - 0.5
    outs = []
    b = Blas(torch)
    assert b.L.cublasSetMathMode(b.h, capi.CUBLAS_PEDANTIC_MATH) == 0
    for _ in range(3):
        c = torch.full((m * n,), float("nan"), device="cuda")
        assert b.L.cublasSgemm_v2(b.h, 0, 0, m, n, k, C.byref(C.c_float(1.0)),
                                  C.c_void_p(a.data_ptr()), m, C.c_void_p(bm.data_ptr()), k,
                                  C.byref(C.c_float(0.0)), C.c_void_p(c.data_ptr()), m) == 0
        outs.append(c)
    torch.cuda.synchronize()
    b.close()
    want = (a.double().view(k, m).T @ bm.double().view(n, k).T)  # m x n
    got = outs[0].view(n, m).T.double()
    assert float((got - want).norm() / want.norm()) <= 1e-6
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@pytest.mark.gpu
def test_gpu_sgemm_error_flat_in_k(cuda, built):
    """The split-tf32 path restarts its tensor-memory accumulator every two k-blocks and
    adds the chunks with round-to-nearest fp32 adds, so its error does not grow with K
    (the tensor core's own fp32 accumulation truncates).  Normwise error against a
    float64 product for K = 256 ... 16384, normal and positive data, beside the FFMA
    kernel (CUBLAS_PEDANTIC_MATH): both stay at the fp32 FMA loop's level."""
    torch = cuda
    m = n = 256
    rows = []
    for k, positive in ((256, False), (4096, False), (16384, False), (16384, True)):
        g = torch.Generator(device="cuda").manual_seed(k + positive)
        A = torch.randn(k, m, device="cuda", generator=g)   # column-major m x k, lda m
        B = torch.randn(n, k, device="cuda", generator=g)   # column-major k x n, ldb k
        if positive:
            A, B = A.abs(), B.abs()
        want = (A.double().t() @ B.double().t())             # m x n
        errs = []
        for mode in (capi.CUBLAS_DEFAULT_MATH, capi.CUBLAS_PEDANTIC_MATH):
            Cm = torch.empty(n, m, device="cuda")
            b = Blas(torch)
            assert b.L.cublasSetMathMode(b.h, mode) == 0
            assert b.L.cublasSgemm_v2(b.h, 0, 0, m, n, k, C.byref(C.c_float(1.0)),
                                      C.c_void_p(A.data_ptr()), m, C.c_void_p(B.data_ptr()), k,
                                      C.byref(C.c_float(0.0)), C.c_void_p(Cm.data_ptr()), m) == 0
            torch.cuda.synchronize()
            b.close()
            got = Cm.double().t()
            errs.append(float((got - want).norm() / want.norm()))
        rows.append((k, positive, *errs))
        assert errs[0] <= 2e-6 and errs[1] <= 5e-6, (k, positive, errs)
    for k, pos, e_tc, e_ffma in rows:
        print(f"K {k:6d} {'positive' if pos else 'normal  '}: split-tf32 {e_tc:.2e}  "
              f"FFMA {e_ffma:.2e}")


@pytest.mark.gpu
def test_gpu_sgemm_split_tf32_stream_switch_and_special_values(cuda, built):
    """The handle's split workspace stays ordered across cublasSetStream, and
    inf / -inf / nan propagate as in an fp32 loop, including an infinity meeting a
    value that tf32 holds exactly (whose lo plane must not be zero)."""
    torch = cuda
    m = n = k = 512
    rng = np.random.default_rng(5)
    A = rng.uniform(-1, 1, m * k).astype(np.float32)
    B = rng.uniform(-1, 1, k * n).astype(np.float32)
    A2 = rng.uniform(-1, 1, m * k).astype(np.float32)
    A2[3 + 7 * m] = np.inf     # row 3, column 7 of A (column-major)
    A2[9 + 7 * m] = -np.inf    # row 9, column 7
    A2[20 + 30 * m] = np.nan   # row 20
    A2[40 + 41 * m] = 0.5      # exactly representable in tf32 (lo is not zero)
    B2 = B.copy()
    B2[41 + 60 * k] = np.inf   # column 60 of B meets the exact 0.5 in row 40
    dA, dA2, dB = (torch.from_numpy(x).cuda() for x in (A, A2, B))
    dB2 = torch.from_numpy(B2).cuda()
    dC, dC2 = torch.zeros(m * n, device="cuda"), torch.zeros(m * n, device="cuda")
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    one, zero = C.byref(C.c_float(1.0)), C.byref(C.c_float(0.0))
    for s, a, bm, c in ((s1, dA, dB, dC), (s2, dA2, dB2, dC2)):
        assert L.cublasSetStream_v2(h, C.c_void_p(s.cuda_stream)) == 0
        assert L.cublasSgemm_v2(h, 0, 0, m, n, k, one, C.c_void_p(a.data_ptr()), m,
                                C.c_void_p(bm.data_ptr()), k, zero, C.c_void_p(c.data_ptr()),
                                m) == 0
    torch.cuda.synchronize()
    assert L.cublasDestroy_v2(h) == 0
    bb = B.reshape(n, k).T.astype(np.float64)
    want = A.reshape(k, m).T.astype(np.float64) @ bb
    assert normwise(dC.cpu().numpy().reshape(n, m).T, want) <= 1e-5
    got2 = dC2.cpu().numpy().reshape(n, m).T
    a2 = A2.reshape(k, m).T.astype(np.float64)
    b2 = B2.reshape(n, k).T.astype(np.float64)
    with np.errstate(invalid="ignore"):
        want2 = a2 @ b2
    assert np.isinf(want2[3]).all() and np.isnan(want2[20]).all() and np.isinf(want2[40, 60])
    assert np.array_equal(np.isinf(got2), np.isinf(want2))
    assert np.array_equal(np.isnan(got2), np.isnan(want2))
    inf = np.isinf(want2)
    assert np.array_equal(np.sign(got2[inf]), np.sign(want2[inf]))
    fin = np.isfinite(want2)
    assert normwise(got2[fin], want2[fin]) <= 1e-5


@pytest.mark.gpu
def test_gpu_sgemm_device_pointer_mode(cuda, built):
    torch = cuda
    rng = np.random.default_rng(1)
    m = n = k = 64
    A, lda, sa, B, ldb, sb, C0, ldc, sc = rand_case(rng, m, n, k, False, False, 1, pad=0)
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C0))
    scal = torch.tensor([2.0, 0.5], dtype=torch.float32, device="cuda")
    b = Blas(torch)
    assert b.L.cublasSetPointerMode_v2(b.h, capi.CUBLAS_POINTER_MODE_DEVICE) == 0
    st = b.L.cublasSgemm_v2(b.h, 0, 0, m, n, k, C.c_void_p(scal.data_ptr()),
                            C.c_void_p(dA.data_ptr()), lda, C.c_void_p(dB.data_ptr()), ldb,
                            C.c_void_p(scal.data_ptr() + 4), C.c_void_p(dC.data_ptr()), ldc)
    b.close()
    assert st == 0
    want = oracle.gemm("f32", False, False, m, n, k, 2.0, A, lda, B, ldb, 0.5, C0.copy(), ldc,
                       accum_f64=True)
    assert normwise(dC.cpu().numpy(), want.astype(np.float64)) <= 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("typ", ["f16", "bf16"])
@pytest.mark.parametrize("m,n,k,ta,tb,batch", [(16, 16, 16, False, False, 1),
                                               (100, 70, 50, True, False, 2),
                                               (64, 128, 96, False, True, 1),
                                               (256, 256, 256, False, False, 3),
                                               (512, 384, 1024, True, True, 1)])
def test_gpu_gemm_ex_16bit(cuda, built, typ, m, n, k, ta, tb, batch):
    torch = cuda
    rng = np.random.default_rng(k)
    A, lda, sa, B, ldb, sb, C0, ldc, sc = rand_case(rng, m, n, k, ta, tb, batch, pad=0)
    conv = oracle.half_bits if typ == "f16" else oracle.bf16_bits
    A16, B16, C16 = conv(A), conv(B), conv(C0)
    dA, dB, dC = (torch.from_numpy(x.view(np.int16).copy()).cuda() for x in (A16, B16, C16))
    dtype = capi.CUDA_R_16F if typ == "f16" else capi.CUDA_R_16BF
    b = Blas(torch)
    st = b.L.cublasGemmStridedBatchedEx(
        b.h, OPS[ta], OPS[tb], m, n, k, C.byref(C.c_float(1.0)), C.c_void_p(dA.data_ptr()), dtype,
        lda, sa, C.c_void_p(dB.data_ptr()), dtype, ldb, sb, C.byref(C.c_float(0.5)),
        C.c_void_p(dC.data_ptr()), dtype, ldc, sc, batch, capi.CUBLAS_COMPUTE_32F, -1)
    b.close()
    assert st == 0
    got = dC.cpu().numpy().view(np.uint16)
    want = oracle.gemm(typ, ta, tb, m, n, k, 1.0, A16, lda, B16, ldb, 0.5, C16.copy(), ldc,
                       stride_a=sa, stride_b=sb, stride_c=sc, batch=batch)
    dec = (lambda v: v.view(np.float16).astype(np.float64)) if typ == "f16" else \
        (lambda v: oracle.bf16_to_f32(v).astype(np.float64))
    assert normwise(dec(got), dec(want)) <= 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("typ", ["bf16", "f16"])
@pytest.mark.parametrize("m,n,k,batch,beta", [(128, 256, 64, 1, 0.0), (256, 512, 1024, 2, 0.0),
                                              (300, 520, 200, 1, 0.5), (1000, 1000, 1000, 1, 0.0),
                                              (129, 257, 65, 3, -1.0), (2048, 2048, 2048, 1, 0.0)])
def test_gpu_gemm_ex_tensor_core_layout(cuda, built, typ, m, n, k, batch, beta):
    """transa = T, transb = N (both operands K-major): the tcgen05 kernel's layout, with
    partial tiles in M, N and K, batches, and beta != 0."""
    torch = cuda
    rng = np.random.default_rng(m + n + k)
    lda = k + (8 if m % 2 else 0)
    ldb = k + 8
    ldc = m + 1
    sa, sb, sc = lda * m + 64, ldb * n, ldc * n + 3
    A = rng.uniform(-1, 1, sa * batch).astype(np.float32)
    B = rng.uniform(-1, 1, sb * batch).astype(np.float32)
    C0 = rng.uniform(-1, 1, sc * batch).astype(np.float32)
    conv = oracle.half_bits if typ == "f16" else oracle.bf16_bits
    A16, B16, C16 = conv(A), conv(B), conv(C0)
    dA, dB, dC = (torch.from_numpy(x.view(np.int16).copy()).cuda() for x in (A16, B16, C16))
    dtype = capi.CUDA_R_16F if typ == "f16" else capi.CUDA_R_16BF
    b = Blas(torch)
    st = b.L.cublasGemmStridedBatchedEx(
        b.h, capi.CUBLAS_OP_T, capi.CUBLAS_OP_N, m, n, k, C.byref(C.c_float(1.0)),
        C.c_void_p(dA.data_ptr()), dtype, lda, sa, C.c_void_p(dB.data_ptr()), dtype, ldb, sb,
        C.byref(C.c_float(beta)), C.c_void_p(dC.data_ptr()), dtype, ldc, sc, batch,
        capi.CUBLAS_COMPUTE_32F, -1)
    b.close()
    assert st == 0
    got = dC.cpu().numpy().view(np.uint16)
    # sampled check against the oracle (full check for the small shapes)
    dec = (lambda v: v.view(np.float16).astype(np.float64)) if typ == "f16" else \
        (lambda v: oracle.bf16_to_f32(v).astype(np.float64))
    want = C16.copy()
    oracle.gemm(typ, True, False, m, n, k, 1.0, A16, lda, B16, ldb, beta, want, ldc,
                stride_a=sa, stride_b=sb, stride_c=sc, batch=batch, threads=16)
    for z in range(batch):
        idx = (z * sc + np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).reshape(-1)
        assert normwise(dec(got[idx]), dec(want[idx])) <= 1e-2
    # untouched padding between columns and batches
    mask = np.ones(len(got), bool)
    for z in range(batch):
        mask[(z * sc + np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).reshape(-1)] = False
    assert np.array_equal(got[mask], C16[mask])


@pytest.mark.gpu
@pytest.mark.parametrize("typ", ["bf16", "f16"])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("m,n,k,batch,beta,pad", [(2048, 2048, 2048, 1, 0.0, 0),
                                                  (1000, 777, 520, 2, 0.5, 8),
                                                  (129, 2304, 72, 3, -1.0, 16),
                                                  (4096, 136, 1000, 1, 0.0, 24),
                                                  (1000, 1536, 256, 2, 0.0, 0)])
def test_gpu_gemm_ex_tensor_core_all_layouts(cuda, built, typ, ta, tb, m, n, k, batch, beta, pad):
    """Every transpose combination on the tcgen05 kernel: K-major operands (A with T,
    B with N) and MN-major ones (A with N, B with T), partial tiles in M, N and K,
    padded leading dimensions, batches, beta != 0.  Against the oracle's 16-bit GEMM
    (cublas_kernels.metal:1008-1045): normwise 1e-2 per batch entry on 16384 sampled
    entries (all entries when fewer), padding untouched.  Unpadded cases keep C's columns
    16-byte aligned (the transposed-output store of T,T writes 16-byte runs there)."""
    torch = cuda
    rng = np.random.default_rng(m * 3 + n * 5 + k * 7 + 11 * ta + 13 * tb)
    lda = (k if ta else m) + pad
    ldb = (n if tb else k) + pad
    ldc = m + 3 if pad else m
    sa = lda * (m if ta else k) + 64
    sb = ldb * (k if tb else n) + 128
    sc = ldc * n + (5 if pad else 64)
    conv = oracle.half_bits if typ == "f16" else oracle.bf16_bits
    A16 = conv(rng.uniform(-1, 1, sa * batch).astype(np.float32))
    B16 = conv(rng.uniform(-1, 1, sb * batch).astype(np.float32))
    C16 = conv(rng.uniform(-1, 1, sc * batch).astype(np.float32))
    dA, dB, dC = (torch.from_numpy(x.view(np.int16).copy()).cuda() for x in (A16, B16, C16))
    dtype = capi.CUDA_R_16F if typ == "f16" else capi.CUDA_R_16BF
    b = Blas(torch)
    st = b.L.cublasGemmStridedBatchedEx(
        b.h, OPS[ta], OPS[tb], m, n, k, C.byref(C.c_float(1.0)), C.c_void_p(dA.data_ptr()), dtype,
        lda, sa, C.c_void_p(dB.data_ptr()), dtype, ldb, sb, C.byref(C.c_float(beta)),
        C.c_void_p(dC.data_ptr()), dtype, ldc, sc, batch, capi.CUBLAS_COMPUTE_32F, -1)
    torch.cuda.synchronize()
    b.close()
    assert st == 0
    got = dC.cpu().numpy().view(np.uint16)
    dec = (lambda v: v.view(np.float16).astype(np.float64)) if typ == "f16" else \
        (lambda v: oracle.bf16_to_f32(v).astype(np.float64))
    total = m * n * batch
    ne = min(total, 16384)
    pick = rng.choice(total, ne, replace=False) if ne < total else np.arange(total)
    z, rem = pick // (m * n), pick % (m * n)
    rows, cols = (rem % m).astype(np.int32), (rem // m)
    want = C16.copy()
    oracle.gemm(typ, ta, tb, m, n, k, 1.0, A16, lda, B16, ldb, beta, want, ldc, stride_a=sa,
                stride_b=sb, stride_c=sc, batch=batch, entries=(rows, (z * n + cols).astype(np.int32)),
                threads=16)
    flat = z * sc + cols * ldc + rows
    for zz in range(batch):
        sel = flat[z == zz]
        assert normwise(dec(got[sel]), dec(want[sel])) <= 1e-2, (zz, typ, ta, tb)
    err = np.abs(dec(got[flat]) - dec(want[flat]))
    assert np.all(err <= 2e-2 * np.abs(dec(want[flat])) + 0.05), float(err.max())
    mask = np.ones(len(got), bool)
    for zz in range(batch):
        mask[(zz * sc + np.arange(n)[:, None] * ldc + np.arange(m)[None, :]).reshape(-1)] = False
    assert np.array_equal(got[mask], C16[mask])


@pytest.mark.gpu
def test_gpu_hgemm_reference_pin(cuda, built):
    """tests/cublas_test.cpp:383-410: 16^3, A = 0.5, B = 0.25 -> 2.0 (fp16 scalars)."""
    torch = cuda
    a = torch.from_numpy(oracle.half_bits(np.full(256, 0.5)).view(np.int16).copy()).cuda()
    bb = torch.from_numpy(oracle.half_bits(np.full(256, 0.25)).view(np.int16).copy()).cuda()
    c = torch.zeros(256, dtype=torch.int16, device="cuda")
    one = C.c_uint16(0x3C00)
    zero = C.c_uint16(0)
    b = Blas(torch)
    st = b.L.cublasHgemm(b.h, 0, 0, 16, 16, 16, C.byref(one), C.c_void_p(a.data_ptr()), 16,
                         C.c_void_p(bb.data_ptr()), 16, C.byref(zero), C.c_void_p(c.data_ptr()), 16)
    b.close()
    assert st == 0
    got = c.cpu().numpy().view(np.float16).astype(np.float32)
    assert np.all(np.abs(got - 2.0) < 1e-2)
