"""cusparseSpMV with opA = TRANSPOSE and fp16 values, and cusparseSpMM.

CPU: the oracle restatements (transposed SpMV fast path and generic branch, SpMM)
against the reference's known answers (tests/cusparse_test.cpp:109-156) and dense
float64 products.  GPU (marked), through the C ABI:
  - SpMM with A not transposed must equal the oracle bit for bit (same per-output
    fma order as the reference kernel), for every order / transpose of B and C;
  - atomically accumulated results (transposed SpMV, transposed-A SpMM) must satisfy
    |got - exact| <= 1e-5 * (|alpha| sum |a b| + |beta c|) against the float64 result;
  - fp16 results must satisfy |got - exact| <= 2^-11 |exact| + 2e-5 * scale + 2^-24
    (one half rounding plus fp32 accumulation).
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import fptr, stream_ptr
from tests.test_sparse import REF_COLS, REF_OFFSETS, REF_VALS, REF_X, random_csr

REF_YT = [160.0, 240.0, 300.0, 400.0]
REF_B = [1.0, 2.0, 3.0, 4.0, 0.5, 1.0, 1.5, 2.0]  # 4 x 2, column-major


def test_oracle_transpose_pin():
    """tests/cusparse_test.cpp:109-125: y = A^T x."""
    for generic in (False, True):
        y = oracle.spmv_csr_t(REF_OFFSETS, REF_COLS, REF_VALS, REF_X, 4, generic=generic)
        np.testing.assert_allclose(y, REF_YT, atol=1e-4)


def test_oracle_spmm_pin():
    """tests/cusparse_test.cpp:127-156: C (4x2, col-major) = A * B (col-major)."""
    c = np.zeros(8, np.float32)
    oracle.spmm_csr(REF_OFFSETS, REF_COLS, REF_VALS, 4, REF_B, 4, 1, c, 4, 1, 2)
    assert c[0] == 70.0 and c[1] == 220.0 and c[4] == 35.0 and c[7] == 265.0


def dense_of(offsets, cols, vals, rows, ncols):
    a = np.zeros((rows, ncols))
    for r in range(rows):
        for k in range(offsets[r], offsets[r + 1]):
            a[r, cols[k]] += vals[k]
    return a


def store(mat, order, ld):
    """Flat storage of a 2-D array in the given order (1 col, 2 row) and leading dim."""
    r, c = mat.shape
    if order == 1:
        buf = np.zeros(ld * (c - 1) + r, np.float32)
        for j in range(c):
            buf[j * ld:j * ld + r] = mat[:, j]
    else:
        buf = np.zeros(ld * (r - 1) + c, np.float32)
        for i in range(r):
            buf[i * ld:i * ld + c] = mat[i, :]
    return buf


def load(buf, order, ld, r, c):
    out = np.zeros((r, c), np.float64)
    for i in range(r):
        for j in range(c):
            out[i, j] = buf[i + j * ld] if order == 1 else buf[i * ld + j]
    return out


@pytest.mark.parametrize("op_a,op_b,order_b,order_c", [(0, 0, 1, 1), (1, 0, 2, 1), (0, 1, 1, 2),
                                                       (1, 1, 2, 2)])
def test_oracle_spmm_matches_dense(op_a, op_b, order_b, order_c):
    rng = np.random.default_rng(op_a * 8 + op_b * 4 + order_b)
    rows, cols, n = 23, 17, 5
    offsets, ci, va = random_csr(rng, rows, cols, rng.integers(0, 6, rows))
    a = dense_of(offsets, ci, va, rows, cols)
    a_eff = a.T if op_a else a
    k = a_eff.shape[1]
    b_eff = rng.standard_normal((k, n)).astype(np.float32)
    b_st = b_eff.T if op_b else b_eff
    ldb = (b_st.shape[0] if order_b == 1 else b_st.shape[1]) + 2
    bb = store(b_st, order_b, ldb)
    m = a_eff.shape[0]
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    ldc = (m if order_c == 1 else n) + 1
    cc = store(c0, order_c, ldc)
    oracle.spmm_csr(offsets, ci, va, cols, bb, ldb, order_b, cc, ldc, order_c, n, op_a=op_a,
                    op_b=op_b, alpha=0.75, beta=-0.5)
    want = 0.75 * a_eff @ b_eff.astype(np.float64) - 0.5 * c0
    np.testing.assert_allclose(load(cc, order_c, ldc, m, n), want, rtol=1e-5, atol=1e-5)


# --------------------------------------------------------------------- GPU --
def _mk(L, fn, *args):
    h = C.c_void_p()
    assert getattr(L, fn)(C.byref(h), *args) == 0
    return h


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t.numel() else C.c_void_p(16)


class Csr:
    """A CSR matrix and a handle on the GPU."""

    def __init__(self, torch, offsets, cols, vals, nrows, ncols, base=0, half=False):
        self.L = capi.cusparse()
        self.torch = torch
        self.h = _mk(self.L, "cusparseCreate")
        assert self.L.cusparseSetStream(self.h, C.c_void_p(stream_ptr(torch))) == 0
        self.ro = torch.as_tensor(np.asarray(offsets, np.int32) + base).cuda()
        self.ci = torch.as_tensor(np.asarray(cols, np.int32) + base).cuda()
        dt = np.float16 if half else np.float32
        self.va = torch.as_tensor(np.asarray(vals, dt)).cuda()
        self.vt = 2 if half else 0
        self.m = _mk(self.L, "cusparseCreateCsr", nrows, ncols, len(vals), _ptr(self.ro),
                     _ptr(self.ci), _ptr(self.va), 2, 2, base, self.vt)

    def spmv(self, op, x, y, alpha, beta):
        vx = _mk(self.L, "cusparseCreateDnVec", x.numel(), _ptr(x), self.vt)
        vy = _mk(self.L, "cusparseCreateDnVec", y.numel(), _ptr(y), self.vt)
        st = self.L.cusparseSpMV(self.h, op, fptr(alpha), self.m, vx, fptr(beta), vy, 0, 0, None)
        self.torch.cuda.synchronize()
        assert self.L.cusparseDestroyDnVec(vx) == 0 and self.L.cusparseDestroyDnVec(vy) == 0
        return st

    def spmm(self, op_a, op_b, b, b_shape, ldb, order_b, c, c_shape, ldc, order_c, alpha, beta):
        mb = _mk(self.L, "cusparseCreateDnMat", b_shape[0], b_shape[1], ldb, _ptr(b), 0, order_b)
        mc = _mk(self.L, "cusparseCreateDnMat", c_shape[0], c_shape[1], ldc, _ptr(c), 0, order_c)
        st = self.L.cusparseSpMM(self.h, op_a, op_b, fptr(alpha), self.m, mb, fptr(beta), mc, 0,
                                 0, None)
        self.torch.cuda.synchronize()
        assert self.L.cusparseDestroyDnMat(mb) == 0 and self.L.cusparseDestroyDnMat(mc) == 0
        return st

    def close(self):
        assert self.L.cusparseDestroySpMat(self.m) == 0
        assert self.L.cusparseDestroy(self.h) == 0


@pytest.mark.gpu
def test_gpu_reference_pins(cuda, built):
    torch = cuda
    for base in (0, 1):
        a = Csr(torch, REF_OFFSETS, REF_COLS, REF_VALS, 4, 4, base=base)
        x = torch.tensor(REF_X, device="cuda")
        y = torch.zeros(4, device="cuda")
        assert a.spmv(1, x, y, 1.0, 0.0) == 0
        np.testing.assert_allclose(y.cpu().numpy(), REF_YT, atol=1e-4)
        b = torch.tensor(REF_B, device="cuda")
        c = torch.zeros(8, device="cuda")
        assert a.spmm(0, 0, b, (4, 2), 4, 1, c, (4, 2), 4, 1, 1.0, 0.0) == 0
        cv = c.cpu().numpy()
        assert cv[0] == 70.0 and cv[1] == 220.0 and cv[4] == 35.0 and cv[7] == 265.0
        a.close()


def _matrix(kind, rng, rows, cols):
    if kind == "avg3":
        lengths = rng.integers(1, 6, rows)
    elif kind == "avg16":
        lengths = rng.integers(8, 25, rows)
    elif kind == "mixed_long":
        lengths = np.where(rng.random(rows) < 0.05, rng.integers(65, min(cols, 2500), rows),
                           rng.integers(0, 20, rows))
    else:  # empty rows and columns
        lengths = rng.integers(0, 3, rows) * (rng.random(rows) < 0.5)
    return random_csr(rng, rows, cols, lengths)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["avg3", "avg16", "mixed_long", "sparse_empty"])
@pytest.mark.parametrize("base", [0, 1])
def test_gpu_spmv_transpose_f32(cuda, built, kind, base):
    torch = cuda
    rng = np.random.default_rng(len(kind) * 7 + base)
    rows, cols = 2100, 3001
    offsets, ci, va = _matrix(kind, rng, rows, cols)
    x = rng.uniform(-1, 1, rows).astype(np.float32)
    y0 = rng.uniform(-1, 1, cols).astype(np.float32)
    a = Csr(torch, offsets, ci, va, rows, cols, base=base)
    for alpha, beta in ((1.0, 0.0), (-0.5, 1.25), (0.0, 2.0)):
        y = torch.from_numpy(y0.copy()).cuda()
        assert a.spmv(1, torch.from_numpy(x).cuda(), y, alpha, beta) == 0
        yo, exact, absr = oracle.spmv_csr_t(offsets, ci, va, x, cols, alpha=alpha, beta=beta,
                                            y=y0, with_abs=True)
        scale = abs(alpha) * absr + abs(beta) * np.abs(y0)
        err = np.abs(y.cpu().numpy().astype(np.float64) - exact)
        assert np.all(err <= 1e-5 * scale + 1e-30), np.max(err / (scale + 1e-30))
        assert np.all(np.abs(yo - exact) <= 1e-5 * scale + 1e-30)
    a.close()


@pytest.mark.gpu
@pytest.mark.parametrize("per_lane", [1, 4])
def test_gpu_scatter_probe_counts(cuda, built, per_lane):
    """The scatter-ceiling probe (mb200ProbeScatter) adds 1 per index: y ends as the
    index histogram, exactly (counts far below 2^24), including a ragged tail that the
    four-per-lane form leaves out (n not a multiple of 4)."""
    torch = cuda
    rng = np.random.default_rng(per_lane)
    n, size = 1_000_003, 70_000
    idx = rng.integers(0, size, n).astype(np.int32)
    idx[:5000] = 17  # one hot entry
    d_idx = torch.from_numpy(idx).cuda()
    y = torch.zeros(size, dtype=torch.float32, device="cuda")
    P = capi.probe()
    assert P.mb200ProbeScatter(C.c_void_p(y.data_ptr()), C.c_void_p(d_idx.data_ptr()), n,
                               per_lane, 296, stream_ptr(torch)) == 0
    torch.cuda.synchronize()
    done = n if per_lane == 1 else n // 4 * 4
    assert np.array_equal(y.cpu().numpy(), np.bincount(idx[:done], minlength=size).astype(np.float32))
    assert P.mb200ProbeScatter(None, C.c_void_p(d_idx.data_ptr()), n, per_lane, 296,
                               stream_ptr(torch)) == 1


def _half_check(got, exact, scale):
    got = got.astype(np.float64)
    bound = 2.0 ** -11 * np.abs(exact) + 2e-5 * scale + 2.0 ** -24
    assert np.all(np.abs(got - exact) <= bound), np.max(np.abs(got - exact) / bound)


@pytest.mark.gpu
@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("kind", ["avg3", "mixed_long"])
def test_gpu_spmv_f16(cuda, built, trans, kind):
    torch = cuda
    rng = np.random.default_rng(trans * 3 + len(kind))
    rows, cols = 1500, 1700
    offsets, ci, va = _matrix(kind, rng, rows, cols)
    va16 = va.astype(np.float16)
    nx, ny = (rows, cols) if trans else (cols, rows)
    x16 = rng.uniform(-1, 1, nx).astype(np.float16)
    y16 = rng.uniform(-1, 1, ny).astype(np.float16)
    a = Csr(torch, offsets, ci, va16, rows, cols, half=True)
    for alpha, beta in ((1.0, 0.0), (0.75, -0.5)):
        y = torch.from_numpy(y16.copy()).cuda()
        assert a.spmv(trans, torch.from_numpy(x16).cuda(), y, alpha, beta) == 0
        va32, x32, y32 = va16.astype(np.float32), x16.astype(np.float32), y16.astype(np.float32)
        if trans:
            _, exact, absr = oracle.spmv_csr_t(offsets, ci, va32, x32, cols, alpha=alpha,
                                               beta=beta, y=y32, generic=True, with_abs=True)
        else:
            _, exact, absr = oracle.spmv_csr(offsets, ci, va32, x32, alpha=alpha, beta=beta,
                                             y=y32.copy(), with_abs=True)
        scale = abs(alpha) * absr + abs(beta) * np.abs(y32)
        _half_check(y.cpu().numpy(), exact, scale)
        ref = oracle.spmv_csr_f16(offsets, ci, va16, x16, cols=cols, trans=bool(trans),
                                  alpha=alpha, beta=beta, y=y16)
        _half_check(ref, exact, scale)
    a.close()


# (rows, cols, ncols): odd sizes, one that fills several 32-column chunks, and
# float4-eligible ones (ncols and ld multiples of 4) for each group width of the
# shared-memory ring kernel (4, 8, 16 and 32 lanes per row)
SPMM_SHAPES = [(300, 200, 7), (257, 300, 130), (500, 400, 64), (600, 3000, 64), (300, 200, 12),
               (260, 500, 32), (257, 400, 128)]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SPMM_SHAPES)
@pytest.mark.parametrize("op_a", [0, 1])
@pytest.mark.parametrize("op_b,order_b,order_c", [(0, 2, 2), (0, 1, 1), (1, 2, 1), (1, 1, 2)])
def test_gpu_spmm(cuda, built, shape, op_a, op_b, order_b, order_c):
    torch = cuda
    rows, cols, n = shape
    rng = np.random.default_rng(rows + op_a * 10 + op_b * 100 + order_b * 1000 + order_c)
    offsets, ci, va = _matrix("mixed_long" if rows in (257, 600) else "avg16", rng, rows, cols)
    k = rows if op_a else cols
    m = cols if op_a else rows
    b_eff = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    b_st = b_eff.T.copy() if op_b else b_eff
    pad = 0 if n % 4 == 0 and order_b == 2 else 3
    ldb = (b_st.shape[0] if order_b == 1 else b_st.shape[1]) + (4 if pad == 0 else pad)
    bb = store(b_st, order_b, ldb)
    c0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    ldc = (m if order_c == 1 else n) + (4 if n % 4 == 0 else 1)
    cc = store(c0, order_c, ldc)
    a = Csr(torch, offsets, ci, va, rows, cols, base=op_b)
    for alpha, beta in ((1.0, 0.0), (-0.75, 0.5)):
        tb = torch.from_numpy(bb).cuda()
        tc = torch.from_numpy(cc.copy()).cuda()
        assert a.spmm(op_a, op_b, tb, b_st.shape, ldb, order_b, tc, (m, n), ldc, order_c, alpha,
                      beta) == 0
        got = tc.cpu().numpy()
        want = cc.copy()
        _, exact, mag = oracle.spmm_csr(offsets, ci, va, cols, bb, ldb, order_b, want, ldc,
                                        order_c, n, op_a=op_a, op_b=op_b, alpha=alpha, beta=beta,
                                        with_abs=True)
        if op_a == 0:
            np.testing.assert_array_equal(got, want)  # bit-exact, gaps of C included
        else:
            g = load(got, order_c, ldc, m, n)
            scale = abs(alpha) * mag + abs(beta) * np.abs(c0.astype(np.float64))
            err = np.abs(g - exact)
            assert np.all(err <= 1e-5 * scale + 1e-30), np.max(err / (scale + 1e-30))
    a.close()


@pytest.mark.gpu
def test_gpu_spmm_long_row_list_overflow(cuda, built):
    """More rows above the scheduler's 256-entry threshold in one length bucket than
    its region of the list holds (8192 of 65536): every row is then taken in the
    chunked phase, and the results stay bit-identical to the oracle (checked on a
    sample of rows)."""
    torch = cuda
    rng = np.random.default_rng(4242)
    rows, cols, n, k = 66000, 2048, 64, 257
    ci = np.sort(rng.integers(0, cols, (rows, k)), axis=1).astype(np.int32)
    offsets = np.arange(rows + 1, dtype=np.int64) * k
    va = rng.uniform(-1, 1, (rows, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (cols, n)).astype(np.float32)
    a = Csr(torch, offsets, ci.reshape(-1), va.reshape(-1), rows, cols)
    tb = torch.from_numpy(b.reshape(-1)).cuda()
    tc = torch.zeros(rows * n, dtype=torch.float32, device="cuda")
    assert a.spmm(0, 0, tb, (cols, n), n, 2, tc, (rows, n), n, 2, 1.0, 0.0) == 0
    got = tc.cpu().numpy().reshape(rows, n)
    sample = np.unique(np.r_[0:64, rows - 64:rows, rng.integers(0, rows, 128)])
    sub_off = np.arange(len(sample) + 1, dtype=np.int64) * k
    want = np.zeros(len(sample) * n, np.float32)
    oracle.spmm_csr(sub_off, ci[sample].reshape(-1), va[sample].reshape(-1), cols, b.reshape(-1),
                    n, 2, want, n, 2, n)
    np.testing.assert_array_equal(got[sample], want.reshape(len(sample), n))
    a.close()


@pytest.mark.gpu
def test_gpu_spmm_long_rows_every_bucket(cuda, built):
    """Long rows in every length bucket of the scheduler (257 .. 6000 entries, the last
    bucket open-ended), between short and empty rows: the first phase takes them
    longest bucket first, the second sorts each 32-row chunk by length, and every
    output stays bit-identical to the oracle's entry-order sums."""
    torch = cuda
    rng = np.random.default_rng(5151)
    rows, cols, n = 3001, 8192, 64
    lengths = np.where(rng.random(rows) < 0.12, rng.integers(257, 6001, rows),
                       rng.integers(0, 24, rows))
    lengths[:8] = [257, 383, 384, 511, 512, 767, 2896, 6000]
    offsets, ci, va = random_csr(rng, rows, cols, lengths)
    b = rng.uniform(-1, 1, (cols, n)).astype(np.float32)
    a = Csr(torch, offsets, ci, va, rows, cols)
    tb = torch.from_numpy(b.reshape(-1)).cuda()
    tc = torch.full((rows * n,), 7.0, dtype=torch.float32, device="cuda")
    assert a.spmm(0, 0, tb, (cols, n), n, 2, tc, (rows, n), n, 2, 1.0, 0.0) == 0
    got = tc.cpu().numpy()
    want = np.zeros(rows * n, np.float32)
    oracle.spmm_csr(offsets, ci, va, cols, b.reshape(-1), n, 2, want, n, 2, n)
    np.testing.assert_array_equal(got, want)
    a.close()
