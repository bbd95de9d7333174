"""cusparseSpMV (CSR, non-transposed, fp32) and the descriptor / argument checks of SpMM.

CPU: the oracle against the reference's known answer and the C-ABI host logic.
GPU (marked): the CUDA path through the C ABI against the oracle.  Index handling
is bit-exact by construction (the same (row, col) pairs are consumed); values
must satisfy |y - y_exact| <= 1e-5 * (|A||x|)_row + 1e-30 against the double-
precision row result, and the fp32 oracle must satisfy the same bound.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import fptr, stream_ptr

REF_OFFSETS = [0, 2, 4, 6, 8]
REF_COLS = [0, 2, 1, 3, 0, 1, 2, 3]
REF_VALS = [10.0, 20.0, 30.0, 40.0, 50.0, 60.0, 70.0, 80.0]
REF_X = [1.0, 2.0, 3.0, 4.0]
REF_Y = [70.0, 220.0, 170.0, 530.0]


def test_oracle_reference_pin():
    """tests/cusparse_test.cpp:41-107 (base 0) and the same matrix 1-based."""
    np.testing.assert_allclose(oracle.spmv_csr(REF_OFFSETS, REF_COLS, REF_VALS, REF_X), REF_Y,
                               atol=1e-4)
    np.testing.assert_allclose(
        oracle.spmv_csr([o + 1 for o in REF_OFFSETS], [c + 1 for c in REF_COLS], REF_VALS, REF_X,
                        base=1), REF_Y, atol=1e-4)


def test_oracle_matches_scipy_free_dense_product():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((50, 40)) * (rng.random((50, 40)) < 0.2)
    rows, cols = np.nonzero(a)
    offsets = np.zeros(51, np.int64)
    np.add.at(offsets, rows + 1, 1)
    offsets = np.cumsum(offsets)
    x = rng.standard_normal(40).astype(np.float32)
    y, exact, absr = oracle.spmv_csr(offsets, cols, a[rows, cols].astype(np.float32), x,
                                     alpha=1.5, with_abs=True)
    want = 1.5 * (a.astype(np.float32).astype(np.float64) @ x.astype(np.float64))
    np.testing.assert_allclose(exact, want, rtol=1e-12, atol=1e-12)
    assert np.all(np.abs(y - want) <= 1e-5 * 1.5 * absr + 1e-30)


def _mk(L, fn, *args):
    h = C.c_void_p()
    assert getattr(L, fn)(C.byref(h), *args) == 0
    return h


def test_host_logic(built):
    L = capi.cusparse()
    h = _mk(L, "cusparseCreate")
    v = C.c_int()
    assert L.cusparseGetVersion(h, C.byref(v)) == 0 and v.value == 12000
    assert L.cusparseGetErrorName(3) == b"CUSPARSE_STATUS_INVALID_VALUE"
    p = C.c_void_p(4096)
    # CSR descriptor validation (cusparse_descriptors.mm:134-167)
    m = C.c_void_p()
    assert L.cusparseCreateCsr(C.byref(m), 4, 4, 8, p, p, p, 3, 2, 0, 0) == \
        capi.CUSPARSE_STATUS_NOT_SUPPORTED
    assert L.cusparseCreateCsr(C.byref(m), 4, 4, 8, p, None, p, 2, 2, 0, 0) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseCreateCsr(C.byref(m), -1, 4, 8, p, p, p, 2, 2, 0, 0) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseCreateCsr(C.byref(m), 4, 4, 8, p, p, p, 2, 2, 2, 0) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseCreateCsr(C.byref(m), 4, 4, 8, p, p, p, 2, 2, 0, 5) == \
        capi.CUSPARSE_STATUS_NOT_SUPPORTED
    m = _mk(L, "cusparseCreateCsr", 4, 4, 8, p, p, p, 2, 2, 0, 0)
    vx = _mk(L, "cusparseCreateDnVec", 4, p, 0)
    vy = _mk(L, "cusparseCreateDnVec", 4, p, 0)
    vbad = _mk(L, "cusparseCreateDnVec", 5, p, 0)
    sz = C.c_size_t(99)
    a, b = fptr(1.0), fptr(0.0)
    assert L.cusparseSpMV_bufferSize(h, 0, a, m, vx, b, vy, 0, 0, C.byref(sz)) == 0
    assert sz.value == 0
    assert L.cusparseSpMV_bufferSize(h, 0, a, m, vbad, b, vy, 0, 0, C.byref(sz)) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseSpMV(h, 0, None, m, vx, b, vy, 0, 0, None) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE
    # unaddressable arrays are rejected before launch, in both directions
    assert L.cusparseSpMV(h, 1, a, m, vx, b, vy, 0, 0, None) == capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseSpMV(h, 0, a, m, vx, b, vy, 0, 0, None) == capi.CUSPARSE_STATUS_INVALID_VALUE
    # dense matrices (cusparse_descriptors.mm:196-223) and SpMM checks (cusparse_ops.mm:213-273)
    d = C.c_void_p()
    assert L.cusparseCreateDnMat(C.byref(d), 4, 2, 3, p, 0, capi.CUSPARSE_ORDER_COL) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE  # ld < rows
    assert L.cusparseCreateDnMat(C.byref(d), 4, 2, 1, p, 0, capi.CUSPARSE_ORDER_ROW) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE  # ld < cols
    assert L.cusparseCreateDnMat(C.byref(d), 4, 2, 4, p, 0, 3) == capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseCreateDnMat(C.byref(d), 4, 2, 4, None, 0, 1) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseCreateDnMat(C.byref(d), 4, 2, 4, p, 5, 1) == capi.CUSPARSE_STATUS_NOT_SUPPORTED
    assert L.cusparseCreateDnMat(C.byref(d), 0, 0, 1, None, 0, 1) == 0
    assert L.cusparseDestroyDnMat(d) == 0
    assert L.cusparseDestroyDnMat(d) == capi.CUSPARSE_STATUS_INVALID_VALUE
    mb = _mk(L, "cusparseCreateDnMat", 4, 2, 4, p, 0, capi.CUSPARSE_ORDER_COL)
    mc = _mk(L, "cusparseCreateDnMat", 4, 2, 2, p, 0, capi.CUSPARSE_ORDER_ROW)
    mh = _mk(L, "cusparseCreateDnMat", 4, 2, 4, p, 2, capi.CUSPARSE_ORDER_COL)  # fp16
    assert L.cusparseSpMM_bufferSize(h, 0, 0, a, m, mb, b, mc, 0, 0, C.byref(sz)) == 0
    assert sz.value == 0
    assert L.cusparseSpMM_bufferSize(h, 0, 1, a, m, mb, b, mc, 0, 0, C.byref(sz)) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE  # op(B) is 2 x 4
    assert L.cusparseSpMM(h, 0, 0, None, m, mb, b, mc, 0, 0, None) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseSpMM(h, 0, 0, a, m, mh, b, mc, 0, 0, None) == \
        capi.CUSPARSE_STATUS_NOT_SUPPORTED
    assert L.cusparseSpMM(h, 0, 0, a, m, mb, b, mc, 0, 0, None) == \
        capi.CUSPARSE_STATUS_INVALID_VALUE  # unaddressable arrays
    for d in (mb, mc, mh):
        assert L.cusparseDestroyDnMat(d) == 0
    for d in (vx, vy, vbad):
        assert L.cusparseDestroyDnVec(d) == 0
    assert L.cusparseDestroySpMat(m) == 0
    assert L.cusparseDestroySpMat(m) == capi.CUSPARSE_STATUS_INVALID_VALUE
    assert L.cusparseDestroy(h) == 0
    assert L.cusparseSpMV(h, 0, a, m, vx, b, vy, 0, 0, None) == \
        capi.CUSPARSE_STATUS_NOT_INITIALIZED
    assert L.cusparseSpMM(h, 0, 0, a, m, m, b, m, 0, 0, None) == \
        capi.CUSPARSE_STATUS_NOT_INITIALIZED


# --------------------------------------------------------------------- GPU --
def gpu_spmv(torch, offsets, cols, vals, x, *, ncols=None, base=0, alpha=1.0, beta=0.0, y0=None):
    L = capi.cusparse()
    ro = torch.as_tensor(np.asarray(offsets, np.int32)).cuda()
    ci = torch.as_tensor(np.asarray(cols, np.int32)).cuda()
    va = torch.as_tensor(np.asarray(vals, np.float32)).cuda()
    xx = torch.as_tensor(np.asarray(x, np.float32)).cuda()
    rows = len(offsets) - 1
    ncols = len(x) if ncols is None else ncols
    yy = torch.as_tensor(np.asarray(y0, np.float32)).cuda() if y0 is not None else \
        torch.zeros(rows, dtype=torch.float32, device="cuda")
    return _spmv_dev(torch, L, ro, ci, va, xx, yy, rows, ncols, len(vals), base, alpha, beta)


def _spmv_dev(torch, L, ro, ci, va, xx, yy, rows, ncols, nnz, base, alpha, beta):
    h = _mk(L, "cusparseCreate")
    assert L.cusparseSetStream(h, C.c_void_p(stream_ptr(torch))) == 0
    ptr = lambda t: C.c_void_p(t.data_ptr()) if t.numel() else C.c_void_p(16)
    m = _mk(L, "cusparseCreateCsr", rows, ncols, nnz, ptr(ro), ptr(ci), ptr(va), 2, 2, base, 0)
    vx = _mk(L, "cusparseCreateDnVec", ncols, ptr(xx), 0)
    vy = _mk(L, "cusparseCreateDnVec", rows, ptr(yy), 0)
    st = L.cusparseSpMV(h, 0, fptr(alpha), m, vx, fptr(beta), vy, 0, 0, None)
    torch.cuda.synchronize()
    for fn, d in (("cusparseDestroyDnVec", vx), ("cusparseDestroyDnVec", vy),
                  ("cusparseDestroySpMat", m)):
        assert getattr(L, fn)(d) == 0
    assert L.cusparseDestroy(h) == 0
    assert st == 0
    return yy.cpu().numpy()


def check(got, exact, absr, y_oracle, tol=1e-5):
    err = np.abs(got.astype(np.float64) - exact)
    assert np.all(err <= tol * absr + 1e-30), f"max err/scale {np.max(err / (absr + 1e-30)):.3e}"
    err_o = np.abs(y_oracle.astype(np.float64) - exact)
    assert np.all(err_o <= tol * absr + 1e-30)


def random_csr(rng, rows, cols, lengths):
    lengths = np.asarray(lengths, np.int64)
    offsets = np.concatenate([[0], np.cumsum(lengths)])
    col = np.concatenate([np.sort(rng.choice(cols, size=k, replace=False)) if k else
                          np.zeros(0, np.int64) for k in lengths]).astype(np.int32)
    vals = rng.uniform(-1, 1, offsets[-1]).astype(np.float32)
    return offsets, col, vals


@pytest.mark.gpu
def test_gpu_reference_pin(cuda, built):
    y = gpu_spmv(cuda, REF_OFFSETS, REF_COLS, REF_VALS, REF_X)
    np.testing.assert_allclose(y, REF_Y, atol=1e-4)
    y = gpu_spmv(cuda, [o + 1 for o in REF_OFFSETS], [c + 1 for c in REF_COLS], REF_VALS, REF_X,
                 base=1)
    np.testing.assert_allclose(y, REF_Y, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["empty_rows", "avg3", "avg6", "avg16", "avg40", "avg200",
                                  "mixed_long", "one_row", "tail_rows"])
@pytest.mark.parametrize("base", [0, 1])
def test_gpu_random_matrices(cuda, built, kind, base):
    rng = np.random.default_rng(abs(hash(kind)) % 1000 + base)
    cols = 3000
    rows = {"one_row": 1, "tail_rows": 1000 + 7}.get(kind, 2000)
    if kind == "empty_rows":
        lengths = rng.integers(0, 3, rows) * (rng.random(rows) < 0.5)
    elif kind.startswith("avg"):
        m = int(kind[3:])
        lengths = rng.integers(max(0, m - m // 2), m + m // 2 + 1, rows)
    elif kind == "mixed_long":
        lengths = np.where(rng.random(rows) < 0.05, rng.integers(65, 2500, rows),
                           rng.integers(1, 20, rows))
    elif kind == "one_row":
        lengths = [2999]
    else:
        lengths = rng.integers(0, 40, rows)
    offsets, col, vals = random_csr(rng, rows, cols, lengths)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    y0 = rng.uniform(-1, 1, len(offsets) - 1).astype(np.float32)
    for alpha, beta in ((1.0, 0.0), (-0.5, 1.25)):
        got = gpu_spmv(cuda, offsets + base, col + base, vals, x, base=base, alpha=alpha,
                       beta=beta, y0=y0)
        yo, exact, absr = oracle.spmv_csr(offsets + base, col + base, vals, x, base=base,
                                          alpha=alpha, beta=beta, y=y0.copy(), with_abs=True)
        scale = abs(alpha) * absr + (abs(beta) * np.abs(y0) if beta else 0)
        check(got, exact, scale, yo)


@pytest.mark.gpu
def test_gpu_config_powerlaw(cuda, built):
    """4M x 4M, power-law row lengths (mean ~16, max 4096), seed 7."""
    torch = cuda
    from muda_b200 import synth
    m = synth.powerlaw_csr(torch, 1 << 22, 1 << 22, seed=7)
    assert 14 * m["rows"] < m["nnz"] < 18 * m["rows"]
    L = capi.cusparse()
    y = torch.zeros(m["rows"], dtype=torch.float32, device="cuda")
    got = _spmv_dev(torch, L, m["row_offsets"], m["col_ind"], m["values"], m["x"], y, m["rows"],
                    m["cols"], m["nnz"], 0, 1.0, 0.0)
    yo, exact, absr = oracle.spmv_csr(m["row_offsets"].cpu().numpy(), m["col_ind"].cpu().numpy(),
                                      m["values"].cpu().numpy(), m["x"].cpu().numpy(),
                                      with_abs=True, threads=16)
    check(got, exact, absr, yo)
    lengths = np.diff(m["row_offsets"].cpu().numpy())
    assert lengths.min() >= 2 and lengths.max() <= 4096


@pytest.mark.gpu
@pytest.mark.parametrize("base", [0, 1])
def test_dist_spmv_single_rank_cuda_path(cuda, built, base):
    """muda_b200.dist_spmv on one rank: the local product runs through cusparseSpMV
    on the GPU (the path each rank takes under torchrun) and matches the oracle."""
    torch = cuda
    from muda_b200.dist_spmv import DistSpMV
    rng = np.random.default_rng(21)
    rows, cols = 3000, 2500
    k = rng.integers(0, 40, rows)
    ro = np.zeros(rows + 1, np.int64)
    ro[1:] = np.cumsum(k)
    ci = np.concatenate([np.sort(rng.choice(cols, kk, replace=False)) for kk in k]).astype(np.int32)
    va = rng.uniform(-1, 1, ro[-1]).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    d = DistSpMV.from_full(torch, None, None, torch.from_numpy((ro + base).astype(np.int32)).cuda(),
                           torch.from_numpy(ci + base).cuda(), torch.from_numpy(va).cuda(), cols,
                           base=base)
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    d.spmv(1.5, d.x_slice(torch.from_numpy(x).cuda()), 0.0, y)
    torch.cuda.synchronize()
    d.close()
    want, exact, absr = oracle.spmv_csr(ro.astype(np.int32), ci, va, x, alpha=1.5, with_abs=True)
    err = np.abs(y.cpu().numpy().astype(np.float64) - exact)  # exact includes alpha
    assert np.all(err <= 1e-5 * 1.5 * absr + 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("mean,long_frac", [(1, 0.001), (10, 0.005), (30, 0.005)])
@pytest.mark.parametrize("base", [0, 1])
def test_gpu_spmv_array_alignment(cuda, built, mean, long_frac, base):
    """fp32 SpMV whose column and value arrays start on a 16-byte boundary and 4 bytes
    past one (element offset 0 and 1 into a fresh allocation) on the same matrix: both
    must meet the oracle's bound.  Rows from empty to 3000 entries (whole-warp rows),
    nnz not a multiple of 4, mean lengths that select 2, 4 and 8 lanes per row."""
    torch = cuda
    rng = np.random.default_rng(100 * mean + base)
    rows, cols = 4099, 5000
    lengths = rng.integers(0, 2 * mean + 1, rows)
    long_rows = rng.random(rows) < long_frac
    lengths[long_rows] = rng.integers(100, 3000, int(long_rows.sum()))
    lengths[-1] = 0
    if lengths.sum() % 4 == 0:
        lengths[0] += 1
    offsets, col, vals = random_csr(rng, rows, cols, lengths)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    y0 = rng.uniform(-1, 1, rows).astype(np.float32)
    L = capi.cusparse()
    nnz = len(vals)
    ro = torch.from_numpy((offsets + base).astype(np.int32)).cuda()
    xx = torch.from_numpy(x).cuda()
    outs = []
    for shift in (0, 1):  # element offset into a fresh (256-byte aligned) allocation
        ci = torch.empty(nnz + 4, dtype=torch.int32, device="cuda")[shift:shift + nnz]
        va = torch.empty(nnz + 4, dtype=torch.float32, device="cuda")[shift:shift + nnz]
        ci.copy_(torch.from_numpy((col + base).astype(np.int32)))
        va.copy_(torch.from_numpy(vals))
        assert (ci.data_ptr() % 16 == 0) == (shift == 0)
        yy = torch.from_numpy(y0.copy()).cuda()
        outs.append(_spmv_dev(torch, L, ro, ci, va, xx, yy, rows, cols, nnz, base, -0.5, 1.25))
    yo, exact, absr = oracle.spmv_csr(offsets + base, col + base, vals, x, base=base, alpha=-0.5,
                                      beta=1.25, y=y0.copy(), with_abs=True)
    scale = 0.5 * absr + 1.25 * np.abs(y0)
    for got in outs:
        check(got, exact, scale, yo)


@pytest.mark.gpu
@pytest.mark.parametrize("base", [0, 1])
def test_gpu_entry_ranges_rows_across_ranges(cuda, built, base):
    """The entry-range kernel (2048 stored entries per warp): rows of 12000, 8192 and 4096
    entries that span several ranges (ranges in which no row starts pass their whole sum
    on), empty rows at the start, between long rows and after the last entry, a row that
    starts exactly on a range boundary; two calls must agree bit for bit (the summation
    order depends on the matrix only)."""
    torch = cuda
    rng = np.random.default_rng(7 + base)
    cols = 20000
    lengths = [0, 0, 5, 12000, 0, 3, 9000, 4096, 1, 0, 2] + list(rng.integers(0, 60, 300)) + \
        [8192, 0, 0]
    lengths = np.asarray(lengths, np.int64)
    # make one row start exactly on a range boundary (a multiple of 4096 entries)
    offs = np.concatenate([[0], np.cumsum(lengths)])
    k = int(np.searchsorted(offs, 3 * 4096))
    lengths[k - 1] = 3 * 4096 - offs[k - 1]
    offsets, col, vals = random_csr(rng, len(lengths), cols, lengths)
    assert (offsets == 3 * 4096).any()
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    y0 = rng.uniform(-1, 1, len(lengths)).astype(np.float32)
    for alpha, beta in ((1.0, 0.0), (0.75, -2.0)):
        got = gpu_spmv(cuda, offsets + base, col + base, vals, x, base=base, alpha=alpha,
                       beta=beta, y0=y0)
        again = gpu_spmv(cuda, offsets + base, col + base, vals, x, base=base, alpha=alpha,
                         beta=beta, y0=y0)
        assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
        yo, exact, absr = oracle.spmv_csr(offsets + base, col + base, vals, x, base=base,
                                          alpha=alpha, beta=beta, y=y0.copy(), with_abs=True)
        scale = abs(alpha) * absr + (abs(beta) * np.abs(y0) if beta else 0)
        check(got, exact, scale, yo)


@pytest.mark.gpu
def test_gpu_spmv_decreasing_offsets_stay_in_bounds(cuda, built):
    """Malformed CSR (row offsets that decrease, or point past nnz) must not make either
    SpMV kernel read or write outside its arrays: the call returns success (the values
    of the malformed rows are unspecified), and a well-formed call right after it on the
    same device gives the oracle's result."""
    torch = cuda
    rng = np.random.default_rng(3)
    cols = 500
    for lengths in ([8] * 200, [1] * 200):  # entry-range kernel, row-tile kernel
        offsets, col, vals = random_csr(rng, len(lengths), cols, lengths)
        bad = offsets.copy()
        bad[50] = bad[40]             # decreasing
        bad[120] = offsets[-1] + 999  # past nnz (clamped)
        x = rng.uniform(-1, 1, cols).astype(np.float32)
        got = gpu_spmv(cuda, bad, col, vals, x)
        assert np.all(np.isfinite(got))
        got = gpu_spmv(cuda, offsets, col, vals, x)
        yo, exact, absr = oracle.spmv_csr(offsets, col, vals, x, with_abs=True)
        check(got, exact, absr, yo)
