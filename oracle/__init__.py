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


def generate_lognormal(seed: int, offset: int, n: int, mean: float = 0.0, stddev: float = 1.0,
                       threads: int = 1) -> tuple[np.ndarray, int]:
    """GenerateHostLogNormal (curand_context.mm:225-235)."""
    out = np.empty(n, dtype=np.float32)
    nxt = lib().oracle_generate_lognormal(seed, offset, out.ctypes.data, n, mean, stddev, threads)
    return out, int(nxt)


def generate_double(seed: int, offset: int, n: int, kind: str = "uniform", mean: float = 0.0,
                    stddev: float = 1.0, threads: int = 1) -> tuple[np.ndarray, int]:
    """Double streams of the reference host generator (curand_context.mm:115-143,
    187-247); kind "uniform", "normal" or "lognormal"."""
    k = {"uniform": 0, "normal": 1, "lognormal": 2}[kind]
    out = np.empty(n, dtype=np.float64)
    nxt = lib().oracle_generate_double(seed, offset, out.ctypes.data, n, k, mean, stddev, threads)
    return out, int(nxt)


def poisson_threshold(lam: float) -> np.float32:
    """exp(-lambda) of the fp32 lambda, rounded once from double (the library's
    threshold for Knuth's method)."""
    return np.float32(np.exp(-np.float64(np.float32(lam))))


def generate_poisson(seed: int, offset: int, n: int, lam: float, *, reference_host=False,
                     threads: int = 8) -> tuple[np.ndarray, int]:
    """Poisson counts: the device-kernel definition (curand_kernels.metal:212-264), or
    with reference_host=True the reference's own host path (curand_context.mm:249-293)."""
    out = np.empty(n, dtype=np.uint32)
    nxt = lib().oracle_generate_poisson(seed, offset, out.ctypes.data, n, lam,
                                        float(poisson_threshold(lam)), int(reference_host),
                                        threads)
    return out, int(nxt)


def philox_gather(ctrs: np.ndarray, seed: int, threads: int = 8) -> np.ndarray:
    """Philox blocks at the given counters, shape (len(ctrs), 4)."""
    ctrs = np.ascontiguousarray(ctrs, dtype=np.uint64)
    out = np.empty((len(ctrs), 4), dtype=np.uint32)
    lib().oracle_philox_gather(_ptr(ctrs, C.c_uint64), len(ctrs), seed, _ptr(out, C.c_uint32),
                               threads)
    return out


# ------------------------------------------------------------- conv/softmax --
def _nchw_strides(shape, fmt: str):
    n, c, h, w = shape
    if fmt == "NCHW":
        return (c * h * w, h * w, w, 1)
    return (h * w * c, 1, w * c, c)  # NHWC


def conv2d(x: np.ndarray, w: np.ndarray, xshape, wshape, *, x_fmt="NCHW", w_fmt="NCHW",
           pad=(0, 0), stride=(1, 1), dil=(1, 1), groups=1, mode="cross", alpha=1.0,
           beta=0.0, y: np.ndarray | None = None, y_fmt=None, accum_f64=False,
           threads: int = 8) -> np.ndarray:
    """Reference direct convolution (cudnn_kernels.metal:20-62) on flat buffers.

    xshape = (n, c, h, w); wshape = (k, c/groups, r, s) logical; layouts by format
    strings; x/w/y dtype float32 or bfloat16-as-uint16 (then the result is bf16)."""
    from oracle.protos import ConvParams
    n, c, h, wd = xshape
    k, cg, r, s = wshape
    oh = 1 + (h + 2 * pad[0] - (1 + (r - 1) * dil[0])) // stride[0]
    ow = 1 + (wd + 2 * pad[1] - (1 + (s - 1) * dil[1])) // stride[1]
    y_fmt = y_fmt or x_fmt
    bf16 = x.dtype == np.uint16
    if y is None:
        y = np.zeros(n * k * oh * ow, dtype=x.dtype)
    xs = _nchw_strides(xshape, x_fmt)
    ys = _nchw_strides((n, k, oh, ow), y_fmt)
    p = ConvParams(n, c, h, wd, *xs, k, oh, ow, groups, *ys, r, s, pad[0], pad[1], stride[0],
                   stride[1], dil[0], dil[1], 0 if w_fmt == "NCHW" else 1,
                   0 if mode == "conv" else 1, alpha, beta)
    x = np.ascontiguousarray(x)
    w = np.ascontiguousarray(w)
    lib().oracle_conv2d_fwd(x.ctypes.data, w.ctypes.data, y.ctypes.data, C.byref(p), int(bf16),
                            int(accum_f64), threads)
    return y


def conv_params(xshape, wshape, *, x_fmt="NCHW", w_fmt="NCHW", y_fmt=None, pad=(0, 0),
                stride=(1, 1), dil=(1, 1), groups=1, mode="cross", alpha=1.0, beta=0.0):
    """OracleConvParams of a forward convolution and its output shape (n, k, oh, ow)."""
    from oracle.protos import ConvParams
    n, c, h, wd = xshape
    k, cg, r, s = wshape
    oh = 1 + (h + 2 * pad[0] - (1 + (r - 1) * dil[0])) // stride[0]
    ow = 1 + (wd + 2 * pad[1] - (1 + (s - 1) * dil[1])) // stride[1]
    xs = _nchw_strides(xshape, x_fmt)
    ys = _nchw_strides((n, k, oh, ow), y_fmt or x_fmt)
    p = ConvParams(n, c, h, wd, *xs, k, oh, ow, groups, *ys, r, s, pad[0], pad[1], stride[0],
                   stride[1], dil[0], dil[1], 0 if w_fmt == "NCHW" else 1,
                   0 if mode == "conv" else 1, alpha, beta)
    return p, (n, k, oh, ow)


def conv_bwd_data(w, dy, xshape, wshape, dx=None, *, accum_f64=False, threads=8, **geom):
    """Reference backward data (cudnn_kernels.metal:194-243): dx (flat, x layout)."""
    p, _ = conv_params(xshape, wshape, **geom)
    dx = np.zeros(int(np.prod(xshape)), np.float32) if dx is None else dx
    lib().oracle_conv_bwd_data(np.ascontiguousarray(w, np.float32).ctypes.data,
                               np.ascontiguousarray(dy, np.float32).ctypes.data, dx.ctypes.data,
                               C.byref(p), int(accum_f64), threads)
    return dx


def conv_bwd_filter(x, dy, xshape, wshape, dw=None, *, accum_f64=False, with_mag=False,
                    threads=8, **geom):
    """Reference backward filter (cudnn_kernels.metal:245-286): dw (flat, w layout)."""
    p, _ = conv_params(xshape, wshape, **geom)
    dw = np.zeros(int(np.prod(wshape)), np.float32) if dw is None else dw
    mag = np.zeros(dw.shape, np.float64) if with_mag else None
    lib().oracle_conv_bwd_filter(np.ascontiguousarray(x, np.float32).ctypes.data,
                                 np.ascontiguousarray(dy, np.float32).ctypes.data, dw.ctypes.data,
                                 C.byref(p), int(accum_f64),
                                 mag.ctypes.data if with_mag else None, threads)
    return (dw, mag) if with_mag else dw


def tensor4(shape, strides=None, fmt="NCHW"):
    from oracle.protos import Tensor4
    st = strides if strides is not None else _nchw_strides(shape, fmt)
    return Tensor4(*shape, *st)


def conv_bwd_bias(dy, shape, db=None, *, strides=None, alpha=1.0, beta=0.0, accum_f64=False):
    """Reference backward bias (cudnn_kernels.metal:288-305); returns (db, sum |dy|)."""
    db = np.zeros(shape[1], np.float32) if db is None else db
    mag = np.zeros(shape[1], np.float64)
    lib().oracle_conv_bwd_bias(np.ascontiguousarray(dy, np.float32).ctypes.data,
                               C.byref(tensor4(shape, strides)), db.ctypes.data, alpha, beta,
                               int(accum_f64), mag.ctypes.data)
    return db, mag


def add_tensor(a, ashape, c, cshape, *, astrides=None, cstrides=None, alpha=1.0, beta=0.0):
    """Reference AddTensor (cudnn_kernels.metal:307-331), c updated in place."""
    lib().oracle_add_tensor(np.ascontiguousarray(a, np.float32).ctypes.data,
                            C.byref(tensor4(ashape, astrides)), c.ctypes.data,
                            C.byref(tensor4(cshape, cstrides)), alpha, beta)
    return c


def activation(x, shape, y, mode, *, coef=0.0, xstrides=None, ystrides=None, alpha=1.0,
               beta=0.0):
    """Reference activation forward (cudnn_kernels.metal:333-384), y updated in place."""
    lib().oracle_activation(np.ascontiguousarray(x, np.float32).ctypes.data,
                            C.byref(tensor4(shape, xstrides)), y.ctypes.data,
                            C.byref(tensor4(shape, ystrides)), mode, coef, alpha, beta)
    return y


def pooling(x, xshape, y, yshape, win, pad, stride, mode, *, xstrides=None, ystrides=None,
            alpha=1.0, beta=0.0):
    """Reference pooling forward (cudnn_kernels.metal:401-445), y updated in place."""
    lib().oracle_pooling(np.ascontiguousarray(x, np.float32).ctypes.data,
                         C.byref(tensor4(xshape, xstrides)), y.ctypes.data,
                         C.byref(tensor4(yshape, ystrides)), win[0], win[1], pad[0], pad[1],
                         stride[0], stride[1], mode, alpha, beta)
    return y


def bn_inference(x, shape, y, scale, bias, mean, var, *, per_activation=False, eps=1e-5,
                 alpha=1.0, beta=0.0):
    """Reference batch-norm inference (cudnn_kernels.metal:570-611), y updated in place."""
    f = lambda a: np.ascontiguousarray(a, np.float32).ctypes.data
    lib().oracle_bn_inference(f(x), C.byref(tensor4(shape)), y.ctypes.data,
                              C.byref(tensor4(shape)), f(scale), f(bias), f(mean), f(var),
                              int(per_activation), eps, alpha, beta)
    return y


def bn_training(x, shape, y, scale, bias, *, running=None, save=None, factor=0.1, eps=1e-5,
                alpha=1.0, beta=0.0, accum_f64=False):
    """Reference batch-norm training (cudnn_kernels.metal:613-714); running = (mean, var)
    and save = (mean, inv_std) arrays are updated in place when given."""
    f = lambda a: np.ascontiguousarray(a, np.float32).ctypes.data
    rm, rv = running if running is not None else (None, None)
    sm, sv = save if save is not None else (None, None)
    lib().oracle_bn_training(f(x), C.byref(tensor4(shape)), y.ctypes.data,
                             C.byref(tensor4(shape)), f(scale), f(bias),
                             rm.ctypes.data if rm is not None else None,
                             rv.ctypes.data if rv is not None else None,
                             sm.ctypes.data if sm is not None else None,
                             sv.ctypes.data if sv is not None else None, factor, eps, alpha, beta,
                             int(accum_f64))
    return y


def softmax(x: np.ndarray, shape, *, algo: int = 1, channel: bool = False, alpha=1.0, beta=0.0,
            y: np.ndarray | None = None, x_strides=None, y_strides=None,
            threads: int = 8) -> np.ndarray:
    """Reference softmax forward (cudnn_ops.mm:656-719 dispatch) on flat float32 buffers."""
    from oracle.protos import Tensor4
    n, c, h, w = shape
    xs = x_strides or _nchw_strides(shape, "NCHW")
    ys = y_strides or xs
    if y is None:
        y = np.zeros_like(x)
    X = Tensor4(n, c, h, w, *xs)
    Y = Tensor4(n, c, h, w, *ys)
    lib().oracle_softmax_fwd(_ptr(x, C.c_float), _ptr(y, C.c_float), C.byref(X), C.byref(Y),
                             algo, int(channel), alpha, beta, threads)
    return y


def spmv_csr(row_offsets, col_ind, values, x, *, base=0, alpha=1.0, beta=0.0, y=None,
             with_abs=False, threads: int = 8):
    """Reference thread-per-row CSR SpMV (cusparse_kernels.metal:54-77).

    Returns y, or with with_abs=True (y, exact row result in float64, |A||x| per row
    in float64)."""
    ro = np.ascontiguousarray(row_offsets, dtype=np.int32)
    ci = np.ascontiguousarray(col_ind, dtype=np.int32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    rows = len(ro) - 1
    y = np.zeros(rows, np.float32) if y is None else y
    absr = np.zeros(rows, np.float64) if with_abs else None
    exact = np.zeros(rows, np.float64) if with_abs else None
    lib().oracle_spmv_csr(rows, ro.ctypes.data, ci.ctypes.data, va.ctypes.data, base,
                          xx.ctypes.data, y.ctypes.data, alpha, beta,
                          exact.ctypes.data if with_abs else None,
                          absr.ctypes.data if with_abs else None, threads)
    return (y, exact, absr) if with_abs else y


def spmv_csr_t(row_offsets, col_ind, values, x, cols, *, base=0, alpha=1.0, beta=0.0, y=None,
               generic=False, with_abs=False):
    """Reference transposed CSR SpMV, y = alpha A^T x + beta y (cusparse_ops.mm:166-191
    and cusparse_kernels.metal:21-52 for generic=False; the generic kernel's op_a = 1
    branch, cusparse_kernels.metal:79-92, for generic=True).

    Returns y, or with with_abs=True (y, exact result in float64, sum |a x| per
    output in float64)."""
    ro = np.ascontiguousarray(row_offsets, dtype=np.int32)
    ci = np.ascontiguousarray(col_ind, dtype=np.int32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    rows = len(ro) - 1
    y = np.zeros(cols, np.float32) if y is None else np.ascontiguousarray(y, np.float32).copy()
    exact = np.zeros(cols, np.float64) if with_abs else None
    absr = np.zeros(cols, np.float64) if with_abs else None
    lib().oracle_spmv_csr_t(rows, cols, ro.ctypes.data, ci.ctypes.data, va.ctypes.data, base,
                            xx.ctypes.data, y.ctypes.data, alpha, beta, int(generic),
                            exact.ctypes.data if with_abs else None,
                            absr.ctypes.data if with_abs else None)
    return (y, exact, absr) if with_abs else y


def spmv_csr_f16(row_offsets, col_ind, values, x, *, cols=None, trans=False, base=0, alpha=1.0,
                 beta=0.0, y=None):
    """Reference fp16 SpMV (cusparse_kernels.metal:94-133 and the warp kernel :159-184):
    half values and vectors widened to fp32, fp32 fma accumulation, one rounding of
    fma(alpha, sum, beta * y) to half.  Returns float16."""
    va = np.asarray(values, np.float16).astype(np.float32)
    xx = np.asarray(x, np.float16).astype(np.float32)
    y32 = None if y is None else np.asarray(y, np.float16).astype(np.float32)
    if trans:
        out = spmv_csr_t(row_offsets, col_ind, va, xx, cols, base=base, alpha=alpha, beta=beta,
                         y=y32, generic=True)
    else:
        rows = len(row_offsets) - 1
        out = spmv_csr(row_offsets, col_ind, va, xx, base=base, alpha=alpha, beta=beta,
                       y=np.zeros(rows, np.float32) if y32 is None else y32.copy())
    return out.astype(np.float16)


def spmm_csr(row_offsets, col_ind, values, a_cols, B, ldb, order_b, C, ldc, order_c, ncols, *,
             op_a=0, op_b=0, base=0, alpha=1.0, beta=0.0, with_abs=False, threads: int = 8):
    """Reference CSR SpMM (cusparse_kernels.metal:201-247), C updated in place (flat
    float32 array with leading dimension ldc; order 1 = column-major, 2 = row-major).
    With with_abs=True also returns (exact, mag) as (out_rows, ncols) float64 arrays."""
    ro = np.ascontiguousarray(row_offsets, dtype=np.int32)
    ci = np.ascontiguousarray(col_ind, dtype=np.int32)
    va = np.ascontiguousarray(values, dtype=np.float32)
    bb = np.ascontiguousarray(B, dtype=np.float32)
    assert C.dtype == np.float32 and C.flags.c_contiguous
    a_rows = len(ro) - 1
    out_rows = a_rows if op_a == 0 else a_cols
    exact = np.zeros((out_rows, ncols), np.float64) if with_abs else None
    mag = np.zeros((out_rows, ncols), np.float64) if with_abs else None
    lib().oracle_spmm_csr(a_rows, a_cols, ro.ctypes.data, ci.ctypes.data, va.ctypes.data, base,
                          op_a, bb.ctypes.data, ldb, order_b, op_b, C.ctypes.data, ldc, order_c,
                          ncols, alpha, beta, exact.ctypes.data if with_abs else None,
                          mag.ctypes.data if with_abs else None, threads)
    return (C, exact, mag) if with_abs else C


def fft_c2c(x: np.ndarray, dims, batch: int, sign: int, *, istride=1, idist=None, ostride=1,
            odist=None, out_len=None, exact=False, threads: int = 8) -> np.ndarray:
    """Reference batched C2C FFT (cufft_exec.mm:101-211) on a flat complex64 array.

    exact=True returns the double-precision result (complex128), otherwise the
    restated single-precision arithmetic (complex64)."""
    dims = list(dims)
    total = int(np.prod(dims))
    idist = total * istride if idist is None else idist
    odist = total * ostride if odist is None else odist
    if out_len is None:
        out_len = (batch - 1) * odist + (total - 1) * ostride + 1
    xin = np.ascontiguousarray(x, dtype=np.complex64)
    d = np.asarray(dims, dtype=np.int32)
    if exact:
        out = np.zeros(out_len, np.complex128)
        lib().oracle_fft_c2c(xin.ctypes.data, None, len(dims), d.ctypes.data, batch, istride,
                             idist, ostride, odist, sign, 1, out.ctypes.data, threads)
    else:
        out = np.zeros(out_len, np.complex64)
        lib().oracle_fft_c2c(xin.ctypes.data, out.ctypes.data, len(dims), d.ctypes.data, batch,
                             istride, idist, ostride, odist, sign, 0, None, threads)
    return out


GEMM_TYPES = {"f32": 0, "f16": 1, "bf16": 2}


def gemm(type_: str, transa: bool, transb: bool, m: int, n: int, k: int, alpha: float,
         A: np.ndarray, lda: int, B: np.ndarray, ldb: int, beta: float, C: np.ndarray, ldc: int,
         *, stride_a=0, stride_b=0, stride_c=0, batch=1, accum_f64=False, entries=None,
         threads: int = 8) -> np.ndarray:
    """Reference column-major GEMM (cublas_kernels.metal:969-1045); updates and returns C.

    16-bit operands are passed as uint16 bit patterns.  entries=(rows, batch*n + cols)
    evaluates only those entries of C."""
    A = np.ascontiguousarray(A)
    B = np.ascontiguousarray(B)
    assert C.flags["C_CONTIGUOUS"]
    rows = cols = None
    ne = 0
    if entries is not None:
        rows = np.ascontiguousarray(entries[0], dtype=np.int32)
        cols = np.ascontiguousarray(entries[1], dtype=np.int32)
        ne = len(rows)
    lib().oracle_gemm(GEMM_TYPES[type_], int(transa), int(transb), m, n, k, alpha, A.ctypes.data,
                      lda, stride_a, B.ctypes.data, ldb, stride_b, beta, C.ctypes.data, ldc,
                      stride_c, batch, int(accum_f64),
                      rows.ctypes.data if rows is not None else None,
                      cols.ctypes.data if cols is not None else None, ne, threads)
    return C


def half_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (round to nearest even)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- cuBLAS level 1 / 2
def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def saxpy(n, alpha, x, incx, y, incy):
    """y = fma(alpha, x, y) in place on a copy of y (cublas_kernels.metal:11-23)."""
    x, y = _f32(x), _f32(y).copy()
    lib().oracle_saxpy(n, alpha, x.ctypes.data, incx, y.ctypes.data, incy)
    return y


def scopy(n, x, incx, y, incy):
    x, y = _f32(x), _f32(y).copy()
    lib().oracle_scopy(n, x.ctypes.data, incx, y.ctypes.data, incy)
    return y


def sscal(n, alpha, x, incx):
    x = _f32(x).copy()
    lib().oracle_sscal(n, alpha, x.ctypes.data, incx)
    return x


def sswap(n, x, incx, y, incy):
    x, y = _f32(x).copy(), _f32(y).copy()
    lib().oracle_sswap(n, x.ctypes.data, incx, y.ctypes.data, incy)
    return x, y


def sreduce(op, n, x, incx, y=None, incy=1):
    """op 'dot' | 'nrm2' | 'asum' -> (fp32 reference formula, float64 value, float64
    sum of term magnitudes)."""
    code = {"dot": 0, "nrm2": 1, "asum": 2}[op]
    x = _f32(x)
    yy = _f32(y) if y is not None else np.zeros(1, np.float32)
    f = np.zeros(1, np.float32)
    d = np.zeros(2, np.float64)
    lib().oracle_sreduce(code, n, x.ctypes.data, incx, yy.ctypes.data, incy, f.ctypes.data,
                         d[:1].ctypes.data, d[1:].ctypes.data)
    return float(f[0]), float(d[0]), float(d[1])


def isamax(n, x, incx):
    return int(lib().oracle_isamax(n, _f32(x).ctypes.data, incx))


def geam(dtype, transa, transb, m, n, alpha, A, lda, beta, B, ldb, C, ldc, threads=1):
    """Reference Sgeam / Dgeam (dtype np.float32 / np.float64) on column-major arrays;
    returns a copy of C with the m x n block written.  A or B may be None when its
    scalar is 0 (the reference does not read it)."""
    dt = np.dtype(dtype)
    C = np.ascontiguousarray(C, dt).copy()
    A = np.zeros(1, dt) if A is None else np.ascontiguousarray(A, dt)
    B = np.zeros(1, dt) if B is None else np.ascontiguousarray(B, dt)
    fn = lib().oracle_sgeam if dt == np.float32 else lib().oracle_dgeam
    fn(1 if transa else 0, 1 if transb else 0, m, n, alpha, A.ctypes.data, lda, beta,
       B.ctypes.data, ldb, C.ctypes.data, ldc, threads)
    return C


# ---------------------------------------------------------------- fp64 BLAS
def _d(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def daxpy(n, alpha, x, incx, y, incy):
    """Reference-BLAS daxpy (oracle/blas64.cpp); returns the updated copy of y."""
    x, y = _d(x), _d(y).copy()
    lib().oracle_daxpy(n, alpha, x.ctypes.data, incx, y.ctypes.data, incy)
    return y


def dcopy(n, x, incx, y, incy):
    x, y = _d(x), _d(y).copy()
    lib().oracle_dcopy(n, x.ctypes.data, incx, y.ctypes.data, incy)
    return y


def dscal(n, alpha, x, incx):
    x = _d(x).copy()
    lib().oracle_dscal(n, alpha, x.ctypes.data, incx)
    return x


def dswap(n, x, incx, y, incy):
    x, y = _d(x).copy(), _d(y).copy()
    lib().oracle_dswap(n, x.ctypes.data, incx, y.ctypes.data, incy)
    return x, y


def dreduce(op, n, x, incx, y=None, incy=1):
    """op "dot" / "nrm2" / "asum": (value in element order, extended value, magnitude sum)."""
    x = _d(x)
    y = _d(y) if y is not None else np.zeros(1)
    out = np.zeros(3)
    lib().oracle_dreduce({"dot": 0, "nrm2": 1, "asum": 2}[op], n, x.ctypes.data, incx,
                         y.ctypes.data, incy, out.ctypes.data)
    return float(out[0]), float(out[1]), float(out[2])


def idamax(n, x, incx):
    return int(lib().oracle_idamax(n, _d(x).ctypes.data, incx))


def dgemv(trans, m, n, alpha, A, lda, x, incx, beta, y, incy, threads=8):
    """Returns (y, bound) with bound_i = |alpha| (|op(A)||x|)_i + |beta y_i|."""
    A, x, y = _d(A), _d(x), _d(y).copy()
    bound = np.zeros(n if trans else m)
    lib().oracle_dgemv(int(trans), m, n, alpha, A.ctypes.data, lda, x.ctypes.data, incx, beta,
                       y.ctypes.data, incy, bound.ctypes.data, threads)
    return y, bound


def dgemm(transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, *, stride_a=0,
          stride_b=0, stride_c=0, batch=1, entries=None, threads=8):
    """Returns (C, bound); bound per evaluated entry (all m*n*batch entries, batch-major
    then column-major, or the given (rows, batch*n + cols) entries)."""
    A, B, C = _d(A), _d(B), _d(C).copy()
    rows = cols = None
    ne = 0
    if entries is not None:
        rows = np.ascontiguousarray(entries[0], dtype=np.int32)
        cols = np.ascontiguousarray(entries[1], dtype=np.int32)
        ne = len(rows)
    bound = np.zeros(ne if ne else m * n * batch)
    lib().oracle_dgemm(int(transa), int(transb), m, n, k, alpha, A.ctypes.data, lda, stride_a,
                       B.ctypes.data, ldb, stride_b, beta, C.ctypes.data, ldc, stride_c, batch,
                       rows.ctypes.data if rows is not None else None,
                       cols.ctypes.data if cols is not None else None, ne, bound.ctypes.data,
                       threads)
    return C, bound


def sgemv(trans, m, n, alpha, A, lda, x, incx, beta, y, incy, threads=8):
    """-> (y after the reference kernel, exact per output, |terms| per output)."""
    A, x, y = _f32(A), _f32(x), _f32(y).copy()
    out_len = n if trans else m
    exact = np.zeros(out_len, np.float64)
    absv = np.zeros(out_len, np.float64)
    lib().oracle_sgemv(1 if trans else 0, m, n, alpha, A.ctypes.data, lda, x.ctypes.data, incx,
                       beta, y.ctypes.data, incy, exact.ctypes.data, absv.ctypes.data, threads)
    return y, exact, absv


# ---------------------------------------------------------------- cuFFT R2C / C2R
def fft_r2c(x, dims, batch, *, istride=1, idist=None, ostride=1, odist=None, threads=8):
    """Reference R2C (libraries/fft/src/cufft_exec.mm:213-303): gather (x, 0) into dense
    complex rows (cufft_kernels.metal:43-56), forward C2C over all axes, keep entries
    0 .. L/2 of the last axis (:58-77).  Returns the float64 result in the output layout."""
    dims = list(dims)
    L = dims[-1]
    H = L // 2 + 1
    epb = int(np.prod(dims))
    prefix = epb // L
    idist = epb if idist is None else idist
    odist = prefix * H if odist is None else odist
    x = np.asarray(x, np.float32)
    dense = np.zeros(batch * epb, np.complex64)
    for b in range(batch):
        dense[b * epb:(b + 1) * epb] = x[b * idist + np.arange(epb) * istride]
    X = fft_c2c(dense, dims, batch, -1, exact=True, threads=threads).reshape(batch, prefix, L)
    out = np.zeros((batch - 1) * odist + (prefix * H - 1) * ostride + 1, np.complex128)
    for b in range(batch):
        out[b * odist + np.arange(prefix * H) * ostride] = X[b, :, :H].reshape(-1)
    return out


def fft_c2r(X, dims, batch, *, istride=1, idist=None, ostride=1, odist=None, threads=8):
    """Reference C2R (cufft_exec.mm:305-436): gather the half spectrum (cufft_kernels.metal:
    79-92), inverse C2C over the leading axes, expand each last-axis row by conjugate
    symmetry (:94-117), inverse C2C of the last axis, keep the real part (:119-132).
    Returns float64 reals in the output layout (no scaling)."""
    dims = list(dims)
    L = dims[-1]
    H = L // 2 + 1
    epb = int(np.prod(dims))
    prefix = epb // L
    idist = prefix * H if idist is None else idist
    odist = epb if odist is None else odist
    X = np.asarray(X, np.complex64)
    A = np.zeros((batch, prefix * H), np.complex128)
    for b in range(batch):
        A[b] = X[b * idist + np.arange(prefix * H) * istride]
    if len(dims) > 1:
        for b in range(batch):
            # leading axes: a (rank-1)-dim transform per last-axis entry h (stride H)
            A[b] = fft_c2c(A[b].astype(np.complex64), dims[:-1], H, +1, istride=H, idist=1,
                           ostride=H, odist=1, exact=True, threads=threads)
    A = A.reshape(batch * prefix, H)
    full = np.zeros((batch * prefix, L), np.complex128)
    full[:, :H] = A[:, :min(H, L)]
    if L > H:
        full[:, H:] = np.conj(A[:, L - np.arange(H, L)])
    y = fft_c2c(full.reshape(-1).astype(np.complex64), [L], batch * prefix, +1, exact=True,
                threads=threads).real.reshape(batch, epb)
    out = np.zeros((batch - 1) * odist + (epb - 1) * ostride + 1, np.float64)
    for b in range(batch):
        out[b * odist + np.arange(epb) * ostride] = y[b]
    return out
