"""ctypes prototypes of the non-RNG oracle functions (test infrastructure only)."""

from __future__ import annotations

import ctypes as C


class ConvParams(C.Structure):
    """Mirror of OracleConvParams in oracle/oracle.h."""
    _fields_ = [
        ("n", C.c_int), ("c_in", C.c_int), ("h_in", C.c_int), ("w_in", C.c_int),
        ("x_ns", C.c_int64), ("x_cs", C.c_int64), ("x_hs", C.c_int64), ("x_ws", C.c_int64),
        ("c_out", C.c_int), ("h_out", C.c_int), ("w_out", C.c_int), ("groups", C.c_int),
        ("y_ns", C.c_int64), ("y_cs", C.c_int64), ("y_hs", C.c_int64), ("y_ws", C.c_int64),
        ("kh", C.c_int), ("kw", C.c_int), ("pad_h", C.c_int), ("pad_w", C.c_int),
        ("stride_h", C.c_int), ("stride_w", C.c_int), ("dil_h", C.c_int), ("dil_w", C.c_int),
        ("w_format", C.c_int), ("conv_mode", C.c_int),
        ("alpha", C.c_float), ("beta", C.c_float),
    ]


class Tensor4(C.Structure):
    """Mirror of OracleTensor4 in oracle/oracle.h."""
    _fields_ = [("n", C.c_int), ("c", C.c_int), ("h", C.c_int), ("w", C.c_int),
                ("ns", C.c_int64), ("cs", C.c_int64), ("hs", C.c_int64), ("ws", C.c_int64)]


vp = C.c_void_p
fp = C.POINTER(C.c_float)

_PROTOS: list[tuple[str, list, object]] = [
    ("oracle_bf16_round", [C.c_float], C.c_float),
    ("oracle_conv2d_fwd", [vp, vp, vp, C.POINTER(ConvParams), C.c_int, C.c_int, C.c_int], None),
    ("oracle_softmax_fwd", [fp, fp, C.POINTER(Tensor4), C.POINTER(Tensor4), C.c_int, C.c_int,
                            C.c_float, C.c_float, C.c_int], None),
    ("oracle_half_round", [C.c_float], C.c_float),
    ("oracle_gemm", [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp,
                     C.c_int64, C.c_int64, vp, C.c_int64, C.c_int64, C.c_float, vp, C.c_int64,
                     C.c_int64, C.c_int, C.c_int, vp, vp, C.c_int64, C.c_int], None),
    ("oracle_saxpy", [C.c_int, C.c_float, vp, C.c_int, vp, C.c_int], None),
    ("oracle_daxpy", [C.c_int, C.c_double, vp, C.c_int, vp, C.c_int], None),
    ("oracle_dcopy", [C.c_int, vp, C.c_int, vp, C.c_int], None),
    ("oracle_dscal", [C.c_int, C.c_double, vp, C.c_int], None),
    ("oracle_dswap", [C.c_int, vp, C.c_int, vp, C.c_int], None),
    ("oracle_dreduce", [C.c_int, C.c_int, vp, C.c_int, vp, C.c_int, vp], None),
    ("oracle_idamax", [C.c_int, vp, C.c_int], C.c_int),
    ("oracle_dgemv", [C.c_int, C.c_int, C.c_int, C.c_double, vp, C.c_int, vp, C.c_int,
                      C.c_double, vp, C.c_int, vp, C.c_int], None),
    ("oracle_dgemm", [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_double, vp, C.c_int64,
                      C.c_int64, vp, C.c_int64, C.c_int64, C.c_double, vp, C.c_int64, C.c_int64,
                      C.c_int, vp, vp, C.c_int, vp, C.c_int], None),
    ("oracle_scopy", [C.c_int, vp, C.c_int, vp, C.c_int], None),
    ("oracle_sscal", [C.c_int, C.c_float, vp, C.c_int], None),
    ("oracle_sswap", [C.c_int, vp, C.c_int, vp, C.c_int], None),
    ("oracle_sreduce", [C.c_int, C.c_int, vp, C.c_int, vp, C.c_int, vp, vp, vp], None),
    ("oracle_isamax", [C.c_int, vp, C.c_int], C.c_int),
    ("oracle_sgeam", [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, vp, C.c_int64, C.c_float,
                      vp, C.c_int64, vp, C.c_int64, C.c_int], None),
    ("oracle_dgeam", [C.c_int, C.c_int, C.c_int, C.c_int, C.c_double, vp, C.c_int64,
                      C.c_double, vp, C.c_int64, vp, C.c_int64, C.c_int], None),
    ("oracle_sgemv", [C.c_int, C.c_int, C.c_int, C.c_float, vp, C.c_int64, vp, C.c_int, C.c_float,
                      vp, C.c_int, vp, vp, C.c_int], None),
    ("oracle_fft_c2c", [vp, vp, C.c_int, vp, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                        C.c_int64, C.c_int, C.c_int, vp, C.c_int], None),
    ("oracle_spmv_csr", [C.c_int64, vp, vp, vp, C.c_int, vp, vp, C.c_float, C.c_float, vp,
                         vp, C.c_int], None),
    ("oracle_generate_lognormal", [C.c_uint64, C.c_uint64, vp, C.c_size_t, C.c_float, C.c_float,
                                   C.c_int], C.c_uint64),
    ("oracle_generate_double", [C.c_uint64, C.c_uint64, vp, C.c_size_t, C.c_int, C.c_double,
                                C.c_double, C.c_int], C.c_uint64),
    ("oracle_generate_poisson", [C.c_uint64, C.c_uint64, vp, C.c_size_t, C.c_double, C.c_float,
                                 C.c_int, C.c_int], C.c_uint64),
    ("oracle_conv_bwd_data", [vp, vp, vp, C.POINTER(ConvParams), C.c_int, C.c_int], None),
    ("oracle_conv_bwd_filter", [vp, vp, vp, C.POINTER(ConvParams), C.c_int, vp, C.c_int], None),
    ("oracle_conv_bwd_bias", [vp, C.POINTER(Tensor4), vp, C.c_float, C.c_float, C.c_int, vp],
     None),
    ("oracle_add_tensor", [vp, C.POINTER(Tensor4), vp, C.POINTER(Tensor4), C.c_float, C.c_float],
     None),
    ("oracle_activation", [vp, C.POINTER(Tensor4), vp, C.POINTER(Tensor4), C.c_int, C.c_float,
                           C.c_float, C.c_float], None),
    ("oracle_pooling", [vp, C.POINTER(Tensor4), vp, C.POINTER(Tensor4)] + [C.c_int] * 7 +
     [C.c_float, C.c_float], None),
    ("oracle_bn_inference", [vp, C.POINTER(Tensor4), vp, C.POINTER(Tensor4), vp, vp, vp, vp,
                             C.c_int, C.c_float, C.c_float, C.c_float], None),
    ("oracle_bn_training", [vp, C.POINTER(Tensor4), vp, C.POINTER(Tensor4), vp, vp, vp, vp, vp, vp,
                            C.c_float, C.c_float, C.c_float, C.c_float, C.c_int], None),
    ("oracle_spmv_csr_t", [C.c_int64, C.c_int64, vp, vp, vp, C.c_int, vp, vp, C.c_float,
                           C.c_float, C.c_int, vp, vp], None),
    ("oracle_spmm_csr", [C.c_int64, C.c_int64, vp, vp, vp, C.c_int, C.c_int, vp, C.c_int64,
                         C.c_int, C.c_int, vp, C.c_int64, C.c_int, C.c_int64, C.c_float,
                         C.c_float, vp, vp, C.c_int], None),
]


def declare(L: C.CDLL) -> None:
    for name, argtypes, restype in _PROTOS:
        fn = getattr(L, name, None)
        if fn is None:
            continue
        fn.argtypes = argtypes
        fn.restype = restype
