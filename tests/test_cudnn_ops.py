"""cuDNN neighbours of the convolution: backward data / filter / bias, AddTensor,
activation, pooling, batch norm (fp32).

CPU: the oracle restatements (cudnn_kernels.metal:194-714) against the reference's
known answers (tests/cudnn_test.cpp:33-160, 163-300) and the adjoint identity
<conv(x, w), dy> = <x, bwd_data(w, dy)> = <w, bwd_filter(x, dy)>; descriptor and
argument checks of the C ABI.
GPU (marked), through the C ABI against the oracle:
  - backward data, AddTensor, ReLU / clipped ReLU / identity and pooling: bit-exact
    (same per-output operation order as the reference);
  - backward filter / bias and batch-norm training (reductions split and combined in
    a fixed order): |got - exact| <= 1e-5 * (|alpha| sum |terms| + |beta * old|) against
    the float64 sums;
  - sigmoid / tanh / ELU / swish and batch-norm inference (device expf, tanhf, rsqrtf
    against host libm): |got - ref| <= 2e-6 * max(1, |ref|).
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import Dnn, fptr


def test_oracle_reference_conv_pins():
    """cudnn_test.cpp:37-145: N=1, C=2, 4x4, K=2, 3x3, pad 1; x = 1, w = 0.5, bias
    (1.25, -0.75); dy = 1."""
    x = np.ones(32, np.float32)
    w = np.full(36, 0.5, np.float32)
    y = oracle.conv2d(x, w, (1, 2, 4, 4), (2, 2, 3, 3), pad=(1, 1))
    b = np.array([1.25, -0.75], np.float32)
    oracle.add_tensor(b, (1, 2, 1, 1), y, (1, 2, 4, 4), beta=1.0)
    assert abs(y[0] - 5.25) < 1e-4 and abs(y[5] - 10.25) < 1e-4
    dy = np.ones(32, np.float32)
    db, _ = oracle.conv_bwd_bias(dy, (1, 2, 4, 4))
    assert np.allclose(db, 16.0, atol=1e-4)
    dw = oracle.conv_bwd_filter(x, dy, (1, 2, 4, 4), (2, 2, 3, 3), pad=(1, 1))
    assert abs(dw[4] - 16.0) < 1e-4
    dx = oracle.conv_bwd_data(w, dy, (1, 2, 4, 4), (2, 2, 3, 3), pad=(1, 1))
    assert abs(dx[5] - 9.0) < 1e-4 and abs(dx[0] - 4.0) < 1e-4  # 2 channels * 0.5 * taps


REF_IN = np.array([-2.0, -0.5, 0.0, 1.5, -3.0, 2.0, 4.0, -1.0], np.float32)


def test_oracle_reference_activation_pool_bn_pins():
    """cudnn_test.cpp:168-300."""
    y = oracle.activation(REF_IN, (1, 2, 2, 2), np.zeros(8, np.float32), capi.CUDNN_ACTIVATION_RELU)
    assert np.array_equal(y, np.maximum(REF_IN, 0))
    p = oracle.pooling(REF_IN, (1, 2, 2, 2), np.zeros(2, np.float32), (1, 2, 1, 1), (2, 2), (0, 0),
                       (2, 2), capi.CUDNN_POOLING_MAX)
    assert p[0] == 1.5 and p[1] == 4.0
    out = oracle.bn_inference(REF_IN, (1, 2, 2, 2), np.zeros(8, np.float32),
                              np.array([1, 2], np.float32), np.array([0.5, -0.5], np.float32),
                              np.zeros(2, np.float32), np.ones(2, np.float32), eps=1e-5)
    assert abs(out[0] - (-1.5)) < 1e-3 and abs(out[5] - 3.5) < 1e-3


GEOMS = [  # xshape, wshape, geometry
    ((2, 6, 9, 8), (4, 3, 3, 2), dict(pad=(1, 0), stride=(2, 1), dil=(1, 2), groups=2)),
    ((1, 4, 7, 7), (5, 4, 3, 3), dict(pad=(1, 1), mode="conv")),
    ((3, 8, 10, 6), (8, 8, 1, 1), dict(stride=(2, 3), x_fmt="NHWC", w_fmt="NHWC")),
    ((2, 3, 12, 12), (6, 3, 5, 3), dict(pad=(2, 1), stride=(3, 2), dil=(2, 1))),
]


@pytest.mark.parametrize("xs,ws,geom", GEOMS)
def test_oracle_adjoint_identity(xs, ws, geom):
    rng = np.random.default_rng(sum(xs))
    x = rng.standard_normal(int(np.prod(xs))).astype(np.float32)
    w = rng.standard_normal(int(np.prod(ws))).astype(np.float32)
    y = oracle.conv2d(x, w, xs, ws, accum_f64=True, **geom)
    dy = rng.standard_normal(y.size).astype(np.float32)
    dx = oracle.conv_bwd_data(w, dy, xs, ws, accum_f64=True, **geom)
    dw = oracle.conv_bwd_filter(x, dy, xs, ws, accum_f64=True, **geom)
    a = np.dot(y.astype(np.float64), dy)
    assert abs(np.dot(x.astype(np.float64), dx) - a) <= 1e-5 * max(1, abs(a))
    assert abs(np.dot(w.astype(np.float64), dw) - a) <= 1e-5 * max(1, abs(a))


def test_host_logic(built):
    with Dnn() as d:
        L = d.L
        act = C.c_void_p()
        assert L.cudnnCreateActivationDescriptor(None) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnCreateActivationDescriptor(C.byref(act)) == 0
        m, nan, coef = C.c_int(), C.c_int(), C.c_double()
        assert L.cudnnGetActivationDescriptor(act, C.byref(m), C.byref(nan), C.byref(coef)) == \
            capi.CUDNN_STATUS_BAD_PARAM  # not configured
        assert L.cudnnSetActivationDescriptor(act, 7, 0, 0.0) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnSetActivationDescriptor(act, capi.CUDNN_ACTIVATION_ELU, 1, 0.75) == 0
        assert L.cudnnGetActivationDescriptor(act, C.byref(m), C.byref(nan), C.byref(coef)) == 0
        assert (m.value, nan.value, coef.value) == (4, 1, 0.75)
        pool = C.c_void_p()
        assert L.cudnnCreatePoolingDescriptor(C.byref(pool)) == 0
        for args in ((0, 0, 0, 2, 0, 0, 1, 1), (0, 0, 2, 2, -1, 0, 1, 1), (0, 0, 2, 2, 0, 0, 0, 1),
                     (4, 0, 2, 2, 0, 0, 1, 1)):
            assert L.cudnnSetPooling2dDescriptor(pool, *args) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnSetPooling2dDescriptor(pool, capi.CUDNN_POOLING_MAX, 0, 3, 2, 1, 0, 2, 2) == 0
        x = d.tensor(2, 3, 9, 8)
        dims = [C.c_int() for _ in range(4)]
        assert L.cudnnGetPooling2dForwardOutputDim(pool, x, *[C.byref(v) for v in dims]) == 0
        assert [v.value for v in dims] == [2, 3, 1 + (9 + 2 - 3) // 2, 1 + (8 - 2) // 2]
        bn = d.tensor(1, 1, 1, 1)
        assert L.cudnnDeriveBNTensorDescriptor(bn, x, capi.CUDNN_BATCHNORM_SPATIAL) == 0
        n_, c_, h_, w_ = (C.c_int() for _ in range(4))
        dt = C.c_int()
        st = [C.c_int() for _ in range(4)]
        assert L.cudnnGetTensor4dDescriptor(bn, C.byref(dt), C.byref(n_), C.byref(c_), C.byref(h_),
                                            C.byref(w_), *[C.byref(v) for v in st]) == 0
        assert (n_.value, c_.value, h_.value, w_.value) == (1, 3, 1, 1)
        assert L.cudnnDeriveBNTensorDescriptor(bn, x, capi.CUDNN_BATCHNORM_PER_ACTIVATION) == 0
        p = C.c_void_p(4096)
        one = fptr(1.0)
        # argument checks before any device access (cudnn_ops.mm:385-460, 550-570, 722-740)
        assert L.cudnnAddTensor(d.h, one, x, None, one, x, p) == capi.CUDNN_STATUS_BAD_PARAM
        big = d.tensor(2, 3, 9, 9)
        assert L.cudnnAddTensor(d.h, one, big, p, one, x, p) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnActivationForward(d.h, act, one, x, p, one, big, p) == \
            capi.CUDNN_STATUS_BAD_PARAM
        xh = d.tensor(2, 3, 9, 8, dtype=capi.CUDNN_DATA_HALF)
        assert L.cudnnActivationForward(d.h, act, one, xh, p, one, xh, p) == \
            capi.CUDNN_STATUS_NOT_SUPPORTED
        assert L.cudnnActivationForward(d.h, act, one, x, p, one, x, p) == \
            capi.CUDNN_STATUS_BAD_PARAM  # unaddressable
        assert L.cudnnBatchNormalizationForwardInference(d.h, 1, one, one, x, p, x, p, bn, p, p,
                                                         p, p, 0.0) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnBatchNormalizationForwardTraining(d.h, 1, one, one, x, p, x, p, bn, p, p,
                                                        0.1, p, None, 1e-5, None, None) == \
            capi.CUDNN_STATUS_BAD_PARAM  # running mean without variance
        db = d.tensor(1, 4, 1, 1)
        assert L.cudnnConvolutionBackwardBias(d.h, one, x, p, one, db, p) == \
            capi.CUDNN_STATUS_BAD_PARAM  # channel mismatch
        assert L.cudnnDestroyActivationDescriptor(act) == 0
        assert L.cudnnDestroyActivationDescriptor(act) == capi.CUDNN_STATUS_BAD_PARAM
        assert L.cudnnDestroyPoolingDescriptor(pool) == 0


# --------------------------------------------------------------------- GPU --
def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _p(t):
    return C.c_void_p(t.data_ptr())


def _strides(shape, fmt):
    n, c, h, w = shape
    return (c * h * w, h * w, w, 1) if fmt == "NCHW" else (h * w * c, 1, w * c, c)


def _tdesc(d, shape, fmt):
    return d.tensor(*shape, strides=_strides(shape, fmt))


def _fmt_code(fmt):
    return capi.CUDNN_TENSOR_NCHW if fmt == "NCHW" else capi.CUDNN_TENSOR_NHWC


@pytest.mark.gpu
def test_gpu_reference_pins(cuda, built):
    """tests/cudnn_test.cpp:33-300 on the GPU."""
    torch = cuda
    with Dnn(torch) as d:
        L = d.L
        x_d, y_d, b_d = d.tensor(1, 2, 4, 4), d.tensor(1, 2, 4, 4), d.tensor(1, 2, 1, 1)
        w_d = d.filter(2, 2, 3, 3)
        cv = d.conv(pad=(1, 1))
        x = _dev(torch, np.ones(32))
        w = _dev(torch, np.full(36, 0.5))
        y = torch.zeros(32, device="cuda")
        b = _dev(torch, [1.25, -0.75])
        one, zero = fptr(1.0), fptr(0.0)
        assert L.cudnnConvolutionForward(d.h, one, x_d, _p(x), w_d, _p(w), cv, 0, None, 0, zero,
                                         y_d, _p(y)) == 0
        assert L.cudnnAddTensor(d.h, one, b_d, _p(b), one, y_d, _p(y)) == 0
        torch.cuda.synchronize()
        yh = y.cpu().numpy()
        assert abs(yh[0] - 5.25) < 1e-4 and abs(yh[5] - 10.25) < 1e-4
        dy = _dev(torch, np.ones(32))
        assert L.cudnnConvolutionBackwardBias(d.h, one, y_d, _p(dy), zero, b_d, _p(b)) == 0
        dw = torch.zeros(36, device="cuda")
        dx = torch.zeros(32, device="cuda")
        assert L.cudnnConvolutionBackwardFilter(d.h, one, x_d, _p(x), y_d, _p(dy), cv, 0, None, 0,
                                                zero, w_d, _p(dw)) == 0
        assert L.cudnnConvolutionBackwardData(d.h, one, w_d, _p(w), y_d, _p(dy), cv, 0, None, 0,
                                              zero, x_d, _p(dx)) == 0
        torch.cuda.synchronize()
        assert np.allclose(b.cpu().numpy(), 16.0, atol=1e-4)
        assert abs(dw.cpu().numpy()[4] - 16.0) < 1e-4
        t = d.tensor(1, 2, 2, 2)
        act = C.c_void_p()
        assert L.cudnnCreateActivationDescriptor(C.byref(act)) == 0
        assert L.cudnnSetActivationDescriptor(act, capi.CUDNN_ACTIVATION_RELU, 0, 0.0) == 0
        xin = _dev(torch, REF_IN)
        out = torch.zeros(8, device="cuda")
        assert L.cudnnActivationForward(d.h, act, one, t, _p(xin), zero, t, _p(out)) == 0
        pool = C.c_void_p()
        assert L.cudnnCreatePoolingDescriptor(C.byref(pool)) == 0
        assert L.cudnnSetPooling2dDescriptor(pool, capi.CUDNN_POOLING_MAX, 0, 2, 2, 0, 0, 2, 2) == 0
        po = torch.zeros(2, device="cuda")
        pd = d.tensor(1, 2, 1, 1)
        assert L.cudnnPoolingForward(d.h, pool, one, t, _p(xin), zero, pd, _p(po)) == 0
        bn = d.tensor(1, 1, 1, 1)
        assert L.cudnnDeriveBNTensorDescriptor(bn, t, capi.CUDNN_BATCHNORM_SPATIAL) == 0
        sc, bi = _dev(torch, [1, 2]), _dev(torch, [0.5, -0.5])
        mu, var = _dev(torch, [0, 0]), _dev(torch, [1, 1])
        bo = torch.zeros(8, device="cuda")
        assert L.cudnnBatchNormalizationForwardInference(d.h, 1, one, zero, t, _p(xin), t, _p(bo),
                                                         bn, _p(sc), _p(bi), _p(mu), _p(var),
                                                         1e-5) == 0
        assert L.cudnnBatchNormalizationForwardTraining(d.h, 1, one, zero, t, _p(xin), t, _p(bo),
                                                        bn, _p(sc), _p(bi), 0.1, _p(mu), _p(var),
                                                        1e-5, None, None) == 0
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), np.maximum(REF_IN, 0))
        assert np.array_equal(po.cpu().numpy(), [1.5, 4.0])
        assert L.cudnnDestroyActivationDescriptor(act) == 0
        assert L.cudnnDestroyPoolingDescriptor(pool) == 0


CONV_CASES = [  # xshape, wshape, pad, stride, dil, groups, mode, fmt
    ((2, 6, 9, 8), (4, 3, 3, 2), (1, 0), (2, 1), (1, 2), 2, "cross", "NCHW"),
    ((1, 4, 7, 7), (5, 4, 3, 3), (1, 1), (1, 1), (1, 1), 1, "conv", "NCHW"),
    ((3, 8, 10, 6), (8, 8, 1, 1), (0, 0), (2, 3), (1, 1), 1, "cross", "NHWC"),
    ((2, 3, 12, 12), (6, 3, 5, 3), (2, 1), (3, 2), (2, 1), 1, "cross", "NCHW"),
    ((4, 32, 14, 14), (64, 32, 3, 3), (1, 1), (1, 1), (1, 1), 1, "cross", "NHWC"),
    # tensor-core paths (split tf32): backward data needs stride 1, NHWC, K % 32 == 0
    ((8, 64, 28, 28), (64, 64, 3, 3), (1, 1), (1, 1), (1, 1), 1, "cross", "NHWC"),
    ((4, 32, 20, 20), (64, 32, 3, 3), (1, 1), (1, 1), (2, 2), 1, "conv", "NHWC"),
    ((2, 64, 16, 16), (32, 64, 5, 5), (2, 2), (1, 1), (1, 1), 1, "cross", "NHWC"),
    ((8, 64, 28, 28), (64, 64, 3, 3), (1, 1), (2, 2), (1, 1), 1, "cross", "NHWC"),
    ((8, 64, 28, 28), (64, 64, 3, 3), (1, 1), (1, 1), (1, 1), 1, "cross", "NCHW"),
    # channels and pixels that fill neither a 32-channel nor a 32-pixel tile
    ((6, 40, 13, 11), (64, 40, 3, 3), (1, 1), (1, 1), (1, 1), 1, "cross", "NHWC"),
]


def _tc_paths(case, ys):
    """(backward data, backward filter) take the split-tf32 tensor-core path: the
    library's selection rule (conv_bwd_tc.cu, conv_tc_kernels.cu tf32_geometry_ok)."""
    xs, ws, pad, stride, dil, groups, mode, fmt = case
    n, c, h, w = xs
    k, _, r, s = ws
    data = (groups == 1 and stride == (1, 1) and fmt == "NHWC" and k % 32 == 0 and c % 4 == 0
            and n * h * w * c * k * r * s >= (1 << 24))
    filt = groups == 1 and (c * r * s) * k * (ys[0] * ys[2] * ys[3]) >= (1 << 24)
    return data, filt


def _conv_setup(d, case):
    xs, ws, pad, stride, dil, groups, mode, fmt = case
    geom = dict(pad=pad, stride=stride, dil=dil, groups=groups, mode=mode, x_fmt=fmt, w_fmt=fmt)
    _, ys = oracle.conv_params(xs, ws, **geom)
    xd = _tdesc(d, xs, fmt)
    yd = _tdesc(d, ys, fmt)
    wd = d.filter(*ws, fmt=_fmt_code(fmt))
    cd = d.conv(pad=pad, stride=stride, dil=dil, groups=groups,
                mode=capi.CUDNN_CONVOLUTION if mode == "conv" else capi.CUDNN_CROSS_CORRELATION)
    return geom, ys, xd, yd, wd, cd


@pytest.mark.gpu
@pytest.mark.parametrize("case", CONV_CASES)
def test_gpu_conv_backward(cuda, built, case):
    torch = cuda
    xs, ws = case[0], case[1]
    rng = np.random.default_rng(sum(xs) + sum(ws))
    with Dnn(torch) as d:
        geom, ys, xd, yd, wd, cd = _conv_setup(d, case)
        x = rng.uniform(-1, 1, int(np.prod(xs))).astype(np.float32)
        w = rng.uniform(-1, 1, int(np.prod(ws))).astype(np.float32)
        dy = rng.uniform(-1, 1, int(np.prod(ys))).astype(np.float32)
        dx0 = rng.uniform(-1, 1, x.size).astype(np.float32)
        dw0 = rng.uniform(-1, 1, w.size).astype(np.float32)
        for alpha, beta in ((1.0, 0.0), (0.75, -0.5)):
            tdx, tdw = _dev(torch, dx0), _dev(torch, dw0)
            assert d.L.cudnnConvolutionBackwardData(d.h, fptr(alpha), wd, _p(_w := _dev(torch, w)),
                                                    yd, _p(_dy := _dev(torch, dy)), cd, 0, None, 0,
                                                    fptr(beta), xd, _p(tdx)) == 0
            assert d.L.cudnnConvolutionBackwardFilter(d.h, fptr(alpha), xd, _p(_x := _dev(torch, x)),
                                                      yd, _p(_dy), cd, 0, None, 0, fptr(beta), wd,
                                                      _p(tdw)) == 0
            torch.cuda.synchronize()
            tc_data, _ = _tc_paths(case, ys)
            if not tc_data:
                want_dx = oracle.conv_bwd_data(w, dy, xs, ws, dx0.copy(), alpha=alpha, beta=beta,
                                               **geom)
                assert np.array_equal(tdx.cpu().numpy(), want_dx)  # bit-exact
            else:
                exact = oracle.conv_bwd_data(w, dy, xs, ws, dx0.copy(), accum_f64=True,
                                             alpha=alpha, beta=beta, **geom)
                mag = oracle.conv_bwd_data(np.abs(w), np.abs(dy), xs, ws, accum_f64=True, **geom)
                scale = abs(alpha) * mag.astype(np.float64) + abs(beta) * np.abs(dx0)
                err = np.abs(tdx.cpu().numpy().astype(np.float64) - exact)
                assert np.all(err <= 1e-5 * scale + 1e-30), np.max(err / (scale + 1e-30))
            exact, mag = oracle.conv_bwd_filter(x, dy, xs, ws, dw0.copy(), accum_f64=True,
                                                with_mag=True, alpha=alpha, beta=beta, **geom)
            scale = abs(alpha) * mag + abs(beta) * np.abs(dw0)
            err = np.abs(tdw.cpu().numpy().astype(np.float64) - exact)
            assert np.all(err <= 1e-5 * scale + 1e-30), np.max(err / (scale + 1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("shape,fmt", [((2, 5, 7, 9), "NCHW"), ((8, 64, 28, 28), "NHWC"),
                                       ((1, 3, 1, 1), "NCHW")])
def test_gpu_backward_bias(cuda, built, shape, fmt):
    torch = cuda
    rng = np.random.default_rng(shape[1])
    with Dnn(torch) as d:
        dyd = _tdesc(d, shape, fmt)
        dbd = d.tensor(1, shape[1], 1, 1)
        dy = rng.uniform(-1, 1, int(np.prod(shape))).astype(np.float32)
        db0 = rng.uniform(-1, 1, shape[1]).astype(np.float32)
        tdb = _dev(torch, db0)
        assert d.L.cudnnConvolutionBackwardBias(d.h, fptr(0.5), dyd, _p(_dev(torch, dy)),
                                                fptr(2.0), dbd, _p(tdb)) == 0
        torch.cuda.synchronize()
        exact, mag = oracle.conv_bwd_bias(dy, shape, db0.copy(), strides=_strides(shape, fmt),
                                          alpha=0.5, beta=2.0, accum_f64=True)
        err = np.abs(tdb.cpu().numpy().astype(np.float64) - exact)
        assert np.all(err <= 1e-5 * (0.5 * mag + 2 * np.abs(db0)) + 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("ashape", [(1, 6, 1, 1), (3, 6, 5, 7), (1, 1, 5, 7), (3, 1, 1, 7)])
@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_gpu_add_tensor(cuda, built, ashape, beta):
    torch = cuda
    cshape = (3, 6, 5, 7)
    rng = np.random.default_rng(sum(ashape))
    with Dnn(torch) as d:
        ad = d.tensor(*ashape)
        cd_ = _tdesc(d, cshape, "NHWC")
        a = rng.uniform(-1, 1, int(np.prod(ashape))).astype(np.float32)
        c0 = rng.uniform(-1, 1, int(np.prod(cshape))).astype(np.float32)
        tc = _dev(torch, c0)
        assert d.L.cudnnAddTensor(d.h, fptr(1.5), ad, _p(_dev(torch, a)), fptr(beta), cd_,
                                  _p(tc)) == 0
        torch.cuda.synchronize()
        want = oracle.add_tensor(a, ashape, c0.copy(), cshape, cstrides=_strides(cshape, "NHWC"),
                                 alpha=1.5, beta=beta)
        assert np.array_equal(tc.cpu().numpy(), want)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", range(7))
@pytest.mark.parametrize("layout", ["packed", "strided"])
def test_gpu_activation(cuda, built, mode, layout):
    torch = cuda
    shape = (4, 6, 9, 10) if layout == "packed" else (3, 5, 7, 9)
    rng = np.random.default_rng(mode)
    x = (rng.standard_normal(int(np.prod(shape))) * 3).astype(np.float32)
    x[:4] = [0.0, -0.0, np.inf, -np.inf]
    with Dnn(torch) as d:
        act = C.c_void_p()
        assert d.L.cudnnCreateActivationDescriptor(C.byref(act)) == 0
        assert d.L.cudnnSetActivationDescriptor(act, mode, 0, 1.25) == 0
        fmt = "NCHW" if layout == "packed" else "NHWC"
        xd, yd = _tdesc(d, shape, "NCHW"), _tdesc(d, shape, fmt)
        y0 = rng.uniform(-1, 1, x.size).astype(np.float32)
        for beta in (0.0, 0.25):
            ty = _dev(torch, y0)
            assert d.L.cudnnActivationForward(d.h, act, fptr(0.5), xd, _p(_dev(torch, x)),
                                              fptr(beta), yd, _p(ty)) == 0
            torch.cuda.synchronize()
            want = oracle.activation(x, shape, y0.copy(), mode, coef=1.25,
                                     ystrides=_strides(shape, fmt), alpha=0.5, beta=beta)
            got = ty.cpu().numpy()
            if mode in (1, 3, 5):
                assert np.array_equal(got, want)
            else:
                fin = np.isfinite(want)
                assert np.array_equal(np.isfinite(got), fin)
                assert np.all(np.abs(got[fin] - want[fin]) <= 2e-6 * np.maximum(1, np.abs(want[fin])))
        assert d.L.cudnnDestroyActivationDescriptor(act) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("mode", range(4))
@pytest.mark.parametrize("win,pad,stride", [((2, 2), (0, 0), (2, 2)), ((3, 3), (1, 1), (2, 2)),
                                            ((3, 2), (1, 0), (1, 2))])
@pytest.mark.parametrize("yfmt", ["NHWC", "NCHW"])  # NCHW in and out: the per-plane kernel
def test_gpu_pooling(cuda, built, mode, win, pad, stride, yfmt):
    torch = cuda
    xs = (2, 5, 11, 10)
    rng = np.random.default_rng(mode + win[0])
    x = rng.standard_normal(int(np.prod(xs))).astype(np.float32)
    with Dnn(torch) as d:
        pool = C.c_void_p()
        assert d.L.cudnnCreatePoolingDescriptor(C.byref(pool)) == 0
        assert d.L.cudnnSetPooling2dDescriptor(pool, mode, 0, *win, *pad, *stride) == 0
        xd = d.tensor(*xs)
        dims = [C.c_int() for _ in range(4)]
        assert d.L.cudnnGetPooling2dForwardOutputDim(pool, xd, *[C.byref(v) for v in dims]) == 0
        ys = tuple(v.value for v in dims)
        yd = _tdesc(d, ys, yfmt)
        y0 = rng.standard_normal(int(np.prod(ys))).astype(np.float32)
        ty = _dev(torch, y0)
        assert d.L.cudnnPoolingForward(d.h, pool, fptr(1.0), xd, _p(_dev(torch, x)), fptr(0.5), yd,
                                       _p(ty)) == 0
        torch.cuda.synchronize()
        want = oracle.pooling(x, xs, y0.copy(), ys, win, pad, stride, mode,
                              ystrides=_strides(ys, yfmt), beta=0.5)
        assert np.array_equal(ty.cpu().numpy(), want)
        assert d.L.cudnnDestroyPoolingDescriptor(pool) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("per_activation", [False, True])
def test_gpu_batchnorm_inference(cuda, built, per_activation):
    torch = cuda
    shape = (4, 8, 6, 5)
    rng = np.random.default_rng(int(per_activation))
    pe = 8 * 6 * 5 if per_activation else 8
    x = rng.standard_normal(int(np.prod(shape))).astype(np.float32)
    sc, bi = rng.uniform(0.5, 2, pe).astype(np.float32), rng.uniform(-1, 1, pe).astype(np.float32)
    mu, var = rng.uniform(-1, 1, pe).astype(np.float32), rng.uniform(0.1, 3, pe).astype(np.float32)
    mode = capi.CUDNN_BATCHNORM_PER_ACTIVATION if per_activation else capi.CUDNN_BATCHNORM_SPATIAL
    with Dnn(torch) as d:
        xd = d.tensor(*shape)
        bn = d.tensor(1, 1, 1, 1)
        assert d.L.cudnnDeriveBNTensorDescriptor(bn, xd, mode) == 0
        y0 = rng.standard_normal(x.size).astype(np.float32)
        ty = _dev(torch, y0)
        assert d.L.cudnnBatchNormalizationForwardInference(
            d.h, mode, fptr(1.0), fptr(0.5), xd, _p(_dev(torch, x)), xd, _p(ty), bn,
            _p(_dev(torch, sc)), _p(_dev(torch, bi)), _p(_dev(torch, mu)), _p(_dev(torch, var)),
            1e-3) == 0
        torch.cuda.synchronize()
        want = oracle.bn_inference(x, shape, y0.copy(), sc, bi, mu, var,
                                   per_activation=per_activation, eps=1e-3, beta=0.5)
        got = ty.cpu().numpy()
        assert np.all(np.abs(got - want) <= 2e-6 * np.maximum(1, np.abs(want)))


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(4, 8, 6, 5), (32, 16, 28, 28), (1, 3, 1, 1)])
def test_gpu_batchnorm_training(cuda, built, shape):
    torch = cuda
    c = shape[1]
    rng = np.random.default_rng(shape[0])
    x = (rng.standard_normal(int(np.prod(shape))) * 2 + 0.7).astype(np.float32)
    sc, bi = rng.uniform(0.5, 2, c).astype(np.float32), rng.uniform(-1, 1, c).astype(np.float32)
    rm0, rv0 = rng.uniform(-1, 1, c).astype(np.float32), rng.uniform(0.5, 2, c).astype(np.float32)
    with Dnn(torch) as d:
        xd = d.tensor(*shape)
        bn = d.tensor(1, 1, 1, 1)
        assert d.L.cudnnDeriveBNTensorDescriptor(bn, xd, capi.CUDNN_BATCHNORM_SPATIAL) == 0
        ty = torch.zeros(x.size, device="cuda")
        trm, trv = _dev(torch, rm0), _dev(torch, rv0)
        tsm, tsv = torch.zeros(c, device="cuda"), torch.zeros(c, device="cuda")
        assert d.L.cudnnBatchNormalizationForwardTraining(
            d.h, capi.CUDNN_BATCHNORM_SPATIAL, fptr(1.0), fptr(0.0), xd, _p(_dev(torch, x)), xd,
            _p(ty), bn, _p(_dev(torch, sc)), _p(_dev(torch, bi)), 0.25, _p(trm), _p(trv), 1e-5,
            _p(tsm), _p(tsv)) == 0
        torch.cuda.synchronize()
        rm, rv = rm0.copy(), rv0.copy()
        sm, sv = np.zeros(c, np.float32), np.zeros(c, np.float32)
        want = oracle.bn_training(x, shape, np.zeros(x.size, np.float32), sc, bi, running=(rm, rv),
                                  save=(sm, sv), factor=0.25, eps=1e-5, accum_f64=True)
        tol = lambda w: 2e-5 * np.maximum(1, np.abs(w))
        assert np.all(np.abs(tsm.cpu().numpy() - sm) <= tol(sm))
        assert np.all(np.abs(tsv.cpu().numpy() - sv) <= tol(sv))
        assert np.all(np.abs(trm.cpu().numpy() - rm) <= tol(rm))
        assert np.all(np.abs(trv.cpu().numpy() - rv) <= tol(rv))
        assert np.all(np.abs(ty.cpu().numpy() - want) <= tol(want))
