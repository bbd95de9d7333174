"""cudnnConvolutionForward / cudnnSoftmaxForward on the GPU through the C ABI,
checked against the pinned oracle.

Bar: fp32 within 1e-5 normwise relative error (and per element 2e-5 relative plus
1e-6 absolute); bf16 conv within 1e-2 normwise relative error of the oracle's
bf16 result.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import Dnn, fptr

pytestmark = pytest.mark.gpu

F32, BF16 = capi.CUDNN_DATA_FLOAT, capi.CUDNN_DATA_BFLOAT16
NCHW, NHWC = capi.CUDNN_TENSOR_NCHW, capi.CUDNN_TENSOR_NHWC


def normwise(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)


def check_f32(got, want, tol=1e-5, scale=None):
    """Normwise relative error <= tol, and per element |err| <= 2*tol*scale + 1e-6 where
    scale is |want| (softmax) or, for a convolution, the same convolution of |x| and |w|
    (the magnitude its rounding error is proportional to)."""
    assert normwise(got, want) <= tol, f"normwise {normwise(got, want):.3e}"
    err = np.abs(got.astype(np.float64) - want)
    scale = np.abs(want) if scale is None else scale
    assert np.all(err <= 2 * tol * scale + 1e-6), f"max elementwise {err.max():.3e}"


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_conv(torch, x, w, xshape, wshape, *, x_fmt=NCHW, w_fmt=NCHW, pad=(0, 0), stride=(1, 1),
             dil=(1, 1), groups=1, mode=capi.CUDNN_CROSS_CORRELATION, alpha=1.0, beta=0.0,
             y0=None, dtype=F32):
    n, c, h, wd = xshape
    k, cg, r, s = wshape
    with Dnn(torch) as d:
        xd = d.tensor(n, c, h, wd, fmt=x_fmt, dtype=dtype)
        wdsc = d.filter(k, cg, r, s, fmt=w_fmt, dtype=dtype)
        cv = d.conv(pad=pad, stride=stride, dil=dil, mode=mode, groups=groups)
        o = [C.c_int() for _ in range(4)]
        assert d.L.cudnnGetConvolution2dForwardOutputDim(cv, xd, wdsc, *[C.byref(v) for v in o]) == 0
        on, oc, oh, ow = [v.value for v in o]
        yd = d.tensor(on, oc, oh, ow, fmt=x_fmt, dtype=dtype)
        xt, wt = dev(torch, x), dev(torch, w)
        yt = dev(torch, y0) if y0 is not None else torch.zeros(
            on * oc * oh * ow, dtype=xt.dtype, device="cuda")
        st = d.L.cudnnConvolutionForward(d.h, fptr(alpha), xd, C.c_void_p(xt.data_ptr()), wdsc,
                                         C.c_void_p(wt.data_ptr()), cv, 0, None, 0, fptr(beta), yd,
                                         C.c_void_p(yt.data_ptr()))
        assert st == 0
        torch.cuda.synchronize()
        return yt.cpu().numpy(), (on, oc, oh, ow)


def test_conv_reference_pin(cuda, built):
    """tests/cudnn_test.cpp:40-107 with the bias folded in through beta = 1."""
    y, _ = run_conv(cuda, np.ones(32, np.float32), np.full(36, 0.5, np.float32), (1, 2, 4, 4),
                    (2, 2, 3, 3), pad=(1, 1), beta=1.0, y0=np.full(32, 1.25, np.float32))
    assert abs(y[0] - 5.25) < 1e-4 and abs(y[5] - 10.25) < 1e-4


CONV_CASES = [
    # xshape, wshape, pad, stride, dil, groups, x_fmt, w_fmt, mode
    ((2, 3, 9, 11), (4, 3, 3, 3), (1, 1), (1, 1), (1, 1), 1, NCHW, NCHW, 1),
    ((2, 8, 10, 7), (6, 8, 3, 3), (1, 1), (1, 1), (1, 1), 1, NHWC, NHWC, 1),
    ((1, 6, 13, 12), (9, 2, 5, 3), (2, 1), (2, 3), (1, 2), 3, NCHW, NCHW, 1),
    ((2, 4, 8, 8), (4, 4, 3, 3), (0, 0), (1, 1), (1, 1), 1, NCHW, NCHW, 0),
    ((3, 16, 12, 12), (32, 16, 1, 1), (0, 0), (2, 2), (1, 1), 1, NHWC, NHWC, 1),
    ((2, 64, 14, 14), (64, 64, 3, 3), (1, 1), (1, 1), (1, 1), 1, NHWC, NHWC, 1),
    ((2, 32, 9, 9), (16, 32, 3, 3), (1, 1), (1, 1), (1, 1), 1, NHWC, NCHW, 1),
]


@pytest.mark.parametrize("case", CONV_CASES)
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (0.5, 2.0)])
def test_conv_f32_matches_oracle(cuda, built, case, alpha, beta):
    xshape, wshape, pad, stride, dil, groups, xf, wf, mode = case
    rng = np.random.default_rng(hash((case, alpha)) & 0xFFFF)
    x = rng.standard_normal(np.prod(xshape)).astype(np.float32)
    w = rng.standard_normal(np.prod(wshape)).astype(np.float32)
    fmt = {NCHW: "NCHW", NHWC: "NHWC"}
    n, c, h, wd = xshape
    k, cg, r, s = wshape
    oh = 1 + (h + 2 * pad[0] - (1 + (r - 1) * dil[0])) // stride[0]
    ow = 1 + (wd + 2 * pad[1] - (1 + (s - 1) * dil[1])) // stride[1]
    y0 = rng.standard_normal(n * k * oh * ow).astype(np.float32)
    got, _ = run_conv(cuda, x, w, xshape, wshape, x_fmt=xf, w_fmt=wf, pad=pad, stride=stride,
                      dil=dil, groups=groups, mode=mode, alpha=alpha, beta=beta, y0=y0)
    want = oracle.conv2d(x, w, xshape, wshape, x_fmt=fmt[xf], w_fmt=fmt[wf], pad=pad,
                         stride=stride, dil=dil, groups=groups,
                         mode="conv" if mode == 0 else "cross", alpha=alpha, beta=beta,
                         y=y0.copy(), accum_f64=True)
    mag = oracle.conv2d(np.abs(x), np.abs(w), xshape, wshape, x_fmt=fmt[xf], w_fmt=fmt[wf],
                        pad=pad, stride=stride, dil=dil, groups=groups,
                        mode="conv" if mode == 0 else "cross", alpha=abs(alpha), beta=abs(beta),
                        y=np.abs(y0), accum_f64=True)
    check_f32(got, want, scale=mag)


@pytest.mark.parametrize("case", CONV_CASES[:2] + CONV_CASES[5:6])
def test_conv_bf16_matches_oracle(cuda, built, case):
    xshape, wshape, pad, stride, dil, groups, xf, wf, mode = case
    rng = np.random.default_rng(7)
    x = oracle.bf16_bits(rng.standard_normal(np.prod(xshape)).astype(np.float32))
    w = oracle.bf16_bits(rng.standard_normal(np.prod(wshape)).astype(np.float32))
    fmt = {NCHW: "NCHW", NHWC: "NHWC"}
    got, _ = run_conv(cuda, x.view(np.int16), w.view(np.int16), xshape, wshape, x_fmt=xf,
                      w_fmt=wf, pad=pad, stride=stride, dil=dil, groups=groups, mode=mode,
                      dtype=BF16)
    want = oracle.conv2d(x, w, xshape, wshape, x_fmt=fmt[xf], w_fmt=fmt[wf], pad=pad,
                         stride=stride, dil=dil, groups=groups)
    g = oracle.bf16_to_f32(got.view(np.uint16))
    wv = oracle.bf16_to_f32(want)
    assert normwise(g, wv) <= 1e-2


TC_CASES = [
    # xshape (n, c, h, w), wshape (k, c, r, s), pad, dil, mode, alpha, beta
    ((2, 64, 14, 14), (64, 64, 3, 3), (1, 1), (1, 1), 1, 1.0, 0.0),
    ((3, 128, 9, 13), (96, 128, 3, 3), (1, 1), (1, 1), 1, 1.0, 0.0),
    ((2, 64, 20, 30), (256, 64, 1, 1), (0, 0), (1, 1), 1, 0.5, 0.0),
    ((1, 192, 17, 17), (300, 192, 3, 3), (0, 2), (2, 1), 1, 1.0, 0.75),
    ((2, 64, 8, 70), (128, 64, 5, 3), (2, 1), (1, 1), 0, 1.0, 0.0),
    ((4, 256, 28, 28), (256, 256, 3, 3), (1, 1), (1, 1), 1, 1.0, 0.0),
]


@pytest.mark.parametrize("case", TC_CASES)
def test_conv_bf16_tensor_core_layout(cuda, built, case):
    """NHWC input/output, KRSC filter, C a multiple of 64: the tcgen05 implicit GEMM."""
    xshape, wshape, pad, dil, mode, alpha, beta = case
    rng = np.random.default_rng(sum(xshape) + sum(wshape))
    x = oracle.bf16_bits((rng.standard_normal(np.prod(xshape)) * 0.5).astype(np.float32))
    w = oracle.bf16_bits((rng.standard_normal(np.prod(wshape)) * 0.5).astype(np.float32))
    n, c, h, wd = xshape
    k, _, r, s = wshape
    oh = 1 + (h + 2 * pad[0] - (1 + (r - 1) * dil[0]))
    ow = 1 + (wd + 2 * pad[1] - (1 + (s - 1) * dil[1]))
    y0 = oracle.bf16_bits(rng.standard_normal(n * k * oh * ow).astype(np.float32))
    got, _ = run_conv(cuda, x.view(np.int16), w.view(np.int16), xshape, wshape, x_fmt=NHWC,
                      w_fmt=NHWC, pad=pad, dil=dil, mode=mode, alpha=alpha, beta=beta,
                      y0=y0.view(np.int16), dtype=BF16)
    want = oracle.conv2d(x, w, xshape, wshape, x_fmt="NHWC", w_fmt="NHWC", pad=pad, dil=dil,
                         mode="conv" if mode == 0 else "cross", alpha=alpha, beta=beta,
                         y=y0.copy())
    g = oracle.bf16_to_f32(got.view(np.uint16)).astype(np.float64)
    wv = oracle.bf16_to_f32(want).astype(np.float64)
    assert normwise(g, wv) <= 1e-2


TC32_CASES = [
    # xshape (n, c, h, w), wshape (k, c, r, s), pad, dil, mode, alpha, beta, filter layout
    ((4, 64, 14, 14), (64, 64, 3, 3), (1, 1), (1, 1), 1, 1.0, 0.0, NHWC),
    ((3, 128, 9, 13), (96, 128, 3, 3), (1, 1), (1, 1), 1, 1.0, 0.0, NCHW),
    ((4, 32, 20, 30), (256, 32, 1, 1), (0, 0), (1, 1), 1, 0.5, 0.0, NHWC),
    ((1, 192, 17, 17), (300, 192, 3, 3), (0, 2), (2, 1), 1, 1.0, 0.75, NCHW),
    ((2, 64, 8, 70), (128, 64, 5, 3), (2, 1), (1, 1), 0, 1.0, 0.0, NHWC),
    ((4, 256, 28, 28), (256, 256, 3, 3), (1, 1), (1, 1), 1, 1.0, 0.0, NHWC),
    ((2, 32, 16, 16), (40, 32, 3, 3), (1, 1), (1, 1), 1, 0.75, 0.5, NHWC),
]


@pytest.mark.parametrize("case", TC32_CASES)
def test_conv_f32_split_tf32_tensor_core(cuda, built, case):
    """fp32 NHWC input/output, KRSC or KCRS filter, C a multiple of 32: the tcgen05
    implicit GEMM in split-tf32 form, held to the fp32 bar (normwise 1e-5, per
    element 2e-5 of conv(|x|, |w|))."""
    xshape, wshape, pad, dil, mode, alpha, beta, wf = case
    rng = np.random.default_rng(sum(xshape) * 3 + sum(wshape))
    x = rng.standard_normal(np.prod(xshape)).astype(np.float32)
    w = rng.standard_normal(np.prod(wshape)).astype(np.float32)
    n, c, h, wd = xshape
    k, _, r, s = wshape
    oh = 1 + (h + 2 * pad[0] - (1 + (r - 1) * dil[0]))
    ow = 1 + (wd + 2 * pad[1] - (1 + (s - 1) * dil[1]))
    y0 = rng.standard_normal(n * k * oh * ow).astype(np.float32)
    got, _ = run_conv(cuda, x, w, xshape, wshape, x_fmt=NHWC, w_fmt=wf, pad=pad, dil=dil,
                      mode=mode, alpha=alpha, beta=beta, y0=y0)
    fmt = {NCHW: "NCHW", NHWC: "NHWC"}
    kw = dict(x_fmt="NHWC", w_fmt=fmt[wf], pad=pad, dil=dil,
              mode="conv" if mode == 0 else "cross", accum_f64=True, threads=16)
    want = oracle.conv2d(x, w, xshape, wshape, alpha=alpha, beta=beta, y=y0.copy(), **kw)
    mag = oracle.conv2d(np.abs(x), np.abs(w), xshape, wshape, alpha=abs(alpha), beta=abs(beta),
                        y=np.abs(y0), **kw)
    check_f32(got, want, scale=mag)


def test_conv_f32_user_workspace_and_repeat(cuda, built):
    """A caller-supplied workSpace large enough for the split planes is used, and two
    calls in a row on one handle (handle workspace reused) give identical output."""
    torch = cuda
    xshape, wshape = (2, 64, 16, 16), (128, 64, 3, 3)
    rng = np.random.default_rng(3)
    x = rng.standard_normal(np.prod(xshape)).astype(np.float32)
    w = rng.standard_normal(np.prod(wshape)).astype(np.float32)
    outs = []
    with Dnn(torch) as d:
        xd = d.tensor(*xshape, fmt=NHWC)
        wdsc = d.filter(*wshape, fmt=NHWC)
        cv = d.conv(pad=(1, 1))
        yd = d.tensor(2, 128, 16, 16, fmt=NHWC)
        xt, wt = dev(torch, x), dev(torch, w)
        ws = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
        for space, size in ((None, 0), (None, 0), (ws.data_ptr(), ws.numel())):
            yt = torch.zeros(2 * 128 * 16 * 16, device="cuda")
            assert d.L.cudnnConvolutionForward(
                d.h, fptr(1.0), xd, C.c_void_p(xt.data_ptr()), wdsc, C.c_void_p(wt.data_ptr()), cv,
                0, C.c_void_p(space) if space else None, size, fptr(0.0), yd,
                C.c_void_p(yt.data_ptr())) == 0
            torch.cuda.synchronize()
            outs.append(yt.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
    want = oracle.conv2d(x, w, xshape, wshape, x_fmt="NHWC", w_fmt="NHWC", pad=(1, 1),
                         accum_f64=True)
    mag = oracle.conv2d(np.abs(x), np.abs(w), xshape, wshape, x_fmt="NHWC", w_fmt="NHWC",
                        pad=(1, 1), accum_f64=True)
    check_f32(outs[0], want, scale=mag)


def test_conv_f32_config_shape_sampled(cuda, built):
    """configs[4] conv through the reference's own fp32 API path: NHWC 64x56x56x256 ->
    256, 3x3, pad 1, KRSC filter; images 0 and 63 checked against the oracle."""
    torch = cuda
    from muda_b200 import synth
    n, c, h, wd, k = 64, 256, 56, 56, 256
    x = synth.normal(torch, n * h * wd * c, seed=11, std=0.02)
    w = synth.normal(torch, k * 9 * c, seed=11, std=0.02, offset=(n * h * wd * c + 3) // 4 * 4)
    xf, wf = x.cpu().numpy(), w.cpu().numpy()
    got, _ = run_conv(torch, xf, wf, (n, c, h, wd), (k, c, 3, 3), x_fmt=NHWC, w_fmt=NHWC,
                      pad=(1, 1))
    per = h * wd * c
    for img in (0, 63):
        xi = xf[img * per:(img + 1) * per]
        kw = dict(x_fmt="NHWC", w_fmt="NHWC", pad=(1, 1), accum_f64=True, threads=16)
        want = oracle.conv2d(xi, wf, (1, c, h, wd), (k, c, 3, 3), **kw)
        mag = oracle.conv2d(np.abs(xi), np.abs(wf), (1, c, h, wd), (k, c, 3, 3), **kw)
        check_f32(got[img * h * wd * k:(img + 1) * h * wd * k], want, scale=mag)


def test_conv_bf16_config_shape_sampled(cuda, built):
    """configs[4] conv: NHWC 64x56x56x256 -> 256, 3x3, pad 1 (bf16 extension path); images
    0 and 63 are checked against the oracle."""
    torch = cuda
    from muda_b200 import synth
    n, c, h, wd, k = 64, 256, 56, 56, 256
    x = synth.normal(torch, n * h * wd * c, seed=11, std=0.02).to(torch.bfloat16)
    w = synth.normal(torch, k * 9 * c, seed=11, std=0.02,
                     offset=(n * h * wd * c + 3) // 4 * 4).to(torch.bfloat16)
    xb = x.view(torch.int16).cpu().numpy()
    wb = w.view(torch.int16).cpu().numpy()
    got, _ = run_conv(torch, xb, wb, (n, c, h, wd), (k, c, 3, 3), x_fmt=NHWC, w_fmt=NHWC,
                      pad=(1, 1), dtype=BF16)
    per = h * wd * c
    for img in (0, 63):
        xi = xb[img * per:(img + 1) * per].view(np.uint16)
        want = oracle.conv2d(xi, wb.view(np.uint16), (1, c, h, wd), (k, c, 3, 3), x_fmt="NHWC",
                             w_fmt="NHWC", pad=(1, 1), threads=16)
        g = oracle.bf16_to_f32(got[img * h * wd * k:(img + 1) * h * wd * k].view(np.uint16))
        assert normwise(g.astype(np.float64), oracle.bf16_to_f32(want).astype(np.float64)) <= 1e-2


# ---------------------------------------------------------------- softmax --
def run_softmax(torch, x, shape, algo, mode, alpha=1.0, beta=0.0, y0=None, fmt=NCHW,
                strides=None):
    n, c, h, w = shape
    with Dnn(torch) as d:
        if strides is None:
            xd = d.tensor(n, c, h, w, fmt=fmt)
            yd = d.tensor(n, c, h, w, fmt=fmt)
        else:
            xd = d.tensor(n, c, h, w, strides=strides)
            yd = d.tensor(n, c, h, w, strides=strides)
        xt = dev(torch, x)
        yt = dev(torch, y0) if y0 is not None else torch.zeros_like(xt)
        assert d.L.cudnnSoftmaxForward(d.h, algo, mode, fptr(alpha), xd, C.c_void_p(xt.data_ptr()),
                                       fptr(beta), yd, C.c_void_p(yt.data_ptr())) == 0
        torch.cuda.synchronize()
        return yt.cpu().numpy()


def test_softmax_reference_pin(cuda, built):
    y = run_softmax(cuda, np.array([1.0, 2.0], np.float32), (1, 2, 1, 1), 1, 1)
    e1, e2 = np.exp(1.0), np.exp(2.0)
    assert abs(y[0] - e1 / (e1 + e2)) < 1e-5 and abs(y[1] - e2 / (e1 + e2)) < 1e-5


@pytest.mark.parametrize("rows,length", [(7, 1), (5, 5), (33, 32), (9, 33), (17, 1000),
                                         (8, 1024), (6, 1025), (40, 4096), (3, 4099),
                                         (5, 8192), (3, 8193), (2, 40000)])
@pytest.mark.parametrize("algo", [0, 1, 2])
def test_softmax_rows(cuda, built, rows, length, algo):
    rng = np.random.default_rng(rows * 7 + length)
    x = (rng.standard_normal(rows * length) * 3).astype(np.float32)
    shape = (rows, length, 1, 1)
    got = run_softmax(cuda, x, shape, algo, 0)
    want = oracle.softmax(x, shape, algo=algo)
    check_f32(got, want)


def test_softmax_alpha_beta(cuda, built):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(16 * 3000).astype(np.float32)
    y0 = rng.standard_normal(16 * 3000).astype(np.float32)
    got = run_softmax(cuda, x, (16, 3000, 1, 1), 1, 0, alpha=0.75, beta=-1.5, y0=y0)
    want = oracle.softmax(x, (16, 3000, 1, 1), algo=1, alpha=0.75, beta=-1.5, y=y0.copy())
    check_f32(got, want)


@pytest.mark.parametrize("algo", [0, 1, 2])
def test_softmax_channel_layouts(cuda, built, algo):
    rng = np.random.default_rng(4)
    n, c, h, w = 3, 37, 5, 6
    x = rng.standard_normal(n * c * h * w).astype(np.float32)
    # NCHW channel mode (strided generic path)
    got = run_softmax(cuda, x, (n, c, h, w), algo, 1)
    want = oracle.softmax(x, (n, c, h, w), algo=algo, channel=True)
    check_f32(got, want)
    # NHWC channel mode (each pixel's channels are contiguous)
    nhwc = (h * w * c, 1, w * c, c)
    got = run_softmax(cuda, x, (n, c, h, w), algo, 1, fmt=NHWC)
    want = oracle.softmax(x, (n, c, h, w), algo=algo, channel=True, x_strides=nhwc)
    check_f32(got, want)
    # INSTANCE mode over a padded (non-packed) layout
    st = (c * h * w + 13, h * w, w, 1)
    xp = rng.standard_normal(n * st[0]).astype(np.float32)
    got = run_softmax(cuda, xp, (n, c, h, w), algo, 0, strides=st)
    want = oracle.softmax(xp, (n, c, h, w), algo=algo, x_strides=st)
    mask = np.zeros(n * st[0], bool)
    for b in range(n):
        mask[b * st[0]: b * st[0] + c * h * w] = True
    check_f32(got[mask], want[mask])


def test_softmax_config_size(cuda, built):
    """Config: 65536 x 4096 fp32, normal(0, 0.02), ACCURATE, INSTANCE, alpha 1, beta 0."""
    torch = cuda
    rows, length = 65536, 4096
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(rows * length, dtype=np.float32) * np.float32(0.02))
    got = run_softmax(torch, x, (rows, length, 1, 1), 1, 0)
    want = oracle.softmax(x, (rows, length, 1, 1), algo=1, threads=16)
    check_f32(got, want)
    # each row sums to 1
    np.testing.assert_allclose(got.reshape(rows, length).astype(np.float64).sum(1), 1.0, rtol=1e-5)
