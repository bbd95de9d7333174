"""cufftPlanMany / cufftExecC2C.

CPU: the oracle against the reference's known answers, and the C-ABI plan logic.
GPU (marked): the CUDA path through the C ABI against the double-precision
oracle; bar: relative L2 error <= 1e-5 per transform.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import stream_ptr

TOL = 1e-5


def ref_signal(n):
    """tests/cufft_test.cpp:41-46."""
    i = np.arange(n, dtype=np.float32)
    phase = np.float32(2.0 * np.pi) * i / np.float32(n)
    return (np.cos(3 * phase) + 0.5 * np.sin(phase) + 1j * 0.25 * np.cos(2 * phase)).astype(
        np.complex64)


@pytest.mark.parametrize("n", [256, 60])
def test_oracle_round_trip_pin(n):
    """tests/cufft_test.cpp:34-74: forward then inverse, divided by N, recovers the input
    (tolerance 1e-3)."""
    x = ref_signal(n)
    y = oracle.fft_c2c(oracle.fft_c2c(x, [n], 1, -1), [n], 1, 1) / n
    assert np.max(np.abs(y.real - x.real)) < 1e-3 and np.max(np.abs(y.imag - x.imag)) < 1e-3


def test_oracle_plan_many_impulse_pin():
    """tests/cufft_test.cpp:195-238: N = 64, batch 4, impulse of amplitude b+1 -> flat spectrum."""
    x = np.zeros(64 * 4, np.complex64)
    for b in range(4):
        x[b * 64] = b + 1
    y = oracle.fft_c2c(x, [64], 4, -1)
    for b in range(4):
        np.testing.assert_allclose(y[b * 64:(b + 1) * 64].real, b + 1, atol=1e-4)


def test_oracle_2d_impulse_pin():
    """tests/cufft_test.cpp:127-153: 16 x 32 impulse -> all-ones spectrum."""
    x = np.zeros(16 * 32, np.complex64)
    x[0] = 1
    y = oracle.fft_c2c(x, [16, 32], 1, -1)
    np.testing.assert_allclose(y.real, 1.0, atol=1e-4)
    np.testing.assert_allclose(y.imag, 0.0, atol=1e-4)


def test_oracle_matches_numpy():
    rng = np.random.default_rng(0)
    for dims, b in (([4096], 2), ([60], 3), ([8, 12], 2)):
        n = int(np.prod(dims))
        x = (rng.standard_normal(n * b) + 1j * rng.standard_normal(n * b)).astype(np.complex64)
        want = np.fft.fftn(x.reshape([b] + dims).astype(np.complex128),
                           axes=tuple(range(1, len(dims) + 1))).reshape(-1)
        got = oracle.fft_c2c(x, dims, b, -1, exact=True)
        assert np.linalg.norm(got - want) <= 1e-12 * np.linalg.norm(want)


def _plan_many(L, dims, batch, inembed=None, istride=1, idist=0, onembed=None, ostride=1,
               odist=0, typ=capi.CUFFT_C2C):
    p = C.c_void_p()
    n = (C.c_int * len(dims))(*dims)
    ie = (C.c_int * len(dims))(*inembed) if inembed else None
    oe = (C.c_int * len(dims))(*onembed) if onembed else None
    st = L.cufftPlanMany(C.byref(p), len(dims), n, ie, istride, idist, oe, ostride, odist, typ,
                         batch)
    return st, p


def test_plan_argument_errors(built):
    """Checks made before any device resource is touched (cufft_plan.mm:36-60)."""
    L = capi.cufft()
    assert _plan_many(L, [64], 0)[0] == capi.CUFFT_INVALID_VALUE
    assert _plan_many(L, [0], 1)[0] == capi.CUFFT_INVALID_SIZE
    assert _plan_many(L, [4, 4, 4, 4], 1)[0] == capi.CUFFT_INVALID_VALUE
    assert _plan_many(L, [64], 1, typ=capi.CUFFT_Z2Z)[0] == capi.CUFFT_NOT_SUPPORTED
    assert _plan_many(L, [64], 1, typ=0x33)[0] == capi.CUFFT_INVALID_TYPE
    assert L.cufftPlan1d(None, 64, capi.CUFFT_C2C, 1) == capi.CUFFT_INVALID_VALUE
    q = C.c_void_p()
    assert L.cufftCreate(C.byref(q)) == 0
    ws = C.c_size_t(0)
    assert L.cufftGetSize(q, C.byref(ws)) == capi.CUFFT_INVALID_PLAN  # not configured
    assert L.cufftExecC2C(q, C.c_void_p(256), C.c_void_p(256), -1) == capi.CUFFT_INVALID_PLAN
    assert L.cufftDestroy(q) == 0
    assert L.cufftDestroy(q) == capi.CUFFT_INVALID_PLAN
    assert L.cufftSetStream(q, None) == capi.CUFFT_INVALID_PLAN


@pytest.mark.gpu
def test_plan_logic(cuda, built):
    L = capi.cufft()
    st, p = _plan_many(L, [64], 4)
    assert st == 0
    ws = C.c_size_t(0)
    assert L.cufftGetSize(p, C.byref(ws)) == 0 and ws.value > 0
    assert L.cufftSetStream(p, None) == 0
    assert L.cufftExecC2C(p, None, None, -1) == capi.CUFFT_INVALID_VALUE
    assert L.cufftExecC2C(p, C.c_void_p(256), C.c_void_p(256), 0) == capi.CUFFT_INVALID_VALUE
    # unaddressable buffers are rejected before launch
    assert L.cufftExecC2C(p, C.c_void_p(256), C.c_void_p(256), -1) == capi.CUFFT_INVALID_VALUE
    assert L.cufftDestroy(p) == 0
    assert L.cufftDestroy(p) == capi.CUFFT_INVALID_PLAN
    assert L.cufftExecC2C(p, C.c_void_p(256), C.c_void_p(256), -1) == capi.CUFFT_INVALID_PLAN
    assert _plan_many(L, [64], 0)[0] == capi.CUFFT_INVALID_VALUE
    assert _plan_many(L, [0], 1)[0] == capi.CUFFT_INVALID_SIZE
    assert _plan_many(L, [4, 4, 4, 4], 1)[0] == capi.CUFFT_INVALID_VALUE
    assert _plan_many(L, [64], 1, typ=capi.CUFFT_Z2Z)[0] == capi.CUFFT_NOT_SUPPORTED
    assert _plan_many(L, [64], 1, typ=0x33)[0] == capi.CUFFT_INVALID_TYPE
    # an unconfigured plan has no size
    q = C.c_void_p()
    assert L.cufftCreate(C.byref(q)) == 0
    assert L.cufftGetSize(q, C.byref(ws)) == capi.CUFFT_INVALID_PLAN
    assert L.cufftMakePlan1d(q, 4096, capi.CUFFT_C2C, 8, C.byref(ws)) == 0 and ws.value > 0
    assert L.cufftDestroy(q) == 0


# --------------------------------------------------------------------- GPU --
def gpu_fft(torch, x, dims, batch, sign, *, inembed=None, istride=1, idist=0, onembed=None,
            ostride=1, odist=0, out_len=None, inplace=False):
    L = capi.cufft()
    st, p = _plan_many(L, dims, batch, inembed, istride, idist, onembed, ostride, odist)
    assert st == 0, st
    try:
        assert L.cufftSetStream(p, C.c_void_p(stream_ptr(torch))) == 0
        xi = torch.from_numpy(np.ascontiguousarray(x).view(np.float32)).cuda()
        if inplace:
            xo = xi
        else:
            xo = torch.zeros(2 * (out_len or len(x)), dtype=torch.float32, device="cuda")
        assert L.cufftExecC2C(p, C.c_void_p(xi.data_ptr()), C.c_void_p(xo.data_ptr()), sign) == 0
        torch.cuda.synchronize()
        return xo.cpu().numpy().view(np.complex64)
    finally:
        assert L.cufftDestroy(p) == 0


def rel_l2_per_transform(got, want, n, batch, dist=None, stride=1):
    dist = n * stride if dist is None else dist
    worst = 0.0
    for b in range(batch):
        idx = b * dist + np.arange(n) * stride
        g, w = got[idx].astype(np.complex128), want[idx]
        worst = max(worst, np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-300))
    return worst


def rand_c64(rng, n):
    return (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384])
@pytest.mark.parametrize("sign", [-1, 1])
def test_gpu_pow2_lengths(cuda, built, n, sign):
    rng = np.random.default_rng(n)
    batch = max(1, min(64, (1 << 16) // n)) + 1
    x = rand_c64(rng, n * batch)
    got = gpu_fft(cuda, x, [n], batch, sign)
    want = oracle.fft_c2c(x, [n], batch, sign, exact=True)
    assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n", [3, 5, 7, 12, 60, 100, 1000, 3000])
def test_gpu_non_pow2_lengths(cuda, built, n):
    rng = np.random.default_rng(n)
    batch = 3
    x = rand_c64(rng, n * batch)
    for sign in (-1, 1):
        got = gpu_fft(cuda, x, [n], batch, sign)
        want = oracle.fft_c2c(x, [n], batch, sign, exact=True)
        assert rel_l2_per_transform(got, want, n, batch) <= TOL


# Lengths that are not powers of two: below 32 the direct DFT; 7-smooth lengths up to
# 12288 the mixed-radix kernel; other lengths 32 .. 4096 the fused Bluestein kernel
# (inner lengths 64 .. 8192), above that Bluestein through global memory.
BLUESTEIN = [31, 33, 47, 97, 127, 255, 257, 1023, 2047, 2049, 4095, 4097]
# 7-smooth lengths: each radix family alone (3^5, 5^4, 7^4), with a power of two, with
# several transforms per CTA, and the largest one shared memory holds (12288); 12500
# is 7-smooth but above that bound, so it runs through global Bluestein.
MIXED = [36, 48, 96, 243, 343, 625, 1000, 1536, 2401, 3000, 3125, 6000, 6144, 10000,
         12000, 12288, 12500]


@pytest.mark.gpu
@pytest.mark.parametrize("n", MIXED)
def test_gpu_mixed_radix_lengths(cuda, built, n):
    """Mixed-radix Stockham (radices 16, 8, 4, 2, 3, 5, 7) against numpy's float64 FFT,
    both directions, with batches that leave a partial last CTA."""
    rng = np.random.default_rng(n + 3)
    batch = max(2, min(40, (1 << 16) // n)) + 1
    x = rand_c64(rng, n * batch)
    xd = x.reshape(batch, n).astype(np.complex128)
    for sign in (-1, 1):
        got = gpu_fft(cuda, x, [n], batch, sign)
        want = (np.fft.fft(xd, axis=1) if sign < 0 else np.fft.ifft(xd, axis=1) * n).reshape(-1)
        assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n", [4097, 8191, 10007, 100003, (1 << 20) - 1])
def test_gpu_bluestein_global_lengths(cuda, built, n):
    """Global-memory Bluestein (inner lengths 16384 .. 2^21, the longer ones through the
    two-pass split) against numpy's float64 FFT, both directions."""
    rng = np.random.default_rng(n)
    batch = max(2, (1 << 21) // n)
    x = rand_c64(rng, n * batch)
    xd = x.reshape(batch, n).astype(np.complex128)
    for sign in (-1, 1):
        got = gpu_fft(cuda, x, [n], batch, sign)
        want = (np.fft.fft(xd, axis=1) if sign < 0 else np.fft.ifft(xd, axis=1) * n).reshape(-1)
        assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n,batch", [((1 << 20) + 7, 2), (3 * (1 << 21) + 1, 1)])
def test_gpu_bluestein_long_lengths(cuda, built, n, batch):
    """Lengths above 2^20 (the reference transforms any length): Bluestein through global
    memory with chirp, inner twiddles and bhat built on the device, inner lengths 2^22 ..
    2^27 through the two-pass split; against numpy's float64 FFT, both directions."""
    rng = np.random.default_rng(n)
    x = rand_c64(rng, n * batch)
    xd = x.reshape(batch, n).astype(np.complex128)
    for sign in (-1, 1):
        got = gpu_fft(cuda, x, [n], batch, sign)
        want = (np.fft.fft(xd, axis=1) if sign < 0 else np.fft.ifft(xd, axis=1) * n).reshape(-1)
        assert rel_l2_per_transform(got, want, n, batch) <= TOL, (n, sign)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [(1 << 25) + 1, (1 << 27) - 1])
def test_gpu_bluestein_longest_length(cuda, built, n):
    """Long non-power-of-two lengths up to the longest served, 2^27 - 1 (inner length
    2^28): the forward transform at three frequencies against float64 sums, and the
    round trip (numpy's own FFT of these lengths takes minutes on the host)."""
    rng = np.random.default_rng(5)
    x = rand_c64(rng, n)
    got = gpu_fft(cuda, x, [n], 1, -1)
    xd = x.astype(np.complex128)
    idx = np.arange(n, dtype=np.float64)
    for k in (1, n // 2, n - 1):
        w = np.exp(-2j * np.pi * ((idx * k) % n) / n)
        want = np.dot(xd, w)
        scale = np.sqrt(n) * np.sqrt(np.mean(np.abs(xd) ** 2))
        assert abs(got[k] - want) <= 1e-5 * scale, (k, abs(got[k] - want) / scale)
    back = gpu_fft(cuda, got, [n], 1, 1) / n
    assert rel_l2_per_transform(back, x, n, 1) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n", BLUESTEIN)
def test_gpu_bluestein_lengths(cuda, built, n):
    """Batches that fill several transforms per CTA plus a partial last CTA, both
    directions, against the double-precision oracle."""
    rng = np.random.default_rng(n + 1)
    batch = max(2, min(40, (1 << 15) // n)) + 1
    x = rand_c64(rng, n * batch)
    for sign in (-1, 1):
        got = gpu_fft(cuda, x, [n], batch, sign)
        want = oracle.fft_c2c(x, [n], batch, sign, exact=True)
        assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n", [60, 1000, 97, 2049])
def test_gpu_non_pow2_in_place_and_strided(cuda, built, n):
    rng = np.random.default_rng(n + 2)
    batch = 6
    x = rand_c64(rng, n * batch)
    got = gpu_fft(cuda, x, [n], batch, -1, inplace=True)
    want = oracle.fft_c2c(x, [n], batch, -1, exact=True)
    assert rel_l2_per_transform(got, want, n, batch) <= TOL
    istride, idist, ostride, odist = 2, 2 * n + 3, 3, 3 * n + 1
    x = rand_c64(rng, (batch - 1) * idist + (n - 1) * istride + 1)
    out_len = (batch - 1) * odist + (n - 1) * ostride + 1
    got = gpu_fft(cuda, x, [n], batch, 1, inembed=[n], istride=istride, idist=idist,
                  onembed=[n], ostride=ostride, odist=odist, out_len=out_len)
    want = oracle.fft_c2c(x, [n], batch, 1, istride=istride, idist=idist, ostride=ostride,
                          odist=odist, out_len=out_len, exact=True)
    assert rel_l2_per_transform(got, want, n, batch, odist, ostride) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("dims", [[100, 60], [33, 5, 40], [48, 1000], [3, 5000]])
def test_gpu_bluestein_multi_dim(cuda, built, dims):
    rng = np.random.default_rng(sum(dims))
    n, batch = int(np.prod(dims)), 2
    x = rand_c64(rng, n * batch)
    for sign in (-1, 1):
        got = gpu_fft(cuda, x, dims, batch, sign)
        want = oracle.fft_c2c(x, dims, batch, sign, exact=True)
        assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n", [32768, 1 << 20])
def test_gpu_large_pow2_split(cuda, built, n):
    rng = np.random.default_rng(5)
    batch = 2
    x = rand_c64(rng, n * batch)
    got = gpu_fft(cuda, x, [n], batch, -1)
    want = np.fft.fft(x.reshape(batch, n).astype(np.complex128), axis=1).reshape(-1)
    assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
def test_gpu_reference_round_trip_in_place(cuda, built):
    """tests/cufft_test.cpp:34-74 on the GPU, in place (idata == odata)."""
    for n in (256, 60):
        x = ref_signal(n)
        L = capi.cufft()
        p = C.c_void_p()
        assert L.cufftPlan1d(C.byref(p), n, capi.CUFFT_C2C, 1) == 0
        t = cuda.from_numpy(x.view(np.float32).copy()).cuda()
        ptr = C.c_void_p(t.data_ptr())
        assert L.cufftSetStream(p, C.c_void_p(stream_ptr(cuda))) == 0
        assert L.cufftExecC2C(p, ptr, ptr, capi.CUFFT_FORWARD) == 0
        assert L.cufftExecC2C(p, ptr, ptr, capi.CUFFT_INVERSE) == 0
        cuda.cuda.synchronize()
        y = t.cpu().numpy().view(np.complex64) / n
        assert L.cufftDestroy(p) == 0
        assert np.max(np.abs(y - x)) < 1e-3


@pytest.mark.gpu
def test_gpu_plan_many_impulse(cuda, built):
    x = np.zeros(64 * 4, np.complex64)
    for b in range(4):
        x[b * 64] = b + 1
    y = gpu_fft(cuda, x, [64], 4, -1, inplace=True)
    for b in range(4):
        np.testing.assert_allclose(y[b * 64:(b + 1) * 64].real, b + 1, atol=1e-4)


@pytest.mark.gpu
def test_gpu_strided_layouts(cuda, built):
    rng = np.random.default_rng(9)
    n, batch = 1024, 5
    istride, idist, ostride, odist = 3, 3 * 1024 + 7, 2, 2 * 1024 + 1
    x = rand_c64(rng, (batch - 1) * idist + (n - 1) * istride + 1)
    out_len = (batch - 1) * odist + (n - 1) * ostride + 1
    got = gpu_fft(cuda, x, [n], batch, -1, inembed=[n], istride=istride, idist=idist,
                  onembed=[n], ostride=ostride, odist=odist, out_len=out_len)
    want = oracle.fft_c2c(x, [n], batch, -1, istride=istride, idist=idist, ostride=ostride,
                          odist=odist, out_len=out_len, exact=True)
    assert rel_l2_per_transform(got, want, n, batch, odist, ostride) <= TOL
    # NULL inembed: the strides are ignored (cufft_plan.mm:68-83)
    x2 = rand_c64(rng, n * batch)
    got = gpu_fft(cuda, x2, [n], batch, -1, istride=5, idist=3, ostride=7, odist=2)
    want = oracle.fft_c2c(x2, [n], batch, -1, exact=True)
    assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("dims", [[16, 32], [4, 6, 8], [64, 64], [3, 1, 128], [1, 256]])
def test_gpu_multi_dim(cuda, built, dims):
    rng = np.random.default_rng(len(dims))
    n, batch = int(np.prod(dims)), 3
    x = rand_c64(rng, n * batch)
    for sign in (-1, 1):
        got = gpu_fft(cuda, x, dims, batch, sign)
        want = oracle.fft_c2c(x, dims, batch, sign, exact=True)
        assert rel_l2_per_transform(got, want, n, batch) <= TOL


@pytest.mark.gpu
def test_gpu_config_size(cuda, built):
    """N = 4096, batch 65536, normal(0,1) re/im (seed 3), forward then inverse
    in place.  64 sampled transforms are checked against the oracle after each
    direction; the whole batch satisfies the round trip ifft(fft(x)) / N = x."""
    torch = cuda
    from muda_b200 import synth
    n, batch = 4096, 65536
    x = synth.normal(torch, 2 * n * batch, seed=3)
    x0 = x.clone()
    L = capi.cufft()
    p = C.c_void_p()
    nn = (C.c_int * 1)(n)
    assert L.cufftPlanMany(C.byref(p), 1, nn, None, 1, n, None, 1, n, capi.CUFFT_C2C, batch) == 0
    assert L.cufftSetStream(p, C.c_void_p(stream_ptr(torch))) == 0
    ptr = C.c_void_p(x.data_ptr())
    rng = np.random.default_rng(0)
    pick = np.sort(rng.choice(batch, 64, replace=False))
    src = x0.view(batch, 2 * n)[torch.from_numpy(pick).cuda()].cpu().numpy().view(np.complex64)
    assert L.cufftExecC2C(p, ptr, ptr, capi.CUFFT_FORWARD) == 0
    torch.cuda.synchronize()
    fwd = x.view(batch, 2 * n)[torch.from_numpy(pick).cuda()].cpu().numpy().view(np.complex64)
    want = oracle.fft_c2c(src.reshape(-1), [n], 64, -1, exact=True)
    assert rel_l2_per_transform(fwd.reshape(-1), want, n, 64) <= TOL
    assert L.cufftExecC2C(p, ptr, ptr, capi.CUFFT_INVERSE) == 0
    torch.cuda.synchronize()
    assert L.cufftDestroy(p) == 0
    err = (x.view(batch, 2 * n) / n - x0.view(batch, 2 * n)).double().norm(dim=1)
    ref = x0.view(batch, 2 * n).double().norm(dim=1)
    assert float((err / ref).max()) <= TOL


@pytest.mark.gpu
def test_gpu_plan2d_plan3d_reference_pins(cuda, built):
    """tests/cufft_test.cpp:128-193 through cufftPlan2d / cufftPlan3d: a 16 x 32
    impulse gives a flat spectrum (1e-4), and the 8 x 8 x 8 forward + inverse round
    trip divided by 512 returns the input (1e-3); cufftMakePlan2d / 3d configure
    the same plans on a created handle."""
    torch = cuda
    L = capi.cufft()
    p = C.c_void_p()
    assert L.cufftPlan2d(C.byref(p), 16, 32, capi.CUFFT_C2C) == 0
    x = torch.zeros(2 * 16 * 32, dtype=torch.float32, device="cuda")
    x[0] = 1.0
    ptr = C.c_void_p(x.data_ptr())
    assert L.cufftExecC2C(p, ptr, ptr, capi.CUFFT_FORWARD) == 0
    torch.cuda.synchronize()
    y = x.cpu().numpy().view(np.complex64)
    assert np.all(np.abs(y.real - 1.0) <= 1e-4) and np.all(np.abs(y.imag) <= 1e-4)
    assert L.cufftDestroy(p) == 0

    i = np.arange(512)
    h = (((i % 7) - 3) * np.float32(0.2) + 1j * ((i % 5) - 2) * np.float32(0.1)).astype(np.complex64)
    for make in (False, True):
        q = C.c_void_p()
        if make:
            ws = C.c_size_t(0)
            assert L.cufftCreate(C.byref(q)) == 0
            assert L.cufftMakePlan3d(q, 8, 8, 8, capi.CUFFT_C2C, C.byref(ws)) == 0
            assert ws.value > 0
        else:
            assert L.cufftPlan3d(C.byref(q), 8, 8, 8, capi.CUFFT_C2C) == 0
        t = torch.from_numpy(h.view(np.float32).copy()).cuda()
        tp = C.c_void_p(t.data_ptr())
        assert L.cufftExecC2C(q, tp, tp, capi.CUFFT_FORWARD) == 0
        assert L.cufftExecC2C(q, tp, tp, capi.CUFFT_INVERSE) == 0
        torch.cuda.synchronize()
        out = t.cpu().numpy().view(np.complex64) / 512
        assert np.all(np.abs(out.real - h.real) < 1e-3) and np.all(np.abs(out.imag - h.imag) < 1e-3)
        assert L.cufftDestroy(q) == 0
    # 2-D real plans through the same entry points
    r = C.c_void_p()
    ws = C.c_size_t(0)
    assert L.cufftCreate(C.byref(r)) == 0
    assert L.cufftMakePlan2d(r, 6, 10, capi.CUFFT_R2C, C.byref(ws)) == 0
    xr = np.random.default_rng(3).standard_normal(60).astype(np.float32)
    tx = torch.from_numpy(xr).cuda()
    X = torch.zeros(6 * 6, dtype=torch.complex64, device="cuda")
    assert L.cufftExecR2C(r, C.c_void_p(tx.data_ptr()), C.c_void_p(X.data_ptr())) == 0
    torch.cuda.synchronize()
    want = np.fft.rfftn(xr.reshape(6, 10).astype(np.float64)).reshape(-1)
    got = X.cpu().numpy()
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= TOL
    assert L.cufftDestroy(r) == 0
