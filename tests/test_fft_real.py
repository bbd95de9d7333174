"""cufftExecR2C / cufftExecC2R (real-data FFTs).

CPU: the oracle restatement of the reference's R2C / C2R steps against numpy's
float64 rfftn / irfftn (times N: no scaling), and the reference's round-trip known
answer (tests/cufft_test.cpp:76-126).  GPU (marked): both paths of the CUDA
implementation — the half-length packed transform (even last axis, unit-stride
reals) and the general gather/scatter path (odd lengths, strided or misaligned
reals) — against the oracle.  Bar: relative L2 error <= 1e-5 per transform.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import stream_ptr


def rel(got, want):
    return np.linalg.norm(np.asarray(got) - want) / max(np.linalg.norm(want), 1e-30)


@pytest.mark.parametrize("dims", [[16], [15], [6, 10], [4, 3, 8], [5, 7], [1, 8], [2]])
def test_oracle_matches_numpy(dims):
    rng = np.random.default_rng(len(dims) + dims[-1])
    batch = 3
    x = rng.standard_normal(batch * int(np.prod(dims))).astype(np.float32)
    got = oracle.fft_r2c(x, dims, batch).reshape(batch, -1)
    ax = tuple(range(1, len(dims) + 1))
    want = np.fft.rfftn(x.reshape(batch, *dims).astype(np.float64), axes=ax).reshape(batch, -1)
    assert rel(got, want) < 1e-12
    H = dims[-1] // 2 + 1
    X = (rng.standard_normal(got.shape) + 1j * rng.standard_normal(got.shape)).astype(np.complex64)
    y = oracle.fft_c2r(X.reshape(-1), dims, batch).reshape(batch, -1)
    yw = np.fft.irfftn(X.astype(np.complex128).reshape(batch, *dims[:-1], H), s=dims,
                       axes=ax).reshape(batch, -1) * np.prod(dims)
    assert rel(y, yw) < 1e-6


def reference_signal(n=128):
    """tests/cufft_test.cpp:89-94."""
    t = np.arange(n, dtype=np.float32) / np.float32(n)
    return (1.5 + np.sin(2 * np.float32(np.pi) * 4 * t)
            - 0.5 * np.cos(2 * np.float32(np.pi) * 7 * t)).astype(np.float32)


def test_oracle_reference_round_trip_pin():
    x = reference_signal()
    X = oracle.fft_r2c(x, [128], 1)
    y = oracle.fft_c2r(X.astype(np.complex64), [128], 1)
    assert np.all(np.abs(y / 128 - x) < 1e-3)


# --------------------------------------------------------------------- GPU --
class Plan:
    def __init__(self, torch, dims, typ, batch, inembed=None, istride=1, idist=0, onembed=None,
                 ostride=1, odist=0):
        self.L = capi.cufft()
        self.h = C.c_void_p()
        n = (C.c_int * len(dims))(*dims)
        ie = (C.c_int * len(dims))(*inembed) if inembed else None
        oe = (C.c_int * len(dims))(*onembed) if onembed else None
        st = self.L.cufftPlanMany(C.byref(self.h), len(dims), n, ie, istride, idist, oe, ostride,
                                  odist, typ, batch)
        assert st == 0, st
        assert self.L.cufftSetStream(self.h, C.c_void_p(stream_ptr(torch))) == 0

    def close(self):
        assert self.L.cufftDestroy(self.h) == 0


def dev_floats(torch, a, offset=0):
    t = torch.zeros(len(a) + 8, dtype=torch.float32, device="cuda")
    t[offset:offset + len(a)] = torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    return t, C.c_void_p(t.data_ptr() + 4 * offset)


# Rows of half length 16 .. 4096 (powers of two) in whole groups of 4096 / (L/2) rows
# take the fused one-kernel path, the rest of the rows the two-kernel path; 8-byte
# aligned (misalign 2) reals the two-kernel packed path, 4-byte (misalign 1) the
# general gather/scatter path.
CASES = [  # dims, batch
    ([128], 1), ([4096], 7), ([60], 5), ([1000], 3), ([15], 4), ([2], 3), ([16384], 2),
    ([6, 10], 2), ([16, 32], 3), ([4, 3, 8], 2), ([8, 8, 8], 1), ([7, 9], 2), ([1, 64], 2),
    ([32], 300), ([64], 200), ([8192], 5), ([512], 40), ([64, 256], 2), ([4, 8, 512], 3),
    ([10000], 2), ([5001], 2)]


@pytest.mark.gpu
@pytest.mark.parametrize("dims,batch", CASES)
@pytest.mark.parametrize("misalign", [0, 1, 2])
def test_gpu_r2c_and_c2r_match_oracle(cuda, built, dims, batch, misalign):
    torch = cuda
    rng = np.random.default_rng(int(np.prod(dims)) + batch)
    epb = int(np.prod(dims))
    H = dims[-1] // 2 + 1
    hpb = epb // dims[-1] * H
    x = rng.standard_normal(batch * epb).astype(np.float32)
    # R2C
    p = Plan(torch, dims, capi.CUFFT_R2C, batch)
    tx, px = dev_floats(torch, x, misalign)
    out = torch.zeros(batch * hpb, dtype=torch.complex64, device="cuda")
    assert p.L.cufftExecR2C(p.h, px, C.c_void_p(out.data_ptr())) == 0
    torch.cuda.synchronize()
    p.close()
    got = out.cpu().numpy().reshape(batch, -1)
    want = oracle.fft_r2c(x, dims, batch).reshape(batch, -1)
    for b in range(batch):
        assert rel(got[b], want[b]) <= 1e-5
    # C2R from an arbitrary half spectrum (non-real first / middle entries included)
    X = (rng.standard_normal(batch * hpb) + 1j * rng.standard_normal(batch * hpb)).astype(np.complex64)
    p = Plan(torch, dims, capi.CUFFT_C2R, batch)
    # misalign 2 also moves the half spectrum by one complex value (8-byte aligned)
    xoff = 1 if misalign == 2 else 0
    tXb = torch.zeros(batch * hpb + 1, dtype=torch.complex64, device="cuda")
    tXb[xoff:xoff + batch * hpb] = torch.from_numpy(X).cuda()
    X_before = tXb.clone()
    ty = torch.zeros(batch * epb + 8, dtype=torch.float32, device="cuda")
    py = C.c_void_p(ty.data_ptr() + 4 * misalign)
    assert p.L.cufftExecC2R(p.h, C.c_void_p(tXb.data_ptr() + 8 * xoff), py) == 0
    torch.cuda.synchronize()
    p.close()
    assert torch.equal(tXb, X_before)  # the input is left as it was
    got = ty.cpu().numpy()[misalign:misalign + batch * epb].reshape(batch, -1)
    want = oracle.fft_c2r(X, dims, batch).reshape(batch, -1)
    for b in range(batch):
        assert rel(got[b], want[b]) <= 1e-5


@pytest.mark.gpu
def test_gpu_reference_round_trip_pin(cuda, built):
    """cufft_test.cpp:76-126 on the GPU: R2C then C2R of N = 128, divided by N."""
    torch = cuda
    x = reference_signal()
    tx, px = dev_floats(torch, x)
    X = torch.zeros(65, dtype=torch.complex64, device="cuda")
    y = torch.zeros(128, dtype=torch.float32, device="cuda")
    L = capi.cufft()
    a, b = C.c_void_p(), C.c_void_p()
    assert L.cufftPlan1d(C.byref(a), 128, capi.CUFFT_R2C, 1) == 0
    assert L.cufftPlan1d(C.byref(b), 128, capi.CUFFT_C2R, 1) == 0
    assert L.cufftExecR2C(a, px, C.c_void_p(X.data_ptr())) == 0
    assert L.cufftExecC2R(b, C.c_void_p(X.data_ptr()), C.c_void_p(y.data_ptr())) == 0
    torch.cuda.synchronize()
    assert L.cufftDestroy(a) == 0 and L.cufftDestroy(b) == 0
    assert np.all(np.abs(y.cpu().numpy() / 128 - x) < 1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("L,batch", [(256, 3), (60, 4), (33, 2)])
def test_gpu_strided_and_in_place_layouts(cuda, built, L, batch):
    """Strided reals (istride 2) take the general path; the in-place padded layout
    (row pitch 2 * (L/2 + 1) reals, the usual cuFFT in-place R2C layout) works."""
    torch = cuda
    rng = np.random.default_rng(L)
    H = L // 2 + 1
    # strided: element t of batch b at b*idist + t*2
    idist = 2 * L + 6
    xs = rng.standard_normal(batch * idist).astype(np.float32)
    p = Plan(torch, [L], capi.CUFFT_R2C, batch, inembed=[L], istride=2, idist=idist,
             onembed=[H], ostride=1, odist=H)
    tx, px = dev_floats(torch, xs)
    out = torch.zeros(batch * H, dtype=torch.complex64, device="cuda")
    assert p.L.cufftExecR2C(p.h, px, C.c_void_p(out.data_ptr())) == 0
    torch.cuda.synchronize()
    p.close()
    want = oracle.fft_r2c(xs, [L], batch, istride=2, idist=idist).reshape(batch, -1)
    got = out.cpu().numpy().reshape(batch, -1)
    for b in range(batch):
        assert rel(got[b], want[b]) <= 1e-5
    # in place: reals with pitch 2H, complex output with pitch H over the same memory
    pitch = 2 * H
    xi = np.zeros(batch * pitch, np.float32)
    for b in range(batch):
        xi[b * pitch:b * pitch + L] = rng.standard_normal(L)
    p = Plan(torch, [L], capi.CUFFT_R2C, batch, inembed=[pitch], istride=1, idist=pitch,
             onembed=[H], ostride=1, odist=H)
    buf = torch.from_numpy(xi).cuda()
    assert p.L.cufftExecR2C(p.h, C.c_void_p(buf.data_ptr()), C.c_void_p(buf.data_ptr())) == 0
    torch.cuda.synchronize()
    p.close()
    got = buf.cpu().numpy().view(np.complex64).reshape(batch, -1)
    want = oracle.fft_r2c(xi, [L], batch, idist=pitch).reshape(batch, -1)
    for b in range(batch):
        assert rel(got[b], want[b]) <= 1e-5


@pytest.mark.gpu
def test_gpu_real_plan_errors(cuda, built):
    torch = cuda
    L = capi.cufft()
    h = C.c_void_p()
    assert L.cufftPlan1d(C.byref(h), 64, capi.CUFFT_R2C, 1) == 0
    buf = torch.zeros(256, dtype=torch.float32, device="cuda")
    p = C.c_void_p(buf.data_ptr())
    assert L.cufftExecC2R(h, p, p) == capi.CUFFT_INVALID_TYPE
    assert L.cufftExecC2C(h, p, p, -1) == capi.CUFFT_INVALID_TYPE
    assert L.cufftExecR2C(h, None, p) == capi.CUFFT_INVALID_VALUE
    assert L.cufftDestroy(h) == 0
    assert L.cufftExecR2C(h, p, p) == capi.CUFFT_INVALID_PLAN


@pytest.mark.gpu
@pytest.mark.parametrize("L,batch", [(4096, 65536), (8192, 4099), (32, 1 << 20)])
def test_gpu_round_trip_at_bench_size(cuda, built, L, batch):
    """At the bench's size (and the largest / smallest fused lengths) a C2R of the R2C,
    divided by L, returns the input (size-independent property; max error 1e-5 of
    the signal's scale), and sampled rows match the oracle."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(L)
    x = torch.randn(L * batch, device="cuda", generator=g)
    H = L // 2 + 1
    X = torch.empty(batch * H, dtype=torch.complex64, device="cuda")
    y = torch.empty_like(x)
    lib = capi.cufft()
    a, b = C.c_void_p(), C.c_void_p()
    assert lib.cufftPlan1d(C.byref(a), L, capi.CUFFT_R2C, batch) == 0
    assert lib.cufftPlan1d(C.byref(b), L, capi.CUFFT_C2R, batch) == 0
    assert lib.cufftExecR2C(a, C.c_void_p(x.data_ptr()), C.c_void_p(X.data_ptr())) == 0
    assert lib.cufftExecC2R(b, C.c_void_p(X.data_ptr()), C.c_void_p(y.data_ptr())) == 0
    torch.cuda.synchronize()
    assert lib.cufftDestroy(a) == 0 and lib.cufftDestroy(b) == 0
    err = (y / L - x).abs().max().item()
    assert err < 1e-5 * max(1.0, x.abs().max().item())
    rows = [0, 1, batch // 2, batch - 1]
    xs = x.view(batch, L)[rows].cpu().numpy().reshape(-1)
    want = oracle.fft_r2c(xs, [L], len(rows)).reshape(len(rows), -1)
    got = X.view(batch, H)[rows].cpu().numpy()
    for r in range(len(rows)):
        assert rel(got[r], want[r]) <= 1e-5
