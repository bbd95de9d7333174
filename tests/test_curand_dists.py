"""cuRAND log-normal, double-precision and Poisson streams, quasi-generator settings.

CPU: the oracle restatements (curand_context.mm:115-293, curand_kernels.metal:173-264)
have the right moments; the reference's own host and device Poisson definitions
differ (counter word 1 vs 2, double vs float), which is the mismatch this library
resolves by giving both of its generator kinds the device definition; the
argument checks of the new entry points.
GPU (marked):
  - UniformDouble and Poisson (lambda < 30) are bit-identical to the oracle, on
    device and host generators, across calls (offset rules);
  - NormalDouble / LogNormalDouble within 1e-13 relative of the host-libm oracle;
  - LogNormal (fp32) within 2e-6 * max(1, |ln x|) + 3e-7 relative of exp of the
    reference normal formula;
  - Poisson for lambda >= 30 (fp32 Gaussian approximation, where device and host
    transcendentals may round differently): >= 99.99 % identical, the rest off by 1.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import curand_generator


@pytest.mark.parametrize("lam", [0.5, 4.5, 29.5, 30.0, 250.0])
def test_oracle_poisson_moments(lam):
    n = 200_000
    for ref in (False, True):
        x, nxt = oracle.generate_poisson(11, 0, n, lam, reference_host=ref)
        assert nxt == n
        tol = 6 * np.sqrt(lam / n) + 1e-3
        assert abs(x.mean() - lam) < tol
        assert abs(x.var() / lam - 1) < 0.03


def test_reference_host_and_device_poisson_differ():
    """The mismatch the library resolves: for lambda < 30 beyond the first block's
    four uniforms, the reference host path reads counter i + 2^32 while its device
    kernel reads (i, 0, 1, 0), so the two generator kinds give different streams."""
    a, _ = oracle.generate_poisson(5, 0, 4096, 12.0)
    b, _ = oracle.generate_poisson(5, 0, 4096, 12.0, reference_host=True)
    assert np.mean(a != b) > 0.2


def test_oracle_double_and_lognormal_streams():
    u, nxt = oracle.generate_double(1234, 6, 10001)
    assert nxt == 6 + 10002 and u.min() > 0 and u.max() <= 1
    z, _ = oracle.generate_double(1234, 0, 200_001, "normal", 1.5, 2.0)
    assert abs(z.mean() - 1.5) < 0.03 and abs(z.std() - 2.0) < 0.03
    ln, _ = oracle.generate_double(1234, 0, 1001, "lognormal", 0.25, 0.5)
    zz, _ = oracle.generate_double(1234, 0, 1001, "normal", 0.25, 0.5)
    np.testing.assert_allclose(ln, np.exp(zz), rtol=1e-15)
    lf, nxt = oracle.generate_lognormal(9, 0, 4001, 0.0, 0.5)
    assert nxt == 4004
    zf, _ = oracle.generate_normal(9, 0, 4001, 0.0, 0.5)
    np.testing.assert_allclose(lf, np.exp(zf.astype(np.float64)), rtol=2e-7)


def test_api_checks(built):
    L = capi.curand()
    g = C.c_void_p()
    assert L.curandCreateGenerator(C.byref(g), capi.CURAND_RNG_PSEUDO_PHILOX4_32_10) == 0
    for fn, args in (("curandGenerateLogNormal", (C.c_float(0), C.c_float(1))),
                     ("curandGenerateNormalDouble", (0.0, 1.0)),
                     ("curandGenerateLogNormalDouble", (0.0, 1.0)),
                     ("curandGeneratePoisson", (3.0,)), ("curandGenerateUniformDouble", ())):
        f = getattr(L, fn)
        assert f(g, None, 4, *args) == capi.CURAND_STATUS_INVALID_VALUE
        assert f(g, None, 0, *args) == 0
        assert f(C.c_void_p(12345), C.c_void_p(4096), 4, *args) == \
            capi.CURAND_STATUS_NOT_INITIALIZED
    assert L.curandSetQuasiRandomGeneratorDimensions(g, 0) == 104  # OUT_OF_RANGE
    assert L.curandSetQuasiRandomGeneratorDimensions(g, 20001) == 104
    assert L.curandSetQuasiRandomGeneratorDimensions(g, 20000) == 0
    assert L.curandSetQuasiRandomGeneratorDimensions(C.c_void_p(12345), 3) == \
        capi.CURAND_STATUS_NOT_INITIALIZED
    v = C.c_void_p()
    assert L.curandGetDirectionVectors32(C.byref(v), 101) == 0
    dirs = np.ctypeslib.as_array(C.cast(v, C.POINTER(C.c_uint32)), (32,))
    assert dirs[0] == 0x80000000 and dirs[31] == 1
    assert L.curandGetDirectionVectors32(C.byref(v), 103) == 104
    assert L.curandGetDirectionVectors32(None, 101) == capi.CURAND_STATUS_INVALID_VALUE
    sc = C.c_void_p()
    assert L.curandGetScrambleConstants32(C.byref(sc)) == 0
    assert C.cast(sc, C.POINTER(C.c_uint32))[0] == 0x6543210F
    assert L.curandDestroyGenerator(g) == 0


# --------------------------------------------------------------------- GPU --
def _gen(torch, g, fn, n, dtype, *args, host=False):
    L = capi.curand()
    if host:
        out = np.zeros(n + 1, dtype)
        ptr = C.c_void_p(out.ctypes.data + out.itemsize)  # odd element offset
        assert getattr(L, fn)(g, ptr, n, *args) == 0
        return out[1:]
    t = torch.zeros(n + 1, dtype={np.float64: torch.float64, np.float32: torch.float32,
                                  np.uint32: torch.int32}[dtype], device="cuda")
    assert getattr(L, fn)(g, C.c_void_p(t.data_ptr() + t.element_size()), n, *args) == 0
    torch.cuda.synchronize()
    return t.cpu().numpy()[1:].view(dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("host", [False, True])
def test_gpu_uniform_double_bit_exact(cuda, built, host):
    with curand_generator(42, cuda, host=host, offset=10) as g:
        a = _gen(cuda, g, "curandGenerateUniformDouble", 100_001, np.float64, host=host)
        b = _gen(cuda, g, "curandGenerateUniformDouble", 7, np.float64, host=host)
    ra, nxt = oracle.generate_double(42, 10, 100_001)
    rb, _ = oracle.generate_double(42, nxt, 7)
    assert np.array_equal(a, ra) and np.array_equal(b, rb)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["normal", "lognormal"])
def test_gpu_normal_lognormal_double(cuda, built, kind):
    fn = "curandGenerateNormalDouble" if kind == "normal" else "curandGenerateLogNormalDouble"
    with curand_generator(7, cuda, offset=3) as g:
        got = _gen(cuda, g, fn, 200_001, np.float64, 0.5, 1.5)
    want, _ = oracle.generate_double(7, 3, 200_001, kind, 0.5, 1.5)
    scale = np.maximum(1.0, np.abs(want)) if kind == "normal" else np.abs(want)
    assert np.all(np.abs(got - want) <= 1e-13 * scale)


@pytest.mark.gpu
@pytest.mark.parametrize("host", [False, True])
def test_gpu_lognormal_f32(cuda, built, host):
    with curand_generator(1234, cuda, host=host) as g:
        got = _gen(cuda, g, "curandGenerateLogNormal", 300_003, np.float32, C.c_float(0.2),
                   C.c_float(0.75), host=host)
        nxt = _gen(cuda, g, "curandGenerateLogNormal", 5, np.float32, C.c_float(0.2),
                   C.c_float(0.75), host=host)
    want, off = oracle.generate_lognormal(1234, 0, 300_003, 0.2, 0.75)
    want2, _ = oracle.generate_lognormal(1234, off, 5, 0.2, 0.75)
    for g_, w in ((got, want), (nxt, want2)):
        rel = np.abs(g_.astype(np.float64) / w - 1)
        assert np.all(rel <= 2e-6 * np.maximum(1, np.abs(np.log(w))) + 3e-7)


@pytest.mark.gpu
@pytest.mark.parametrize("lam", [0.25, 3.0, 12.0, 29.9])
@pytest.mark.parametrize("host", [False, True])
def test_gpu_poisson_small_lambda_bit_exact(cuda, built, lam, host):
    with curand_generator(99, cuda, host=host, offset=17) as g:
        a = _gen(cuda, g, "curandGeneratePoisson", 100_003, np.uint32, lam, host=host)
        b = _gen(cuda, g, "curandGeneratePoisson", 11, np.uint32, lam, host=host)
    ra, nxt = oracle.generate_poisson(99, 17, 100_003, lam)
    rb, _ = oracle.generate_poisson(99, nxt, 11, lam)
    assert np.array_equal(a, ra) and np.array_equal(b, rb)


@pytest.mark.gpu
@pytest.mark.parametrize("lam", [30.0, 1000.0, 1e6])
def test_gpu_poisson_large_lambda(cuda, built, lam):
    with curand_generator(3, cuda) as g:
        got = _gen(cuda, g, "curandGeneratePoisson", 1_000_000, np.uint32, lam)
    want, _ = oracle.generate_poisson(3, 0, 1_000_000, lam)
    diff = got.astype(np.int64) - want.astype(np.int64)
    assert np.mean(diff == 0) >= 0.9999 and np.all(np.abs(diff) <= 1)
    assert abs(got.mean() - lam) < 6 * np.sqrt(lam / len(got)) + 1e-3
