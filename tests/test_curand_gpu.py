"""Philox4x32-10 on the GPU through the C ABI, checked against the pinned oracle.

Bar: uint32 and uniform streams bit-exact; normal within an absolute bound of
NORMAL_TOL * max(1, |z|) (CUDA's logf/sincosf and glibc's differ by a few ulp;
both are correctly rounded sqrt and explicitly rounded affine steps).
"""

import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from muda_b200 import capi
from tests.helpers import curand_generator, ulp_distance_f32

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
NORMAL_TOL = 2e-6  # absolute, scaled by max(1, |z|)


def _gen(torch, fn, g, n, dtype, offset_elems=0, *extra):
    buf = torch.empty(n + offset_elems + 4, dtype=dtype, device="cuda")
    ptr = buf.data_ptr() + offset_elems * buf.element_size()
    assert fn(g, C.c_void_p(ptr), n, *extra) == 0
    torch.cuda.synchronize()
    return buf[offset_elems:offset_elems + n].cpu().numpy()


# The last three cases put the counter's high word change (block 2^32) inside the call,
# right after its last full block (the partial block then runs as its own segment), and
# in a call of fewer than four words just below it.
CASES = [(1234, 0, 1 << 16), (1234, 4096, 1000), (42, 0, 4097), (777, 1024, 1023),
         (9999, 6, 19), (0xDEADBEEFCAFEF00D, (1 << 34) - 64, 100003), (5, 0, 1), (5, 0, 3),
         (0xDEADBEEFCAFEF00D, (1 << 34) - 64, 67), (7, (1 << 34) - 4, 2),
         (11, (1 << 35) - 4 * 300000, 1 << 21)]


@pytest.mark.parametrize("seed,offset,n", CASES)
@pytest.mark.parametrize("misalign", [0, 1])
def test_uint_and_uniform_bit_exact(cuda, built, seed, offset, n, misalign):
    torch = cuda
    L = capi.curand()
    with curand_generator(seed, torch, offset=offset) as g:
        got_u = _gen(torch, L.curandGenerate, g, n, torch.int32, misalign).view(np.uint32)
    want_u, _ = oracle.generate_uint(seed, offset, n)
    assert np.array_equal(got_u, want_u)
    with curand_generator(seed, torch, offset=offset) as g:
        got_f = _gen(torch, L.curandGenerateUniform, g, n, torch.float32, misalign)
    want_f, _ = oracle.generate_uniform(seed, offset, n)
    assert np.array_equal(got_f.view(np.uint32), want_f.view(np.uint32))


@pytest.mark.parametrize("seed,offset,n", CASES)
def test_normal_within_tolerance(cuda, built, seed, offset, n):
    torch = cuda
    L = capi.curand()
    for mean, std in ((0.0, 1.0), (3.0, 1.0), (10.0, 3.0)):
        with curand_generator(seed, torch, offset=offset) as g:
            got = _gen(torch, L.curandGenerateNormal, g, n, torch.float32, 0,
                       C.c_float(mean), C.c_float(std))
        want, _ = oracle.generate_normal(seed, offset, n, mean, std)
        err = np.abs(got.astype(np.float64) - want.astype(np.float64))
        bound = NORMAL_TOL * std * np.maximum(1.0, np.abs(want.astype(np.float64) - mean)) + \
            4 * np.spacing(np.float32(abs(mean) + 1))
        assert np.all(err <= bound), f"max err {err.max()} (ulp {ulp_distance_f32(got, want).max()})"


def test_golden_vectors_on_gpu(cuda, built):
    torch = cuda
    L = capi.curand()
    for c in json.loads((GOLDEN / "philox.json").read_text())["cases"]:
        with curand_generator(c["seed"], torch, offset=c["offset"]) as g:
            got = _gen(torch, L.curandGenerate, g, c["n"], torch.int32).view(np.uint32)
        assert [int(v) for v in got] == c["uint"]
        with curand_generator(c["seed"], torch, offset=c["offset"]) as g:
            got = _gen(torch, L.curandGenerateUniform, g, c["n"], torch.float32)
        assert [int(v) for v in got.view(np.uint32)] == c["uniform_bits"]


def test_config_sequence_uniform_then_normal(cuda, built):
    """Config: seed 1234, offset 0, uniform then normal on the same generator and
    stream; the normal call continues at offset 4*ceil(n/4)."""
    torch = cuda
    L = capi.curand()
    n = (1 << 20) + 3
    with curand_generator(1234, torch) as g:
        u = _gen(torch, L.curandGenerateUniform, g, n, torch.float32)
        z = _gen(torch, L.curandGenerateNormal, g, n, torch.float32, 0, C.c_float(0.0),
                 C.c_float(1.0))
    want_u, off = oracle.generate_uniform(1234, 0, n, threads=8)
    want_z, _ = oracle.generate_normal(1234, off, n, 0.0, 1.0, threads=8)
    assert off == 4 * ((n + 3) // 4)
    assert np.array_equal(u.view(np.uint32), want_u.view(np.uint32))
    err = np.abs(z.astype(np.float64) - want_z)
    assert np.all(err <= NORMAL_TOL * np.maximum(1.0, np.abs(want_z)))
    exact = np.mean(z.view(np.uint32) == want_z.view(np.uint32))
    print(f"normal: {exact:.4%} bit-identical, max |err| {err.max():.3e}")


def test_host_generator_matches_device_stream(cuda, built):
    torch = cuda
    L = capi.curand()
    n = (1 << 26) + 4096 + 5  # crosses the 256 MiB staging chunk
    out = np.zeros(n, dtype=np.float32)
    with curand_generator(77, None, host=True, offset=40) as g:
        assert L.curandGenerateUniform(g, out.ctypes.data_as(C.c_void_p), n) == 0
    want, _ = oracle.generate_uniform(77, 40, n, threads=8)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_reference_gpu_moments(cuda, built):
    """tests/curand_test.cpp:203-314: seed 9999, 65536 draws."""
    torch = cuda
    L = capi.curand()
    with curand_generator(9999, torch) as g:
        u = _gen(torch, L.curandGenerateUniform, g, 65536, torch.float32).astype(np.float64)
        z = _gen(torch, L.curandGenerateNormal, g, 65536, torch.float32, 0, C.c_float(0.0),
                 C.c_float(1.0)).astype(np.float64)
    assert np.all(u > 0) and np.all(u <= 1)
    assert abs(u.mean() - 0.5) < 0.015
    assert abs(z.mean()) < 0.03 and abs(z.var() - 1.0) < 0.05


def test_config_streams_against_reference(cuda, built):
    """configs[1] at full size: seed 1234, curandGenerateUniform of 2^30 words from
    offset 0, then curandGenerateNormal of 2^30 words on the same generator and
    stream (offset 2^30, first counter 2^28).  2^16 randomly sampled Philox blocks
    of each call plus the first and last blocks are compared with the reference's
    own host generator (oracle/_ref, its curand_context.mm compiled here): uniform
    bit for bit, normal within NORMAL_TOL * max(1, |z|).  The oracle restatement
    is checked on the same blocks, so the test also runs where oracle/_ref is
    missing."""
    import oracle.ref as ref
    torch = cuda
    L = capi.curand()
    n = 1 << 30
    u = torch.empty(n, dtype=torch.float32, device="cuda")
    z = torch.empty(n, dtype=torch.float32, device="cuda")
    with curand_generator(1234, torch) as g:
        assert L.curandGenerateUniform(g, C.c_void_p(u.data_ptr()), n) == 0
        assert L.curandGenerateNormal(g, C.c_void_p(z.data_ptr()), n, C.c_float(0.0),
                                      C.c_float(1.0)) == 0
    torch.cuda.synchronize()
    blocks = n // 4
    rng = np.random.default_rng(0)
    idx = np.unique(np.concatenate([rng.integers(0, blocks, 1 << 16), [0, 1, blocks - 1]]))
    sel = torch.from_numpy(idx).cuda()
    got_u = u.view(-1, 4)[sel].cpu().numpy()
    got_z = z.view(-1, 4)[sel].cpu().numpy().astype(np.float64)
    del u, z
    torch.cuda.empty_cache()
    words = oracle.philox_gather(idx.astype(np.uint64), 1234)
    want_u = ((words.astype(np.float32) + np.float32(1.0)) *
              np.float32(2.3283064365386963e-10)).astype(np.float32)
    assert np.array_equal(got_u.view(np.uint32), want_u.view(np.uint32))
    offs = 4 * idx.astype(np.uint64)
    if ref.available():
        ref_u = ref.generate_at(ref.UNIFORM, 1234, offs, 4)
        assert np.array_equal(got_u.view(np.uint32), ref_u.view(np.uint32))
        want_z = ref.generate_at(ref.NORMAL, 1234, offs + np.uint64(n), 4).astype(np.float64)
    else:
        want_z = np.stack([oracle.generate_normal(1234, n + int(o), 4)[0] for o in offs])
        want_z = want_z.astype(np.float64)
    err = np.abs(got_z - want_z)
    assert np.all(err <= NORMAL_TOL * np.maximum(1.0, np.abs(want_z))), f"max err {err.max()}"
    exact = np.mean(got_z.astype(np.float32).view(np.uint32) == want_z.astype(np.float32).view(np.uint32))
    print(f"config normal vs {'reference' if ref.available() else 'oracle'}: "
          f"max |err| {err.max():.3e}, {exact:.2%} bit-identical")


def test_normal_transform_error_budget(cuda, built):
    """The error bound of the normal transform from its parts, each measured over every
    fp32 input of its step (mb200ProbeNormalError runs the shipped device code):
    |dz| <= |dr| |cos| + r |dcos| (+ the product's rounding and the reference formula's
    own rounding, 2^-24 |z| each) stays below NORMAL_TOL * max(1, |z|) for r up to the
    hardware path's threshold; above it the polynomial path's error is negligible."""
    torch = cuda
    P = capi.probe()
    out = torch.zeros(8, dtype=torch.float32, device="cuda")
    assert P.mb200ProbeNormalError(C.c_void_p(out.data_ptr()),
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    dr, dc_hw, ds_hw, dc_poly, ds_poly, r_max = (float(v) for v in out[:6].cpu())
    print(f"radius {dr:.3e} * max(1, r); hw cos {dc_hw:.3e} sin {ds_hw:.3e}; "
          f"poly cos {dc_poly:.3e} sin {ds_poly:.3e}; hw up to r = {r_max}")
    d_trig = max(dc_hw, ds_hw)
    rounding = 2.0 * 2.0 ** -24
    # |z| < 1 (then |cos| <= 1 / r): |dz| <= dr * max(1, r) |cos| + r d_trig <= dr + r d_trig
    worst_small = dr + r_max * d_trig + rounding
    # |z| >= 1: |dz| / |z| <= dr + d_trig / |cos| <= dr + r d_trig (|cos| >= 1 / r)
    worst_rel = dr + r_max * d_trig + rounding
    assert worst_small <= NORMAL_TOL and worst_rel <= NORMAL_TOL, (worst_small, worst_rel)
    # the fallback (polynomials, reduction by pi/2) for radii up to sqrt(-2 ln 2^-32) = 6.66
    assert max(dc_poly, ds_poly) <= 2e-7
    assert dr + 6.67 * max(dc_poly, ds_poly) + rounding <= NORMAL_TOL


def test_config_normal_every_output(cuda, built):
    """The whole normal call of configs[1] (2^30 words from offset 2^30, seed 1234):
    every output against the oracle restatement of the reference formula (glibc
    float functions), within NORMAL_TOL * max(1, |z|), in chunks of 2^26 words."""
    import os
    torch = cuda
    L = capi.curand()
    n = 1 << 30
    z = torch.empty(n, dtype=torch.float32, device="cuda")
    with curand_generator(1234, torch, offset=n) as g:
        assert L.curandGenerateNormal(g, C.c_void_p(z.data_ptr()), n, C.c_float(0.0),
                                      C.c_float(1.0)) == 0
    torch.cuda.synchronize()
    chunk = 1 << 26
    worst = 0.0
    exact = 0
    for c0 in range(0, n, chunk):
        got = z[c0:c0 + chunk].cpu().numpy()
        want, _ = oracle.generate_normal(1234, n + c0, chunk, 0.0, 1.0,
                                         threads=os.cpu_count() or 1)
        err = np.abs(got.astype(np.float64) - want.astype(np.float64))
        ratio = err / (NORMAL_TOL * np.maximum(1.0, np.abs(want.astype(np.float64))))
        worst = max(worst, float(ratio.max()))
        exact += int(np.count_nonzero(got.view(np.uint32) == want.view(np.uint32)))
        assert worst <= 1.0, f"chunk at {c0}: max err / bound {worst}"
    del z
    torch.cuda.empty_cache()
    print(f"2^30 normals: max err / bound {worst:.3f}, {exact / n:.2%} bit-identical")


@pytest.mark.parametrize("seed,offset,n", [(1234, 0, 4099), (9, 6, 1001), (1234, 1 << 30, 65537)])
def test_streams_against_reference(cuda, built, seed, offset, n):
    """uint32, uniform and normal against the reference's compiled host generator."""
    import oracle.ref as ref
    if not ref.available():
        pytest.skip("oracle/_ref/libcurand_ref.so missing: build() ran without the reference tree")
    torch = cuda
    L = capi.curand()
    with curand_generator(seed, torch, offset=offset) as g:
        got = _gen(torch, L.curandGenerate, g, n, torch.int32).view(np.uint32)
    assert np.array_equal(got, ref.generate(ref.UINT, seed, offset, n)[0])
    with curand_generator(seed, torch, offset=offset) as g:
        got = _gen(torch, L.curandGenerateUniform, g, n, torch.float32)
    assert np.array_equal(got.view(np.uint32), ref.generate(ref.UNIFORM, seed, offset, n)[0].view(np.uint32))
    with curand_generator(seed, torch, offset=offset) as g:
        got = _gen(torch, L.curandGenerateNormal, g, n, torch.float32, 0, C.c_float(0.0),
                   C.c_float(1.0)).astype(np.float64)
    want = ref.generate(ref.NORMAL, seed, offset, n)[0].astype(np.float64)
    assert np.all(np.abs(got - want) <= NORMAL_TOL * np.maximum(1.0, np.abs(want)))


def test_unaddressable_output_is_rejected(cuda, built):
    torch = cuda
    L = capi.curand()
    host = np.zeros(64, dtype=np.float32)  # pageable host memory: not device-addressable
    with curand_generator(1, torch) as g:
        st = L.curandGenerateUniform(g, host.ctypes.data_as(C.c_void_p), 64)
        assert st == capi.CURAND_STATUS_ALLOCATION_FAILED
        small = torch.empty(16, dtype=torch.float32, device="cuda")
        # a span longer than the whole allocation segment is rejected before launch
        st = L.curandGenerateUniform(g, C.c_void_p(small.data_ptr()), 1 << 40)
        assert st == capi.CURAND_STATUS_ALLOCATION_FAILED
