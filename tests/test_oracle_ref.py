"""The Philox oracle against the reference's own host generator, compiled here.

oracle/_ref/libcurand_ref.so is the reference's unmodified
libraries/rand/src/curand_context.mm built by oracle/ref/build.py.  Both are
compiled by the same g++ against the same libm with -ffp-contract=off, so every
stream must agree bit for bit: uint32, uniform, normal, log-normal, the double
streams and the host Poisson path, with the same next offset.  The committed
golden vectors are checked against it as well.
"""

import json
from pathlib import Path

import numpy as np
import pytest

import oracle
import oracle.ref as ref
from oracle.ref.build import build as build_ref

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module", autouse=True)
def reference_lib():
    build_ref()
    if not ref.available():
        pytest.skip("oracle/_ref/libcurand_ref.so not built (reference tree absent)")
    return ref.lib()


SEEDS = [0, 1, 1234, 42, 0xDEADBEEFCAFEF00D, 0xFFFFFFFFFFFFFFFF]
OFFSETS = [0, 1, 2, 3, 4, 6, 1024, 1 << 30, (1 << 34) - 64, (1 << 63) - 8]
SIZES = [0, 1, 3, 4, 5, 4099]


def _bits(a):
    return a.view({4: np.uint32, 8: np.uint64}[a.dtype.itemsize])


def test_philox_step_matches(reference_lib):
    rng = np.random.default_rng(5)
    for ctr, seed in zip(rng.integers(0, 2**63, 2000, dtype=np.uint64),
                         rng.integers(0, 2**63, 2000, dtype=np.uint64)):
        ctr, seed = int(ctr) * 2 + 1, int(seed)
        assert np.array_equal(ref.philox_step(ctr, seed), oracle.philox_block(ctr, seed))


@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("offset", OFFSETS)
def test_float_streams_bit_exact(seed, offset):
    for n in SIZES:
        for kind, ours in ((ref.UINT, oracle.generate_uint),
                           (ref.UNIFORM, oracle.generate_uniform)):
            want, nxt = ref.generate(kind, seed, offset, n)
            got, onxt = ours(seed, offset, n)
            assert np.array_equal(_bits(got), _bits(want)) and nxt == onxt
        for mean, std in ((0.0, 1.0), (10.0, 3.0)):
            want, nxt = ref.generate(ref.NORMAL, seed, offset, n, mean, std)
            got, onxt = oracle.generate_normal(seed, offset, n, mean, std)
            assert np.array_equal(_bits(got), _bits(want)) and nxt == onxt
            want, nxt = ref.generate(ref.LOGNORMAL, seed, offset, n, mean / 10, std / 3)
            got, onxt = oracle.generate_lognormal(seed, offset, n, mean / 10, std / 3)
            assert np.array_equal(_bits(got), _bits(want)) and nxt == onxt


@pytest.mark.parametrize("seed", SEEDS[:4])
@pytest.mark.parametrize("offset", [0, 1, 2, 3, 1 << 30])
def test_double_streams_bit_exact(seed, offset):
    for n in (0, 1, 2, 3, 1001):
        for kind, name in ((ref.UNIFORM_DOUBLE, "uniform"), (ref.NORMAL_DOUBLE, "normal"),
                           (ref.LOGNORMAL_DOUBLE, "lognormal")):
            want, nxt = ref.generate(kind, seed, offset, n, 0.5, 2.0)
            got, onxt = oracle.generate_double(seed, offset, n, name, 0.5, 2.0)
            assert np.array_equal(_bits(got), _bits(want)) and nxt == onxt, (name, n)


@pytest.mark.parametrize("lam", [0.5, 4.0, 29.5, 30.0, 100.0, 1e4])
def test_poisson_host_path_bit_exact(lam):
    """The oracle's restatement of the reference's host Poisson path (mode 1) equals
    the reference; the library's own definition (mode 0, the device kernel's) is a
    different stream, as the reference's host and GPU kernels are."""
    for seed, offset, n in ((7, 0, 3001), (1234, 12345, 257)):
        want, nxt = ref.generate(ref.POISSON, seed, offset, n, lam=lam)
        got, onxt = oracle.generate_poisson(seed, offset, n, lam, reference_host=True)
        assert np.array_equal(got, want) and nxt == onxt


def test_config_streams_sampled():
    """seed 1234, uniform from offset 0, normal from offset 2^30: sampled
    Philox blocks of each 2^30-word call, first and last included, agree bit for bit."""
    blocks = (1 << 30) // 4
    rng = np.random.default_rng(11)
    idx = np.unique(np.concatenate([rng.integers(0, blocks, 4096), [0, 1, blocks - 1]]))
    for kind, base, ours in ((ref.UNIFORM, 0, oracle.generate_uniform),
                             (ref.NORMAL, 1 << 30, oracle.generate_normal)):
        want = ref.generate_at(kind, 1234, base + 4 * idx.astype(np.uint64), 4)
        got = np.stack([ours(1234, base + 4 * int(i), 4)[0] for i in idx[:512]])
        assert np.array_equal(_bits(got), _bits(want[:512]))


def test_parallel_reference_call_is_one_call():
    """The bench's reference arm splits one GenerateHost* call over host threads; the
    output and next offset equal the single-threaded call."""
    for kind in (ref.UINT, ref.UNIFORM, ref.NORMAL, ref.UNIFORM_DOUBLE):
        for n in (0, 1, 5, 4097, 100003):
            want, nxt = ref.generate(kind, 1234, 1 << 30, n, 0.0, 1.0)
            got, pnxt = ref.generate_parallel(kind, 1234, 1 << 30, n, 0.0, 1.0, threads=7)
            assert np.array_equal(_bits(got), _bits(want)) and nxt == pnxt


def test_golden_file_is_the_reference():
    doc = json.loads((GOLDEN / "philox.json").read_text())
    for c in doc["cases"]:
        u, nxt = ref.generate(ref.UINT, c["seed"], c["offset"], c["n"])
        assert [int(v) for v in u] == c["uint"] and nxt == c["next_offset"]
        f, _ = ref.generate(ref.UNIFORM, c["seed"], c["offset"], c["n"])
        assert [int(v) for v in f.view(np.uint32)] == c["uniform_bits"]
        z, _ = ref.generate(ref.NORMAL, c["seed"], c["offset"], c["n"], 0.0, 1.0)
        assert [int(v) for v in z.view(np.uint32)] == c["normal_bits"]
