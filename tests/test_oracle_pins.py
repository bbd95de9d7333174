"""Pins the CPU oracle against the reference's own known-answer tests (CPU only).

Each test restates a check from the reference's test suite and runs it on the
oracle; the GPU tests then compare the CUDA kernels with this pinned oracle.
"""

import json
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


# ---------------------------------------------------------------- Philox --
def test_philox_host_moments_match_reference_test():
    """tests/curand_test.cpp:117-201 (seed 42, 100000 samples, host generator)."""
    u, off = oracle.generate_uniform(42, 0, 100000)
    assert np.all(u > 0.0) and np.all(u <= 1.0)
    assert abs(u.astype(np.float64).mean() - 0.5) < 0.01
    assert abs(u.astype(np.float64).var() - 0.08333) < 0.005
    z, off = oracle.generate_normal(42, off, 100000, 10.0, 3.0)
    assert abs(z.astype(np.float64).mean() - 10.0) < 0.05
    assert abs(z.astype(np.float64).var() - 9.0) < 0.25


def test_philox_determinism_and_offset_match_reference_test():
    """tests/curand_test.cpp:316-363: same seed -> same stream; offset 1024 reproduces
    the second batch of 1024 draws."""
    a, off_a = oracle.generate_uint(777, 0, 1024)
    b, _ = oracle.generate_uint(777, 0, 1024)
    assert np.array_equal(a, b)
    nxt1, _ = oracle.generate_uint(777, off_a, 1024)
    nxt3, _ = oracle.generate_uint(777, 1024, 1024)
    assert off_a == 1024
    assert np.array_equal(nxt1, nxt3)


def test_philox_offset_advances_by_whole_blocks():
    """curand_api.mm:275 — offset += 4*ceil(n/4)."""
    for n, expect in [(1, 4), (4, 4), (5, 8), (1023, 1024)]:
        _, off = oracle.generate_uniform(1, 0, n)
        assert off == expect


def test_philox_thread_count_does_not_change_output():
    a, _ = oracle.generate_normal(1234, 8, 4099, 0.0, 1.0, threads=1)
    b, _ = oracle.generate_normal(1234, 8, 4099, 0.0, 1.0, threads=7)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_philox_golden_vectors():
    data = json.loads((GOLDEN / "philox.json").read_text())
    for c in data["cases"]:
        w, nxt = oracle.generate_uint(c["seed"], c["offset"], c["n"])
        assert [int(v) for v in w] == c["uint"]
        assert nxt == c["next_offset"]
        u, _ = oracle.generate_uniform(c["seed"], c["offset"], c["n"])
        assert [int(v) for v in u.view(np.uint32)] == c["uniform_bits"]
        z, _ = oracle.generate_normal(c["seed"], c["offset"], c["n"])
        np.testing.assert_array_equal(z, np.asarray(c["normal"], dtype=np.float32))


def test_philox_uniform_range_includes_one_excludes_zero():
    # u = 0xFFFFFFFF rounds to 2^32 as float; +1 keeps 2^32; * 2^-32 = 1.0 exactly.
    words = np.array([0, 0xFFFFFFFF, 0xFFFFFF7F, 1 << 31], dtype=np.uint32)
    f = ((words.astype(np.float32) + np.float32(1.0)) * np.float32(2.3283064365386963e-10))
    assert f[1] == np.float32(1.0)
    assert f[0] > 0.0
