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


# ------------------------------------------------------------- conv/softmax --
def test_conv_pin_reference_test():
    """tests/cudnn_test.cpp:40-107: 1x2x4x4 ones, 2x2x3x3 filter of 0.5, pad 1, stride 1,
    then + bias 1.25 -> corner 5.25, centre 10.25.  The bias is folded in with beta = 1
    over a y pre-filled with 1.25."""
    x = np.ones(32, np.float32)
    w = np.full(36, 0.5, np.float32)
    y = np.full(32, 1.25, np.float32)
    oracle.conv2d(x, w, (1, 2, 4, 4), (2, 2, 3, 3), pad=(1, 1), beta=1.0, y=y)
    assert abs(y[0] - 5.25) < 1e-4
    assert abs(y[1 * 4 + 1] - 10.25) < 1e-4


def test_conv_krsc_equals_kcrs_and_flip():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(2 * 3 * 5 * 6).astype(np.float32)
    w_kcrs = rng.standard_normal(4 * 3 * 3 * 2).astype(np.float32).reshape(4, 3, 3, 2)
    w_krsc = np.ascontiguousarray(w_kcrs.transpose(0, 2, 3, 1))
    a = oracle.conv2d(x, w_kcrs.reshape(-1), (2, 3, 5, 6), (4, 3, 3, 2), pad=(1, 0))
    b = oracle.conv2d(x, w_krsc.reshape(-1), (2, 3, 5, 6), (4, 3, 3, 2), pad=(1, 0), w_fmt="NHWC")
    np.testing.assert_array_equal(a, b)
    # CONVOLUTION mode = cross-correlation with the spatially flipped filter
    c = oracle.conv2d(x, np.ascontiguousarray(w_kcrs[:, :, ::-1, ::-1]).reshape(-1),
                      (2, 3, 5, 6), (4, 3, 3, 2), pad=(1, 0), mode="conv")
    np.testing.assert_allclose(a, c, rtol=1e-6, atol=1e-6)


def test_conv_oracle_matches_numpy_double():
    rng = np.random.default_rng(1)
    n, c, h, w, k, r, s = 2, 4, 7, 6, 6, 3, 3
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    f = rng.standard_normal((k, c // 2, r, s)).astype(np.float32)
    got = oracle.conv2d(x.reshape(-1), f.reshape(-1), (n, c, h, w), (k, c // 2, r, s),
                        pad=(2, 1), stride=(2, 1), dil=(2, 1), groups=2).reshape(n, k, -1)
    oh = 1 + (h + 4 - 5) // 2
    ow = 1 + (w + 2 - 3) // 1
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (2, 2), (1, 1)))
    want = np.zeros((n, k, oh, ow))
    for oc in range(k):
        g = oc // (k // 2)
        for i in range(oh):
            for j in range(ow):
                patch = xp[:, g * 2:(g + 1) * 2, i * 2:i * 2 + 5:2, j:j + 3]
                want[:, oc, i, j] = (patch * f[oc].astype(np.float64)).sum(axis=(1, 2, 3))
    np.testing.assert_allclose(got.reshape(n, k, oh, ow), want, rtol=1e-5, atol=1e-5)


def test_softmax_pin_reference_test():
    """tests/cudnn_test.cpp:221-236: softmax over [1, 2] (CHANNEL, ACCURATE)."""
    y = oracle.softmax(np.array([1.0, 2.0], np.float32), (1, 2, 1, 1), channel=True)
    e1, e2 = np.exp(1.0), np.exp(2.0)
    assert abs(y[0] - e1 / (e1 + e2)) < 1e-5 and abs(y[1] - e2 / (e1 + e2)) < 1e-5


def test_softmax_algos_and_modes():
    rng = np.random.default_rng(2)
    x = rng.standard_normal(3 * 5 * 2 * 4).astype(np.float32)
    x64 = x.astype(np.float64).reshape(3, 5, 2, 4)
    # INSTANCE over (c, h, w); CHANNEL over c per pixel
    inst = np.exp(x64 - x64.max(axis=(1, 2, 3), keepdims=True))
    inst /= inst.sum(axis=(1, 2, 3), keepdims=True)
    chan = np.exp(x64 - x64.max(axis=1, keepdims=True))
    chan /= chan.sum(axis=1, keepdims=True)
    for algo in (0, 1):
        y = oracle.softmax(x, (3, 5, 2, 4), algo=algo)
        np.testing.assert_allclose(y.reshape(inst.shape), inst, rtol=1e-5, atol=1e-7)
        y = oracle.softmax(x, (3, 5, 2, 4), algo=algo, channel=True)
        np.testing.assert_allclose(y.reshape(chan.shape), chan, rtol=1e-5, atol=1e-7)
    y = oracle.softmax(x, (3, 5, 2, 4), algo=2)
    np.testing.assert_allclose(y.reshape(inst.shape), np.log(inst), rtol=1e-5, atol=1e-5)
