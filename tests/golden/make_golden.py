"""Generates the committed golden vectors under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

Philox goldens come from the reference's own host generator: its unmodified
libraries/rand/src/curand_context.mm compiled as C++ by oracle/ref/build.py
(GenerateHostUint / GenerateHostUniform / GenerateHostNormal, lines 75-185).
Two independent restatements must agree with it bit for bit before a file is
written: the C++ oracle (oracle/philox.cpp) and the vectorised numpy
restatement below.  The committed file then pins the oracle, and gives the GPU
tests fixed expected values, on machines where the reference tree is absent.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
import oracle.ref as ref  # noqa: E402
from oracle.ref.build import build as build_ref  # noqa: E402

OUT = Path(__file__).resolve().parent

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = np.uint32(0x9E3779B9)
W1 = np.uint32(0xBB67AE85)
MASK = np.uint64(0xFFFFFFFF)


def philox_numpy(ctr: np.ndarray, seed: int) -> np.ndarray:
    """Philox4x32-10 of counters (ctr_lo, ctr_hi, 0, 0) under key (seed_lo, seed_hi)."""
    ctr = ctr.astype(np.uint64)
    c0 = ctr & MASK
    c1 = ctr >> np.uint64(32)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = np.uint64(seed & 0xFFFFFFFF)
    k1 = np.uint64((seed >> 32) & 0xFFFFFFFF)
    for _ in range(10):
        p0 = M0 * c0
        p1 = M1 * c2
        c0, c1, c2, c3 = ((p1 >> np.uint64(32)) ^ c1 ^ k0, p1 & MASK,
                          (p0 >> np.uint64(32)) ^ c3 ^ k1, p0 & MASK)
        k0 = (k0 + np.uint64(W0)) & MASK
        k1 = (k1 + np.uint64(W1)) & MASK
    return np.stack([c0, c1, c2, c3], axis=1).astype(np.uint32)


def stream_numpy(seed: int, offset: int, n: int) -> np.ndarray:
    blocks = (n + 3) // 4
    ctr = np.arange(blocks, dtype=np.uint64) + np.uint64(offset >> 2)
    return philox_numpy(ctr, seed).reshape(-1)[:n]


def uniform_numpy(words: np.ndarray) -> np.ndarray:
    f = words.astype(np.float32)  # round-to-nearest conversion
    return ((f + np.float32(1.0)) * np.float32(2.3283064365386963e-10)).astype(np.float32)


def main() -> None:
    if build_ref() is None:
        raise SystemExit("the reference tree is needed: oracle/ref/build.py found none")
    cases = []
    # (seed, offset, n): config seed, reference test seeds, tails, odd offsets,
    # a counter that crosses 2^32 and a 64-bit seed.
    for seed, offset, n in [
        (1234, 0, 64), (1234, 4, 64), (1234, 1024, 64), (1234, 1 << 30, 64),
        (42, 0, 67), (777, 1024, 33), (9999, 6, 19), (12345, 0, 16),
        (0xDEADBEEFCAFEF00D, (1 << 34) - 8, 40), (0, 0, 8),
    ]:
        words, nxt = ref.generate(ref.UINT, seed, offset, n)
        uni, nxt_u = ref.generate(ref.UNIFORM, seed, offset, n)
        nor, nxt_n = ref.generate(ref.NORMAL, seed, offset, n, 0.0, 1.0)
        o_words, o_nxt = oracle.generate_uint(seed, offset, n)
        o_uni, _ = oracle.generate_uniform(seed, offset, n)
        o_nor, _ = oracle.generate_normal(seed, offset, n, 0.0, 1.0)
        np_words = stream_numpy(seed, offset, n)
        if not (np.array_equal(words, o_words) and np.array_equal(words, np_words)
                and nxt == o_nxt == nxt_u == nxt_n):
            raise SystemExit(f"uint disagreement at seed={seed} offset={offset}")
        if not (np.array_equal(uni.view(np.uint32), o_uni.view(np.uint32)) and
                np.array_equal(uni.view(np.uint32), uniform_numpy(np_words).view(np.uint32))):
            raise SystemExit(f"uniform disagreement at seed={seed} offset={offset}")
        if not np.array_equal(nor.view(np.uint32), o_nor.view(np.uint32)):
            raise SystemExit(f"normal disagreement at seed={seed} offset={offset}")
        cases.append({
            "seed": seed, "offset": offset, "n": n, "next_offset": nxt,
            "uint": [int(v) for v in words],
            "uniform_bits": [int(v) for v in uni.view(np.uint32)],
            "normal": [float(v) for v in nor],
            "normal_bits": [int(v) for v in nor.view(np.uint32)],
        })
    doc = {"source": "reference libraries/rand/src/curand_context.mm:42-185 compiled by "
                     "oracle/ref/build.py (g++ -ffp-contract=off, glibc libm); the oracle and "
                     "the numpy restatement agree bit for bit",
           "cases": cases}
    (OUT / "philox.json").write_text(json.dumps(doc, indent=0) + "\n")
    print(f"wrote {OUT / 'philox.json'} ({len(cases)} cases)")


if __name__ == "__main__":
    main()
