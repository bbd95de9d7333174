"""Generates the committed golden vectors under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

Philox goldens are produced twice, independently: by the C++ oracle
(oracle/philox.cpp, a restatement of libraries/rand/src/curand_context.mm:42-185)
and by the vectorised numpy restatement below; the script refuses to write a
file unless both agree bit for bit.  The reference itself cannot run here (it
builds only on macOS with Metal), so these files pin the oracle against drift
and give the GPU tests fixed expected values.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402

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
    cases = []
    # (seed, offset, n): config seed, reference test seeds, tails, odd offsets,
    # a counter that crosses 2^32 and a 64-bit seed.
    for seed, offset, n in [
        (1234, 0, 64), (1234, 4, 64), (1234, 1024, 64), (1234, 1 << 30, 64),
        (42, 0, 67), (777, 1024, 33), (9999, 6, 19), (12345, 0, 16),
        (0xDEADBEEFCAFEF00D, (1 << 34) - 8, 40), (0, 0, 8),
    ]:
        words, nxt = oracle.generate_uint(seed, offset, n)
        ref = stream_numpy(seed, offset, n)
        if not np.array_equal(words, ref):
            raise SystemExit(f"oracle and numpy restatement disagree at seed={seed} offset={offset}")
        uni, _ = oracle.generate_uniform(seed, offset, n)
        if not np.array_equal(uni.view(np.uint32), uniform_numpy(ref).view(np.uint32)):
            raise SystemExit(f"uniform disagreement at seed={seed} offset={offset}")
        nor, _ = oracle.generate_normal(seed, offset, n, 0.0, 1.0)
        cases.append({
            "seed": seed, "offset": offset, "n": n, "next_offset": nxt,
            "uint": [int(v) for v in words],
            "uniform_bits": [int(v) for v in uni.view(np.uint32)],
            "normal": [float(v) for v in nor],
        })
    (OUT / "philox.json").write_text(json.dumps({"cases": cases}, indent=0) + "\n")
    print(f"wrote {OUT / 'philox.json'} ({len(cases)} cases)")


if __name__ == "__main__":
    main()
