"""Compiles the CPU oracle into oracle/_build/liboracle.so (test infrastructure only).

g++ with -ffp-contract=off so that each float operation of the restated code
rounds on its own, and std::thread for the multi-core CPU baseline.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "liboracle.so"
FLAGS = ["-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
         "-pthread", "-Wall"]


def build(force: bool = False) -> Path:
    srcs = sorted(HERE.glob("*.cpp"))
    deps = srcs + sorted(HERE.glob("*.h"))
    if (not force and OUT.exists()
            and OUT.stat().st_mtime >= max(p.stat().st_mtime for p in deps)):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cxx = os.environ.get("CXX", "g++")
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [cxx, *FLAGS, *map(str, srcs), "-o", str(tmp)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{' '.join(cmd)}\n{proc.stderr}")
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
