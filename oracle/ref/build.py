"""Compiles the reference's own host Philox generator into oracle/_ref/ (test infrastructure).

Recipe: the reference file ``libraries/rand/src/curand_context.mm`` is compiled
unmodified, as C++ (``g++ -x c++``), straight from the reference tree.  Its
host generators (``PhiloxHostStep`` and ``GenerateHost*``, lines 42-293) are
plain C++; the file's only Objective-C dependencies are two framework imports and
a pipeline lookup returning ``id<MTLComputePipelineState>``, which the
compile-only headers in ``oracle/ref/stubs/`` satisfy without touching any
generator.  The reference's own headers come from the reference tree too:
``curand_context.hpp``, ``curand.h``, ``handle_table.hpp`` and its
``cuda_runtime.h``.  ``oracle/ref/shim.cpp`` adds C entry points.

The result, ``oracle/_ref/libcurand_ref.so``, is built only where the reference
tree exists (``MUDA_REFERENCE_ROOT``, else BASELINE.json's ``reference_path``);
elsewhere a previously built library is used as is.  Nothing is copied out of the
reference tree: the compiler reads it in place, and only the shared library is
written (into ``oracle/_ref/``, which git ignores).

Flags follow the reference's host semantics: ``-O2 -ffp-contract=off
-fno-fast-math`` so that every float operation rounds on its own, as a
non-contracting compile of the reference does.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE = HERE.parent
ROOT = ORACLE.parent
OUT = ORACLE / "_ref" / "libcurand_ref.so"

REF_SOURCE = "libraries/rand/src/curand_context.mm"
REF_INCLUDES = ["libraries/rand/include", "libraries/rand/src", "runtime/src", "runtime/include"]
FLAGS = ["-O2", "-std=c++20", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
         "-pthread", "-Wno-deprecated", "-w"]


def reference_root() -> Path | None:
    env = os.environ.get("MUDA_REFERENCE_ROOT")
    if env:
        p = Path(env)
    else:
        try:
            p = Path(json.loads((ROOT / "BASELINE.json").read_text())["reference_path"])
        except (OSError, KeyError, ValueError):
            return None
    return p if (p / REF_SOURCE).is_file() else None


def command(ref: Path, out: Path) -> list[str]:
    cxx = os.environ.get("CXX", "g++")
    incs = [f"-I{HERE / 'stubs'}"] + [f"-I{ref / d}" for d in REF_INCLUDES]
    defs = ['-DMUDA_CURAND_METALLIB_PATH="unused"', '-DMUDA_CURAND_METAL_SOURCE_PATH="unused"']
    return [cxx, *FLAGS, *incs, *defs, "-x", "c++", str(ref / REF_SOURCE), "-x", "none",
            str(HERE / "shim.cpp"), "-o", str(out)]


def build(force: bool = False) -> Path | None:
    """Builds the library when the reference tree is present; returns its path, or
    None when neither the tree nor a previous build exists."""
    ref = reference_root()
    if ref is None:
        return OUT if OUT.exists() else None
    deps = [ref / REF_SOURCE, HERE / "shim.cpp", *HERE.glob("stubs/**/*.h*"), Path(__file__)]
    if (not force and OUT.exists()
            and OUT.stat().st_mtime >= max(p.stat().st_mtime for p in deps)):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = command(ref, tmp)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"reference build failed:\n{' '.join(cmd)}\n{proc.stderr}")
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
