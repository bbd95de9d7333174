"""Builds the five C-ABI shared libraries for sm_100a.

Each library is compiled from its own sources under ``muda_b200/csrc`` and
linked into ``muda_b200/lib/libmuda_<name>.so`` with the CUDA runtime linked
statically, so the files run wherever the driver is present.  Objects go to
``muda_b200/_build``; a source is recompiled when it, or any header of the
package or of ``include/``, is newer than its object.

Run ``python -m muda_b200.build`` (or ``__graft_entry__.build()``).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

# library name -> sources relative to csrc/
LIBS: dict[str, list[str]] = {
    "curand": ["rand/curand_api.cpp", "rand/philox_kernels.cu"],
    "cudnn": ["dnn/cudnn_api.cpp", "dnn/softmax_kernels.cu", "dnn/conv_direct_kernels.cu",
              "dnn/conv_tc_kernels.cu", "dnn/conv_dispatch.cu", "blas/tf32_split.cu",
              "dnn/dnn_ops_kernels.cu", "dnn/conv_bwd_tc.cu", "blas/gemm_tc_kernels.cu"],
    "cusparse": ["sparse/cusparse_api.cpp", "sparse/spmv_kernels.cu",
                 "sparse/spmm_kernels.cu"],
    "cufft": ["fft/cufft_api.cpp", "fft/stockham_kernels.cu", "fft/dft_kernels.cu",
              "fft/bluestein_kernels.cu", "fft/mixed_kernels.cu",
              "fft/fft_static.cu", "fft/real_kernels.cu"],
    "peer": ["peer/peer_exchange.cu"],
    "probe": ["probe/gather_probe.cu", "probe/normal_probe.cu"],
    "cublas": ["blas/cublas_api.cpp", "blas/gemm_simt_kernels.cu", "blas/gemm_tc_kernels.cu",
               "blas/tf32_split.cu", "blas/level12_kernels.cu",
               "blas/geam_kernels.cu", "blas/dblas_kernels.cu"],
}

COMMON_FLAGS = ["-O3", "-std=c++17", f"-I{INCLUDE}", f"-I{CSRC}"]
HOST_FLAGS = ["-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra", "-Wno-unused-parameter"]


def _headers() -> list[Path]:
    return list(CSRC.rglob("*.hpp")) + list(CSRC.rglob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _compile_cmd(src: Path, obj: Path) -> list[str]:
    host = ",".join(HOST_FLAGS)
    if src.suffix == ".cu":
        return [NVCC, *ARCH, "-lineinfo", *COMMON_FLAGS, "-Xcompiler", host,
                "-Xptxas", "-warn-spills", "-c", str(src), "-o", str(obj)]
    return [CXX, *COMMON_FLAGS, f"-I{CUDA_HOME / 'include'}", *HOST_FLAGS, "-c", str(src), "-o", str(obj)]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n"
                           f"{proc.stdout}\n{proc.stderr}")
    if proc.stderr.strip():
        sys.stderr.write(proc.stderr)


def lib_path(name: str) -> Path:
    return LIBDIR / f"libmuda_{name}.so"


def build(names: list[str] | None = None, jobs: int | None = None, verbose: bool = False) -> list[Path]:
    """Compiles and links the requested libraries (default: all); returns their paths."""
    if shutil.which(NVCC) is None and not Path(NVCC).exists():
        raise RuntimeError(f"nvcc not found at {NVCC}")
    names = list(LIBS) if names is None else names
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)

    jobs_list: dict[Path, Path] = {}  # object -> source (a source shared by two libraries builds once)
    objs: dict[str, list[Path]] = {}
    for name in names:
        objs[name] = []
        for rel in LIBS[name]:
            src = CSRC / rel
            obj = BUILD / (rel.replace("/", "__") + ".o")
            objs[name].append(obj)
            stale = (not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime
                     or obj.stat().st_mtime < newest_header)
            if stale:
                jobs_list[obj] = src

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        futs = [pool.submit(_run, _compile_cmd(s, o)) for o, s in jobs_list.items()]
        for f in futs:
            f.result()
    if verbose and jobs_list:
        print(f"compiled {len(jobs_list)} source(s)")

    out = []
    for name in names:
        so = lib_path(name)
        newest_obj = max(o.stat().st_mtime for o in objs[name])
        if not so.exists() or so.stat().st_mtime < newest_obj:
            _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(so),
                  *[str(o) for o in objs[name]], "-Xlinker", "-Bsymbolic"])
        out.append(so)
    return out


if __name__ == "__main__":
    for p in build(sys.argv[1:] or None, verbose=True):
        print(p)
