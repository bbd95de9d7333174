"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

Every random number comes from this library's own Philox4x32-10 generator
(``curandGenerateUniform`` / ``curandGenerateNormal`` through the C ABI), so an
input is fixed by (seed, offset) and can be regenerated bit for bit.  No dataset
is involved: the reference's configurations are all synthetic.
"""

from __future__ import annotations

import ctypes as C
import math

from muda_b200 import capi


def _gen(torch, seed: int, offset: int):
    L = capi.curand()
    g = C.c_void_p()
    assert L.curandCreateGenerator(C.byref(g), capi.CURAND_RNG_PSEUDO_PHILOX4_32_10) == 0
    assert L.curandSetPseudoRandomGeneratorSeed(g, seed) == 0
    assert L.curandSetGeneratorOffset(g, offset) == 0
    assert L.curandSetStream(g, C.c_void_p(int(torch.cuda.current_stream().cuda_stream))) == 0
    return L, g


def uniform(torch, n: int, seed: int, offset: int = 0):
    """n draws in (0, 1] starting at generator offset `offset`."""
    L, g = _gen(torch, seed, offset)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    try:
        assert L.curandGenerateUniform(g, C.c_void_p(out.data_ptr()), n) == 0
    finally:
        assert L.curandDestroyGenerator(g) == 0
    return out


def uniform_pm1(torch, n: int, seed: int, offset: int = 0):
    """Uniform[-1, 1): 2u - 1 of the Philox uniform stream."""
    return uniform(torch, n, seed, offset).mul_(2.0).sub_(1.0)


def normal(torch, n: int, seed: int, std: float = 1.0, mean: float = 0.0, offset: int = 0):
    L, g = _gen(torch, seed, offset)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    try:
        assert L.curandGenerateNormal(g, C.c_void_p(out.data_ptr()), n, C.c_float(mean),
                                      C.c_float(std)) == 0
    finally:
        assert L.curandDestroyGenerator(g) == 0
    return out


def _round4(n: int) -> int:
    return (n + 3) // 4 * 4


def powerlaw_csr(torch, rows: int, cols: int, *, seed: int = 7, exponent: float = 2.0,
                 kmin: float = 2.2, kmax: int = 4096):
    """CSR matrix with power-law row lengths.

    Row length k = floor of a continuous power law p(k) ~ k^-exponent on
    [kmin, kmax] (kmin 2.2 gives a mean of about 16 entries per row), clamped to
    [2, min(kmax, cols)]; columns uniform in [0, cols), sorted within each row
    (duplicates are rare and kept: CSR allows them); values and x uniform[-1, 1).
    Draw order on the seed's stream: row lengths, columns, values, x.
    """
    off = 0
    u = uniform(torch, rows, seed, off).double()
    off += _round4(rows)
    a = 1.0 - exponent
    lo, hi = kmin ** a, float(kmax) ** a
    k = torch.floor((lo + u * (hi - lo)) ** (1.0 / a))
    k = k.clamp_(2, min(kmax, cols)).to(torch.int64)
    nnz = int(k.sum().item())
    row_offsets = torch.zeros(rows + 1, dtype=torch.int64, device="cuda")
    row_offsets[1:] = torch.cumsum(k, 0)
    uc = uniform(torch, nnz, seed, off)
    off += _round4(nnz)
    col = torch.clamp((uc.double() * cols).to(torch.int64), max=cols - 1)
    del uc
    row_id = torch.repeat_interleave(torch.arange(rows, device="cuda"), k)
    key = row_id * cols + col
    del row_id, col
    key, _ = torch.sort(key)
    col_ind = (key % cols).to(torch.int32)
    del key
    values = uniform_pm1(torch, nnz, seed, off)
    off += _round4(nnz)
    x = uniform_pm1(torch, cols, seed, off)
    return {"row_offsets": row_offsets.to(torch.int32), "col_ind": col_ind, "values": values,
            "x": x, "rows": rows, "cols": cols, "nnz": nnz}


def powerlaw_mean(exponent: float = 2.0, kmin: float = 2.2, kmax: int = 4096) -> float:
    """Mean of the continuous law before flooring (for documentation)."""
    if exponent == 2.0:
        return math.log(kmax / kmin) / (1.0 / kmin - 1.0 / kmax)
    a = 1.0 - exponent
    b = 2.0 - exponent
    return (a / b) * (kmax ** b - kmin ** b) / (kmax ** a - kmin ** a)
