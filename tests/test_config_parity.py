"""Parity at the benchmark configurations themselves, with the benchmark's own inputs.

The inputs come from muda_b200.synth exactly as bench.py draws them (the
library's Philox stream, seeds and distributions of the configs), and the
results are checked against the oracle restatements of the reference kernels:

* SGEMM fp32 1024^3, A and B uniform[-1, 1] from one seed-0 stream
  (A first), called as the row-major caller does, cublasSgemm(N, N, n, m, k, B, A):
  every entry within 1e-5 of (|A||B|)_ij of the double-precision product and the
  oracle's sequential-fma result (cublas_kernels.metal:969-1006), normwise 1e-5.
* bf16 GEMM M = N = K = 8192, batch 8, normal(0, 0.02) seed 11 (A then
  B), fp32 accumulate: 16384 sampled (batch, i, j) entries against the oracle's
  bf16 restatement (cublas_kernels.metal:1008-1045 with bf16 storage), per entry
  within 1e-2 relative (plus 1e-4 absolute for entries that cancel to ~0),
  normwise 1e-2 against the double-accumulated product.  Both operand layouts a
  caller can use for the config are run: T,N (both K-major) and N,N (the
  column-major call a row-major caller makes).
"""

import ctypes as C

import numpy as np
import pytest

import oracle
from muda_b200 import capi, synth
from tests.helpers import stream_ptr

pytestmark = pytest.mark.gpu


def _normwise(got, want):
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def test_sgemm_config0_inputs(cuda, built):
    torch = cuda
    m = n = k = 1024
    a = synth.uniform_pm1(torch, m * k, seed=0)
    b = synth.uniform_pm1(torch, k * n, seed=0, offset=(m * k + 3) // 4 * 4)
    c = torch.full((m * n,), 7.0, dtype=torch.float32, device="cuda")  # beta = 0: not read
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(stream_ptr(torch))) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    st = L.cublasSgemm_v2(h, 0, 0, n, m, k, C.byref(one), C.c_void_p(b.data_ptr()), n,
                          C.c_void_p(a.data_ptr()), k, C.byref(zero), C.c_void_p(c.data_ptr()), n)
    torch.cuda.synchronize()
    assert L.cublasDestroy_v2(h) == 0
    assert st == 0
    A = a.cpu().numpy()
    B = b.cpu().numpy()
    got = c.cpu().numpy().reshape(m, n).astype(np.float64)  # row-major C = A B
    Ar = A.reshape(m, k).astype(np.float64)
    Br = B.reshape(k, n).astype(np.float64)
    want = Ar @ Br
    scale = np.abs(Ar) @ np.abs(Br)
    assert np.all(np.abs(got - want) <= 1e-5 * scale), float((np.abs(got - want) / scale).max())
    assert _normwise(got, want) <= 1e-5
    seq = oracle.gemm("f32", False, False, n, m, k, 1.0, B, n, A, k, 0.0,
                      np.zeros(m * n, np.float32), n).reshape(m, n).astype(np.float64)
    assert np.all(np.abs(got - seq) <= 1e-5 * scale)


@pytest.mark.parametrize("layout", ["TN", "NN"])
def test_bf16_gemm_config4_sampled(cuda, built, layout):
    torch = cuda
    m = n = k = 8192
    batch = 8
    a = synth.normal(torch, m * k * batch, seed=11, std=0.02).to(torch.bfloat16)
    b = synth.normal(torch, n * k * batch, seed=11, std=0.02,
                     offset=(m * k * batch + 3) // 4 * 4).to(torch.bfloat16)
    c = torch.empty(m * n * batch, dtype=torch.bfloat16, device="cuda")
    ta = 1 if layout == "TN" else 0
    lda = k if ta else m
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, C.c_void_p(stream_ptr(torch))) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    st = L.cublasGemmStridedBatchedEx(
        h, ta, 0, m, n, k, C.byref(one), C.c_void_p(a.data_ptr()), capi.CUDA_R_16BF, lda, m * k,
        C.c_void_p(b.data_ptr()), capi.CUDA_R_16BF, k, n * k, C.byref(zero),
        C.c_void_p(c.data_ptr()), capi.CUDA_R_16BF, m, m * n, batch, capi.CUBLAS_COMPUTE_32F, -1)
    torch.cuda.synchronize()
    assert L.cublasDestroy_v2(h) == 0
    assert st == 0
    rng = np.random.default_rng(4)
    ne = 16384
    zb = rng.integers(0, batch, ne)
    rows = rng.integers(0, m, ne).astype(np.int32)
    cols = rng.integers(0, n, ne)
    ent_cols = (zb * n + cols).astype(np.int32)
    flat = torch.from_numpy(zb * m * n + cols * m + rows).cuda()
    got = oracle.bf16_to_f32(c[flat].view(torch.int16).cpu().numpy().view(np.uint16))
    del c
    A = a.view(torch.int16).cpu().numpy().view(np.uint16)
    B = b.view(torch.int16).cpu().numpy().view(np.uint16)
    del a, b
    torch.cuda.empty_cache()
    kw = dict(stride_a=m * k, stride_b=n * k, stride_c=m * n, batch=batch,
              entries=(rows, ent_cols), threads=16)
    want = oracle.gemm("bf16", bool(ta), False, m, n, k, 1.0, A, lda, B, k, 0.0,
                       np.zeros(m * n * batch, np.uint16), m, **kw)
    want = oracle.bf16_to_f32(want[(zb * m * n + cols * m + rows)]).astype(np.float64)
    got = got.astype(np.float64)
    err = np.abs(got - want)
    assert np.all(err <= 1e-2 * np.abs(want) + 1e-4), float(err.max())
    # double-accumulated product of the same bf16 operands, for the normwise bar
    Af = oracle.bf16_to_f32(A)
    Bf = oracle.bf16_to_f32(B)
    exact = np.empty(ne)
    for t in range(ne):
        z, i, j = int(zb[t]), int(rows[t]), int(cols[t])
        if ta:
            arow = Af[z * m * k + i * k: z * m * k + (i + 1) * k]
        else:
            arow = Af[z * m * k + i: (z + 1) * m * k: m]
        exact[t] = np.dot(arow.astype(np.float64),
                          Bf[z * n * k + j * k: z * n * k + (j + 1) * k].astype(np.float64))
    assert _normwise(got, exact) <= 1e-2
    print(f"bf16 {layout} 8192^3 x 8: max |err| vs oracle {err.max():.3e}, "
          f"normwise vs f64 {_normwise(got, exact):.3e}")
