"""Benchmark of the B200 hot path (one JSON line on rank 0).

Headline workload: Philox4x32-10
``curandGenerateUniform`` of 2^30 fp32 followed by ``curandGenerateNormal`` of
2^30 fp32 (mean 0, std 1) on the same generator and stream, seed 1234, offset 0.
One step = both calls.  ``value`` is bytes written by all ranks per second
(GB/s, 1e9), with the output already resident in HBM; ``e2e`` is the same
metric through the host-generator C-ABI call into pinned host arrays, the
device-to-host copies inside the timed region.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): each rank draws
its own disjoint counter range of one global stream (rank r starts at generator
offset r * 2 * 2^30 words), so per-GPU work is fixed and there is no collective
on the data path ("scaling": "weak").  Timing is on the device with CUDA events,
barrier + synchronize on both sides, max over ranks.

``--impl reference`` times the reference's CPU path for the same workload: its own
host generator (libraries/rand/src/curand_context.mm, compiled unmodified into
oracle/_ref by oracle/ref/build.py) on all host cores, one generator per thread
on consecutive Philox-block slices of each call (the oracle restatement
oracle/philox.cpp where that library is absent).  N > 1 adds the strong-scaling
split of the same two calls and the multi-GPU paths of the other routines
(batch-sharded FFT / GEMM / conv / softmax and the row-block SpMV with its x
exchange); the final line carries a compact summary of every routine, the full
per-routine records go to stderr, one JSON line each.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_WORDS = 1 << 30          # per call, per rank
SEED = 1234
BYTES_PER_CALL = 4 * N_WORDS
BYTES_PER_STEP = 2 * BYTES_PER_CALL
METRIC = ("RNG HBM GB/s: Philox4x32-10 curandGenerateUniform + curandGenerateNormal, "
          "2^30 fp32 each, seed 1234")
UNIT = "GB/s"
CPU_SAMPLE_WORDS = 1 << 30  # per call: the full config size (about 1.3 s on 16 host cores)


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        out = {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
        for key in ("bf16_tflops", "bf16_tflops_sustained"):
            if key in d:
                out[key] = float(d[key])
        return out
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def _traffic_record() -> dict | None:
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from muda_b200 import capi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    L = capi.curand()
    stream = torch.cuda.Stream()
    sp = C.c_void_p(int(stream.cuda_stream))
    gen = C.c_void_p()
    assert L.curandCreateGenerator(C.byref(gen), capi.CURAND_RNG_PSEUDO_PHILOX4_32_10) == 0
    assert L.curandSetPseudoRandomGeneratorSeed(gen, SEED) == 0
    from muda_b200.partition import rng_rank_offset
    base_offset = rng_rank_offset(rank, N_WORDS)
    assert L.curandSetGeneratorOffset(gen, base_offset) == 0
    assert L.curandSetStream(gen, sp) == 0

    uni = torch.empty(N_WORDS, dtype=torch.float32, device="cuda")
    nor = torch.empty(N_WORDS, dtype=torch.float32, device="cuda")
    pu, pn = C.c_void_p(uni.data_ptr()), C.c_void_p(nor.data_ptr())

    def step(ev=None):
        # each step redraws the same 2^31 words of this rank's counter range
        assert L.curandSetGeneratorOffset(gen, base_offset) == 0
        if ev is not None:
            ev[0].record(stream)
        assert L.curandGenerateUniform(gen, pu, N_WORDS) == 0
        if ev is not None:
            ev[1].record(stream)
        assert L.curandGenerateNormal(gen, pn, N_WORDS, C.c_float(0.0), C.c_float(1.0)) == 0
        if ev is not None:
            ev[2].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        t0.record(stream)
        for k in range(args.steps):
            step(evs[k])
        t1.record(stream)
        barrier()
    ms = t0.elapsed_time(t1)
    uni_ms = [e[0].elapsed_time(e[1]) for e in evs]
    nor_ms = [e[1].elapsed_time(e[2]) for e in evs]
    ms_t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    # ---- end to end: host generator into pinned host arrays, D2H in the timed region
    e2e = None
    if not args.no_e2e:
        hgen = C.c_void_p()
        assert L.curandCreateGeneratorHost(C.byref(hgen), capi.CURAND_RNG_PSEUDO_PHILOX4_32_10) == 0
        assert L.curandSetPseudoRandomGeneratorSeed(hgen, SEED) == 0
        assert L.curandSetStream(hgen, sp) == 0
        hu = torch.empty(N_WORDS, dtype=torch.float32, pin_memory=True)
        hn = torch.empty(N_WORDS, dtype=torch.float32, pin_memory=True)
        e_steps = max(1, min(args.steps, 3))

        def estep():
            assert L.curandSetGeneratorOffset(hgen, base_offset) == 0
            assert L.curandGenerateUniform(hgen, C.c_void_p(hu.data_ptr()), N_WORDS) == 0
            assert L.curandGenerateNormal(hgen, C.c_void_p(hn.data_ptr()), N_WORDS,
                                          C.c_float(0.0), C.c_float(1.0)) == 0
        estep()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e_steps):
            estep()
        e1.record(stream)
        barrier()
        et = torch.tensor([e0.elapsed_time(e1)], device="cuda")
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e_ms = float(et.item()) / e_steps
        e2e = {"value": world * BYTES_PER_STEP / (e_ms * 1e-3) / 1e9, "unit": UNIT,
               "ms_per_step": e_ms, "h2d_bytes_per_step": 0,
               "d2h_bytes_per_step": BYTES_PER_STEP,
               "path": "curandCreateGeneratorHost -> curandGenerateUniform/Normal into pinned host arrays"}
        assert L.curandDestroyGenerator(hgen) == 0
        del hu, hn

    # ---- CPU baseline (rank 0, N=1 only): the oracle port on all host cores, bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline()

    # ---- strong scaling of the same workload (N > 1): the config's two 2^30-word calls
    # split over the ranks, rank r drawing words [r n/N, (r+1) n/N) of each call
    strong = None
    if world > 1:
        part = N_WORDS // world
        ps = [torch.cuda.Event(enable_timing=True) for _ in range(2)]

        def sstep():
            assert L.curandSetGeneratorOffset(gen, rank * part) == 0
            assert L.curandGenerateUniform(gen, pu, part) == 0
            assert L.curandSetGeneratorOffset(gen, N_WORDS + rank * part) == 0
            assert L.curandGenerateNormal(gen, pn, part, C.c_float(0.0), C.c_float(1.0)) == 0
        for _ in range(args.warmup):
            sstep()
        barrier()
        ps[0].record(stream)
        for _ in range(args.steps):
            sstep()
        ps[1].record(stream)
        barrier()
        st_ms = torch.tensor([ps[0].elapsed_time(ps[1]) / args.steps], device="cuda")
        dist.all_reduce(st_ms, op=dist.ReduceOp.MAX)
        strong = {"value": BYTES_PER_STEP / (float(st_ms.item()) * 1e-3) / 1e9, "unit": UNIT,
                  "ms_per_step": float(st_ms.item()), "scaling": "strong",
                  "partition": f"the config's 2 x 2^30 words split {world} ways by counter range"}

    assert L.curandDestroyGenerator(gen) == 0
    del uni, nor
    torch.cuda.empty_cache()
    suite = None
    if args.suite != "none":
        if world == 1:
            names = list(SUITE) if args.suite == "all" else args.suite.split(",")
            suite = run_suite(names, args, torch)
        else:
            names = list(SHARDED) + ["spmv_dist"] if args.suite == "all" else \
                args.suite.split(",")
            suite = run_suite_sharded(names, args, torch, dist, world, rank, local)
    if rank == 0 and suite:
        for name, res in suite.items():  # full per-routine records, one JSON line each
            print(json.dumps({"routine": name, **res}), file=sys.stderr, flush=True)
    if rank == 0:
        peaks = _peaks()
        mu, mn = statistics.mean(uni_ms), statistics.mean(nor_ms)
        dom_name, dom_ms = ("philox_fill<normal>", mn) if mn >= mu else ("philox_fill<uniform>", mu)
        achieved = BYTES_PER_CALL / (dom_ms * 1e-3) / 1e9
        traffic = None
        rec = _traffic_record()
        if rec and dom_name in rec.get("kernels", {}):
            traffic = rec["kernels"][dom_name].get("dram_bytes_per_launch_scaled")
        line = {
            "metric": METRIC, "value": world * BYTES_PER_STEP / (ms_max / args.steps * 1e-3) / 1e9,
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u32->f32", "data": "synthetic (counter-based RNG output)",
            "config": {"workload": "configs[1]: Philox4x32-10 uniform 2^30 + normal(0,1) 2^30, "
                                   "seed 1234, offset 0, same generator and stream",
                       "words_per_call": N_WORDS, "bytes_per_step_per_gpu": BYTES_PER_STEP,
                       "partition": "rank r draws counters [r*2^29, (r+1)*2^29) (offset r*2^31)",
                       "l2": "output 4.3 GB per call > 126 MB L2 (no flush needed)"},
            "per_call_ms": {"uniform": mu, "normal": mn},
            "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": achieved,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "peak_source": peaks["source"], "traffic": traffic,
                         "algorithmic_bytes_per_launch": BYTES_PER_CALL},
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
            "e2e": e2e,
            "cpu_baseline": cpu,
            "strong": strong,
            "suite_summary": summarize(suite),
            "suite_summary_fields": ["value", "unit", "roofline frac (of measured)", "ms per call"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------------------------ suite --
# Every other hot-path routine at its BASELINE.json configuration, device-resident
# inputs, CUDA events around each call on the library stream (max over steps is
# not used: mean of the timed calls).  Workloads whose inputs fit in L2 flush it
# (a 256 MB write) before every timed call, outside the events.

L2_FLUSH_BYTES = 256 << 20


class Suite:
    def __init__(self, torch, steps, warmup, cpu, scale=1):
        self.torch = torch
        self.steps = steps
        self.warmup = warmup
        self.cpu = cpu
        self.scale = scale
        self.stream = torch.cuda.Stream()
        self.sp = C.c_void_p(int(self.stream.cuda_stream))
        self.peaks = _peaks()
        self._flush = None
        self.e2e = True         # time the host-buffer legs (bench.py --no-e2e turns them off)
        self.shard = 1          # ranks sharing a batch-sharded workload (its 1/shard per rank)
        self.barrier = None     # called around the timed region under torchrun

    def flush(self):
        """Evicts L2 by writing a buffer twice its size (outside the timed region)."""
        if self._flush is None:
            self._flush = self.torch.empty(L2_FLUSH_BYTES // 4, dtype=torch_float(self.torch),
                                           device="cuda")
        with self.torch.cuda.stream(self.stream):
            self._flush.fill_(1.0)

    def time(self, fn, flush=False, launches_per_call=1):
        torch = self.torch
        if self.barrier is not None:
            self.barrier()
        with torch.cuda.stream(self.stream):
            for _ in range(self.warmup):
                fn()
            ms = []
            for _ in range(self.steps):
                if flush:
                    self.flush()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(self.stream)
                fn()
                e1.record(self.stream)
                ms.append((e0, e1))
            self.stream.synchronize()
        if self.barrier is not None:
            self.barrier()
        t = [a.elapsed_time(b) for a, b in ms]
        return statistics.mean(t), launches_per_call * self.steps

    def roof(self, kernel, achieved, bound):
        if bound == "hbm":
            peak, unit = self.peaks["hbm_gbs"], "GB/s"
        elif bound == "tensor":
            peak, unit = self.peaks.get("bf16_tflops", 1651.6), "TFLOP/s"
        elif bound == "tensor-tf32x3":
            # fp32 work done as three tf32 MMAs per product: tf32 runs at half the bf16
            # rate, so the ceiling for fp32 FLOP/s is bf16 / 2 / 3
            peak, unit = self.peaks.get("bf16_tflops", 1651.6) / 6.0, "TFLOP/s"
        elif bound == "fp64":  # DFMA pipe at the maximum SM clock
            peak, unit = DFMA_PEAK_TFLOPS, "TFLOP/s"
        else:  # fp32 FFMA pipe at the maximum SM clock
            peak, unit = FFMA_PEAK_TFLOPS, "TFLOP/s"
        source = {"ffma": "148 SMs x 128 FMA x 2 x 1965 MHz",
                  "fp64": "148 SMs x 64 DFMA x 2 x 1965 MHz (nominal)",
                  "tensor-tf32x3": self.peaks["source"] + " bf16 GEMM / 2 (tf32 rate) / 3 (MMAs "
                                   "per fp32 product)"}.get(bound, self.peaks["source"])
        out = {"bound": bound, "kernel": kernel, "achieved": achieved, "peak": peak,
               "unit": unit, "frac": achieved / peak, "peak_source": source}
        if bound == "tensor-tf32x3":
            out["frac_of_ffma_peak"] = achieved / FFMA_PEAK_TFLOPS
        return out


FFMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
DFMA_PEAK_TFLOPS = 148 * 64 * 2 * 1.965e9 / 1e12


def torch_float(torch):
    return torch.float32


def cpu_time(fn):
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


def suite_sgemm(s: Suite) -> dict:
    """SGEMM fp32 row-major C = A*B, M = N = K = 1024, alpha 1, beta 0,
    A/B uniform[-1, 1] seed 0, through cublasSgemm(N, N, n, m, k, B, A) (C^T = B^T A^T)."""
    from muda_b200 import capi, synth
    torch = s.torch
    m = n = k = 1024 // s.scale
    a = synth.uniform_pm1(torch, m * k, seed=0)
    b = synth.uniform_pm1(torch, k * n, seed=0, offset=(m * k + 3) // 4 * 4)
    c = torch.zeros(m * n, dtype=torch.float32, device="cuda")
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, s.sp) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    args = (h, 0, 0, n, m, k, C.byref(one), C.c_void_p(b.data_ptr()), n,
            C.c_void_p(a.data_ptr()), k, C.byref(zero), C.c_void_p(c.data_ptr()), n)
    ms, launches = s.time(lambda: L.cublasSgemm_v2(*args), flush=True)
    flop = 2.0 * m * n * k
    # end to end through the C ABI with host buffers: A and B copied in from pinned host
    # memory, the call, C copied back, all inside the timed region
    e2e = None
    if s.e2e:
        ha, hb = (t.cpu().pin_memory() for t in (a, b))
        hc = torch.empty(m * n, dtype=torch.float32, pin_memory=True)
        da, db, dc = torch.empty_like(a), torch.empty_like(b), torch.empty_like(c)
        e_args = (h, 0, 0, n, m, k, C.byref(one), C.c_void_p(db.data_ptr()), n,
                  C.c_void_p(da.data_ptr()), k, C.byref(zero), C.c_void_p(dc.data_ptr()), n)

        def e2e_call():
            da.copy_(ha, non_blocking=True)
            db.copy_(hb, non_blocking=True)
            assert L.cublasSgemm_v2(*e_args) == 0
            hc.copy_(dc, non_blocking=True)
        e_ms, _ = s.time(e2e_call, flush=True)
        e2e = {"value": flop / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": e_ms,
               "h2d_bytes_per_step": 4 * (m * k + k * n), "d2h_bytes_per_step": 4 * m * n,
               "path": "pinned host -> device copies of A and B, cublasSgemm_v2, device -> "
                       "pinned host copy of C"}
        del ha, hb, hc, da, db, dc
    # the FFMA kernel the same call runs under CUBLAS_PEDANTIC_MATH, for comparison
    assert L.cublasSetMathMode(h, capi.CUBLAS_PEDANTIC_MATH) == 0
    ms_ffma, _ = s.time(lambda: L.cublasSgemm_v2(*args), flush=True)
    assert L.cublasDestroy_v2(h) == 0
    tf = flop / (ms * 1e-3) / 1e12
    out = {"value": tf, "unit": "TFLOP/s", "ms": ms, "e2e": e2e,
           "dtype": "f32 (split-tf32 on tcgen05)",
           "config": f"{m}x{n}x{k} fp32, L2 flushed before each call; hi/lo split of A and B, "
                     "split-K GEMM, split-order reduction",
           "roofline": s.roof("tc_gemm_split_kernel<SplitGemmProblem<256>,256,2,2>", tf,
                              "tensor-tf32x3"),
           "launches": launches,
           "pedantic_ffma": {"ms": ms_ffma, "TFLOP/s": flop / (ms_ffma * 1e-3) / 1e12,
                             "frac_of_ffma_peak": flop / (ms_ffma * 1e-3) / 1e12 /
                             FFMA_PEAK_TFLOPS,
                             "kernel": "gemm_ffma_vec<false,false,stream-K> + "
                                       "ffma_stream_reduce"}}
    if s.cpu:
        import oracle
        A = a.cpu().numpy()
        B = b.cpu().numpy()
        Cm = np.zeros(m * n, np.float32)
        dt = cpu_time(lambda: oracle.gemm("f32", False, False, n, m, k, 1.0, B, n, A, k, 0.0, Cm,
                                          n, threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": flop / dt / 1e12, "unit": "TFLOP/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": "full problem, oracle/gemm.cpp sequential-fma loop"}
    return out


def suite_spmv(s: Suite) -> dict:
    """CSR SpMV 4M x 4M, power-law row lengths (mean ~16, max 4096), seed 7."""
    from muda_b200 import capi, synth
    torch = s.torch
    rows = (1 << 22) // s.scale
    mtx = synth.powerlaw_csr(torch, rows, rows, seed=7)
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    L = capi.cusparse()
    h, ma, vx, vy = (C.c_void_p() for _ in range(4))
    assert L.cusparseCreate(C.byref(h)) == 0
    assert L.cusparseSetStream(h, s.sp) == 0
    assert L.cusparseCreateCsr(C.byref(ma), rows, rows, mtx["nnz"],
                               C.c_void_p(mtx["row_offsets"].data_ptr()),
                               C.c_void_p(mtx["col_ind"].data_ptr()),
                               C.c_void_p(mtx["values"].data_ptr()), 2, 2, 0, 0) == 0
    assert L.cusparseCreateDnVec(C.byref(vx), rows, C.c_void_p(mtx["x"].data_ptr()), 0) == 0
    assert L.cusparseCreateDnVec(C.byref(vy), rows, C.c_void_p(y.data_ptr()), 0) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    ms, launches = s.time(lambda: L.cusparseSpMV(h, 0, C.byref(one), ma, vx, C.byref(zero), vy,
                                                 0, 0, None), flush=True)
    nnz = mtx["nnz"]
    alg_bytes = nnz * 8 + (rows + 1) * 4 + rows * 4 + rows * 4
    # end to end through the C ABI with host buffers: the CSR arrays and x copied in from
    # pinned host memory into the buffers a second descriptor names, the call, y copied
    # back, all inside the timed region
    e2e = None
    if s.shard == 1 and s.e2e:
        keys = ("row_offsets", "col_ind", "values", "x")
        host = {kk: mtx[kk].cpu().pin_memory() for kk in keys}
        dev = {kk: torch.empty_like(mtx[kk]) for kk in keys}
        hy = torch.empty(rows, dtype=torch.float32, pin_memory=True)
        dy = torch.empty_like(y)
        mb, ex, ey = C.c_void_p(), C.c_void_p(), C.c_void_p()
        assert L.cusparseCreateCsr(C.byref(mb), rows, rows, nnz,
                                   C.c_void_p(dev["row_offsets"].data_ptr()),
                                   C.c_void_p(dev["col_ind"].data_ptr()),
                                   C.c_void_p(dev["values"].data_ptr()), 2, 2, 0, 0) == 0
        assert L.cusparseCreateDnVec(C.byref(ex), rows, C.c_void_p(dev["x"].data_ptr()), 0) == 0
        assert L.cusparseCreateDnVec(C.byref(ey), rows, C.c_void_p(dy.data_ptr()), 0) == 0

        def e2e_call():
            for kk in keys:
                dev[kk].copy_(host[kk], non_blocking=True)
            assert L.cusparseSpMV(h, 0, C.byref(one), mb, ex, C.byref(zero), ey, 0, 0,
                                  None) == 0
            hy.copy_(dy, non_blocking=True)
        steps, warm = s.steps, s.warmup
        s.steps, s.warmup = 3, 1
        e_ms, _ = s.time(e2e_call)
        s.steps, s.warmup = steps, warm
        e2e = {"value": alg_bytes / (e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms": e_ms,
               "h2d_bytes_per_step": sum(host[kk].numel() * 4 for kk in keys),
               "d2h_bytes_per_step": rows * 4,
               "path": "pinned host -> device copies of row offsets, column indices, values "
                       "and x, cusparseSpMV, device -> pinned host copy of y"}
        for fn, d in (("cusparseDestroyDnVec", ex), ("cusparseDestroyDnVec", ey),
                      ("cusparseDestroySpMat", mb)):
            assert getattr(L, fn)(d) == 0
        del host, dev, hy, dy
    for fn, d in (("cusparseDestroyDnVec", vx), ("cusparseDestroyDnVec", vy),
                  ("cusparseDestroySpMat", ma)):
        assert getattr(L, fn)(d) == 0
    assert L.cusparseDestroy(h) == 0
    ceiling = gather_ceiling(s, mtx["x"], mtx["col_ind"], nnz)
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32/i32", "e2e": e2e,
           "config": f"{rows} rows, nnz {nnz} ({nnz / rows:.2f}/row), power law k^-2 on "
                     "[2.2, 4096], L2 flushed before each call",
           "reference_formula_gbs": (nnz * 8 + 2 * rows * 4) / (ms * 1e-3) / 1e9,
           "roofline": s.roof("spmv_csr_ranges", gbs, "hbm"), "launches": launches,
           "algorithmic_bytes_per_launch": alg_bytes,
           "gather_ceiling": {**ceiling, "spmv_gathers_per_s": nnz / (ms * 1e-3),
                              "spmv_frac_of_ceiling": ceiling["ms"] / ms}}
    if s.cpu:
        import oracle
        ro, ci, va, xx = (mtx[k].cpu().numpy() for k in ("row_offsets", "col_ind", "values", "x"))
        dt = cpu_time(lambda: oracle.spmv_csr(ro, ci, va, xx, threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": alg_bytes / dt / 1e9, "unit": "GB/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": "full problem, oracle/spmv.cpp thread-per-row loop"}
    return out


def gather_ceiling(s: Suite, x, col_ind, nnz: int) -> dict:
    """The matrix's own column stream read and its x gathered, nothing else
    (mb200ProbeGather): the least work of any CSR SpMV of this matrix.  Best of one
    and four indices per lane, 4 and 8 CTAs of 256 per SM."""
    from muda_b200 import capi
    P = capi.probe()
    sms = s.torch.cuda.get_device_properties(s.torch.cuda.current_device()).multi_processor_count
    best = None
    for per_lane in (1, 4):
        for ctas in (4, 8):
            grid = sms * ctas
            out = s.torch.empty(grid * 256, dtype=s.torch.float32, device="cuda")
            ms, _ = s.time(lambda: P.mb200ProbeGather(
                C.c_void_p(x.data_ptr()), C.c_void_p(col_ind.data_ptr()), nnz, per_lane,
                C.c_void_p(out.data_ptr()), grid, s.sp), flush=True)
            n_done = nnz if per_lane == 1 else nnz // 4 * 4
            rate = n_done / (ms * 1e-3)
            if best is None or rate > best["gathers_per_s"]:
                best = {"gathers_per_s": rate, "ms": nnz / rate * 1e3, "per_lane": per_lane,
                        "grid": grid}
    best["what"] = ("mb200ProbeGather: column indices streamed (evict-first) and x gathered "
                    "(L2-only), no values, rows or y")
    return best


def scatter_ceiling(s: Suite, y, col_ind, nnz: int) -> dict:
    """The matrix's own column stream read and 1.0 added to y[col] by reductions that
    return nothing (mb200ProbeScatter): the scatter of A^T x without its loads of values
    and x.  Best of one and four indices per lane, 4 and 8 CTAs of 256 per SM.  Leaves
    garbage in y."""
    from muda_b200 import capi
    P = capi.probe()
    sms = s.torch.cuda.get_device_properties(s.torch.cuda.current_device()).multi_processor_count
    best = None
    for per_lane in (1, 4):
        for ctas in (4, 8):
            grid = sms * ctas
            ms, _ = s.time(lambda: P.mb200ProbeScatter(
                C.c_void_p(y.data_ptr()), C.c_void_p(col_ind.data_ptr()), nnz, per_lane, grid,
                s.sp), flush=True)
            n_done = nnz if per_lane == 1 else nnz // 4 * 4
            rate = n_done / (ms * 1e-3)
            if best is None or rate > best["reductions_per_s"]:
                best = {"reductions_per_s": rate, "ms": nnz / rate * 1e3, "per_lane": per_lane,
                        "grid": grid}
    best["what"] = ("mb200ProbeScatter: column indices streamed (evict-first), 1.0 added to "
                    "y[col] by red.global.add.f32, no values or x")
    return best


def _csr_handle(L, s, mtx, rows, cols):
    h, ma = C.c_void_p(), C.c_void_p()
    assert L.cusparseCreate(C.byref(h)) == 0
    assert L.cusparseSetStream(h, s.sp) == 0
    assert L.cusparseCreateCsr(C.byref(ma), rows, cols, mtx["nnz"],
                               C.c_void_p(mtx["row_offsets"].data_ptr()),
                               C.c_void_p(mtx["col_ind"].data_ptr()),
                               C.c_void_p(mtx["values"].data_ptr()), 2, 2, 0, 0) == 0
    return h, ma


def suite_spmv_t(s: Suite) -> dict:
    """y = A^T x on the configs[2] matrix (4M x 4M power law, seed 7), beta 0."""
    from muda_b200 import capi, synth
    torch = s.torch
    rows = (1 << 22) // s.scale
    mtx = synth.powerlaw_csr(torch, rows, rows, seed=7)
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    L = capi.cusparse()
    h, ma = _csr_handle(L, s, mtx, rows, rows)
    vx, vy = C.c_void_p(), C.c_void_p()
    assert L.cusparseCreateDnVec(C.byref(vx), rows, C.c_void_p(mtx["x"].data_ptr()), 0) == 0
    assert L.cusparseCreateDnVec(C.byref(vy), rows, C.c_void_p(y.data_ptr()), 0) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    ms, launches = s.time(lambda: L.cusparseSpMV(h, 1, C.byref(one), ma, vx, C.byref(zero), vy,
                                                 0, 0, None), flush=True, launches_per_call=2)
    for fn, d in (("cusparseDestroyDnVec", vx), ("cusparseDestroyDnVec", vy),
                  ("cusparseDestroySpMat", ma)):
        assert getattr(L, fn)(d) == 0
    assert L.cusparseDestroy(h) == 0
    nnz = mtx["nnz"]
    alg_bytes = nnz * 8 + (rows + 1) * 4 + rows * 4 + rows * 4
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    ceiling = scatter_ceiling(s, y, mtx["col_ind"], nnz)
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32/i32",
           "config": f"A^T x, {rows} rows, nnz {nnz}, power law, L2 flushed before each call",
           "roofline": s.roof("spmv_t_scatter<4,float>", gbs, "hbm"), "launches": launches,
           "algorithmic_bytes_per_call": alg_bytes,
           "scatter_ceiling": {**ceiling, "spmv_t_reductions_per_s": nnz / (ms * 1e-3),
                               "spmv_t_frac_of_ceiling": ceiling["ms"] / ms}}
    if s.cpu:
        import oracle
        sample = max(1, rows // 16)
        ro = mtx["row_offsets"][: sample + 1].cpu().numpy()
        ci = mtx["col_ind"][: int(ro[-1])].cpu().numpy()
        va = mtx["values"][: int(ro[-1])].cpu().numpy()
        xx = mtx["x"][:sample].cpu().numpy()
        dt = cpu_time(lambda: oracle.spmv_csr_t(ro, ci, va, xx, rows))
        sb = int(ro[-1]) * 8 + (sample + 1) * 4 + sample * 4 + rows * 4
        out["cpu_baseline"] = {"value": sb / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
                               "sample": f"first {sample} rows, oracle/spmv.cpp row-order scatter"}
    return out


def suite_spmm(s: Suite) -> dict:
    """C = A B, A the power-law generator at 1M x 1M (seed 9), B and C row-major with 64
    columns (the float4 path), beta 0."""
    from muda_b200 import capi, synth
    torch = s.torch
    rows, n = (1 << 20) // s.scale, 64
    mtx = synth.powerlaw_csr(torch, rows, rows, seed=9)
    b = synth.uniform_pm1(torch, rows * n, seed=10)
    c = torch.zeros(rows * n, dtype=torch.float32, device="cuda")
    L = capi.cusparse()
    h, ma = _csr_handle(L, s, mtx, rows, rows)
    mb, mc = C.c_void_p(), C.c_void_p()
    assert L.cusparseCreateDnMat(C.byref(mb), rows, n, n, C.c_void_p(b.data_ptr()), 0,
                                 capi.CUSPARSE_ORDER_ROW) == 0
    assert L.cusparseCreateDnMat(C.byref(mc), rows, n, n, C.c_void_p(c.data_ptr()), 0,
                                 capi.CUSPARSE_ORDER_ROW) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    # two kernels a call: spmm_find_long (the long-row list) and spmm_rows_ring
    ms, launches = s.time(lambda: L.cusparseSpMM(h, 0, 0, C.byref(one), ma, mb, C.byref(zero), mc,
                                                 0, 0, None), flush=True, launches_per_call=2)
    for fn, d in (("cusparseDestroyDnMat", mb), ("cusparseDestroyDnMat", mc),
                  ("cusparseDestroySpMat", ma)):
        assert getattr(L, fn)(d) == 0
    assert L.cusparseDestroy(h) == 0
    nnz = mtx["nnz"]
    alg_bytes = nnz * 8 + (rows + 1) * 4 + 2 * rows * n * 4
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    # the row gathers alone (mb200ProbeRowGather on the matrix's own column indices)
    P = capi.probe()
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    best = None
    for ctas in (4, 8):
        grid = sms * ctas
        scratch = torch.empty(grid * 256, dtype=torch.float32, device="cuda")
        g_ms, _ = s.time(lambda: P.mb200ProbeRowGather(
            C.c_void_p(b.data_ptr()), C.c_void_p(mtx["col_ind"].data_ptr()), nnz,
            C.c_void_p(scratch.data_ptr()), grid, s.sp), flush=True)
        if best is None or g_ms < best["ms"]:
            best = {"ms": g_ms, "grid": grid, "row_bytes_per_s": nnz * n * 4 / (g_ms * 1e-3)}
    best["what"] = ("mb200ProbeRowGather: column indices streamed, row col of B (256 bytes) "
                    "gathered per entry with L2-only 16-byte loads, no values, no products, "
                    "no C")
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32/i32",
           "gflops": 2 * nnz * n / (ms * 1e-3) / 1e9,
           "row_gather_ceiling": {**best, "spmm_frac_of_ceiling": best["ms"] / ms},
           "config": f"{rows} rows, nnz {nnz}, N {n} row-major, L2 flushed before each call; "
                     "bytes = A + B + C once (B rows re-gathered per entry come through L2)",
           "roofline": s.roof("spmm_rows_ring<16>", gbs, "hbm"), "launches": launches,
           "algorithmic_bytes_per_call": alg_bytes}
    if s.cpu:
        import oracle
        sample = max(1, rows // 64)
        ro = mtx["row_offsets"][: sample + 1].cpu().numpy()
        ci = mtx["col_ind"][: int(ro[-1])].cpu().numpy()
        va = mtx["values"][: int(ro[-1])].cpu().numpy()
        bb = b.cpu().numpy()
        cc = np.zeros(sample * n, np.float32)
        dt = cpu_time(lambda: oracle.spmm_csr(ro, ci, va, rows, bb, n, 2, cc, n, 2, n,
                                              threads=os.cpu_count() or 1))
        sb = int(ro[-1]) * 8 + (sample + 1) * 4 + 2 * sample * n * 4
        out["cpu_baseline"] = {"value": sb / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(),
                               "kind": "port",
                               "sample": f"first {sample} rows, oracle/spmv.cpp per-output loop"}
    return out


class _DnnSetup:
    """cuDNN handle plus descriptors for the neighbour routines' benchmarks."""

    def __init__(self, s):
        from muda_b200 import capi
        self.L = capi.cudnn()
        self.h = C.c_void_p()
        assert self.L.cudnnCreate(C.byref(self.h)) == 0
        assert self.L.cudnnSetStream(self.h, s.sp) == 0
        self.owned = []

    def tensor(self, n, c, h, w, fmt=0):
        d = C.c_void_p()
        assert self.L.cudnnCreateTensorDescriptor(C.byref(d)) == 0
        assert self.L.cudnnSetTensor4dDescriptor(d, fmt, 0, n, c, h, w) == 0
        self.owned.append(("cudnnDestroyTensorDescriptor", d))
        return d

    def close(self):
        for fn, d in self.owned:
            assert getattr(self.L, fn)(d) == 0
        assert self.L.cudnnDestroy(self.h) == 0


def suite_conv_bwd(s: Suite) -> dict:
    """Backward data and backward filter of a 3x3 pad-1 fp32 convolution, NHWC x
    32x64x56x56, KRSC w 64x64x3x3 (the forward fp32 config's layouts), normal(0, 1)
    seeds 12-14."""
    from muda_b200 import synth
    torch = s.torch
    n, c, hw, k = 32 // s.scale, 64, 56, 64
    x = synth.normal(torch, n * c * hw * hw, seed=12)
    dy = synth.normal(torch, n * k * hw * hw, seed=13)
    w = synth.normal(torch, k * c * 9, seed=14)
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    d = _DnnSetup(s)
    L = d.L
    xd, yd = d.tensor(n, c, hw, hw, fmt=1), d.tensor(n, k, hw, hw, fmt=1)
    wd, cd = C.c_void_p(), C.c_void_p()
    assert L.cudnnCreateFilterDescriptor(C.byref(wd)) == 0
    assert L.cudnnSetFilter4dDescriptor(wd, 0, 1, k, c, 3, 3) == 0
    assert L.cudnnCreateConvolutionDescriptor(C.byref(cd)) == 0
    assert L.cudnnSetConvolution2dDescriptor(cd, 1, 1, 1, 1, 1, 1, 1, 0) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    p = lambda t: C.c_void_p(t.data_ptr())
    ms_d, ld = s.time(lambda: L.cudnnConvolutionBackwardData(
        d.h, C.byref(one), wd, p(w), yd, p(dy), cd, 0, None, 0, C.byref(zero), xd, p(dx)))
    ms_f, lf = s.time(lambda: L.cudnnConvolutionBackwardFilter(
        d.h, C.byref(one), xd, p(x), yd, p(dy), cd, 0, None, 0, C.byref(zero), wd, p(dw)),
        launches_per_call=2)
    assert L.cudnnDestroyFilterDescriptor(wd) == 0
    assert L.cudnnDestroyConvolutionDescriptor(cd) == 0
    d.close()
    flop = 2.0 * n * k * hw * hw * c * 9
    tf_d, tf_f = flop / (ms_d * 1e-3) / 1e12, flop / (ms_f * 1e-3) / 1e12
    return {"value": flop * 2 / ((ms_d + ms_f) * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms": ms_d + ms_f, "dtype": "f32",
            "config": f"N {n} C {c} K {k} {hw}x{hw} 3x3 pad 1, NHWC / KRSC",
            "backward_data": {"ms": ms_d, "TFLOP/s": tf_d,
                              "kernel": "transpose_filter + tc_gemm_split_kernel<ConvProblem>"},
            "backward_filter": {"ms": ms_f, "TFLOP/s": tf_f,
                                "kernel": "im2col + split-tf32 GEMM"},
            "roofline": s.roof("tc_gemm_split_kernel (backward data)", tf_d, "tensor-tf32x3"),
            "launches": ld + lf}


def suite_dnn_elementwise(s: Suite) -> dict:
    """ReLU over 2^28 fp32 (packed NCHW), max pooling 3x3 stride 2 pad 1 of
    32x64x112x112, batch-norm training of 32x64x56x56 (spatial, running averages)."""
    from muda_b200 import synth
    torch = s.torch
    out = {}
    d = _DnnSetup(s)
    L = d.L
    one, zero = C.c_float(1.0), C.c_float(0.0)
    p = lambda t: C.c_void_p(t.data_ptr())
    # activation
    n_act = (1 << 28) // s.scale
    x = synth.normal(torch, n_act, seed=15)
    y = torch.empty_like(x)
    td = d.tensor(n_act // (64 * 64 * 64), 64, 64, 64)
    act = C.c_void_p()
    assert L.cudnnCreateActivationDescriptor(C.byref(act)) == 0
    assert L.cudnnSetActivationDescriptor(act, 1, 0, 0.0) == 0
    ms, _ = s.time(lambda: L.cudnnActivationForward(d.h, act, C.byref(one), td, p(x),
                                                    C.byref(zero), td, p(y)))
    gbs = 8 * n_act / (ms * 1e-3) / 1e9
    out["relu"] = {"ms": ms, "GB/s": gbs, "roofline": s.roof("activation_vec4", gbs, "hbm")}
    assert L.cudnnDestroyActivationDescriptor(act) == 0
    del x, y
    # pooling
    n, c = 32 // s.scale, 64
    xp = synth.normal(torch, n * c * 112 * 112, seed=16)
    yp = torch.empty(n * c * 56 * 56, device="cuda")
    pool = C.c_void_p()
    assert L.cudnnCreatePoolingDescriptor(C.byref(pool)) == 0
    assert L.cudnnSetPooling2dDescriptor(pool, 0, 0, 3, 3, 1, 1, 2, 2) == 0
    xd, yd = d.tensor(n, c, 112, 112), d.tensor(n, c, 56, 56)
    ms, _ = s.time(lambda: L.cudnnPoolingForward(d.h, pool, C.byref(one), xd, p(xp),
                                                 C.byref(zero), yd, p(yp)))
    gbs = 4 * (xp.numel() + yp.numel()) / (ms * 1e-3) / 1e9
    out["maxpool"] = {"ms": ms, "GB/s": gbs, "roofline": s.roof("pooling_fwd", gbs, "hbm")}
    assert L.cudnnDestroyPoolingDescriptor(pool) == 0
    del xp, yp
    # batch-norm training
    xb = synth.normal(torch, n * c * 56 * 56, seed=17)
    yb = torch.empty_like(xb)
    sc, bi = torch.ones(c, device="cuda"), torch.zeros(c, device="cuda")
    rm, rv = torch.zeros(c, device="cuda"), torch.ones(c, device="cuda")
    xd = d.tensor(n, c, 56, 56)
    bn = d.tensor(1, c, 1, 1)
    ms, _ = s.time(lambda: L.cudnnBatchNormalizationForwardTraining(
        d.h, 1, C.byref(one), C.byref(zero), xd, p(xb), xd, p(yb), bn, p(sc), p(bi), 0.1, p(rm),
        p(rv), 1e-5, None, None))
    gbs = 8 * xb.numel() / (ms * 1e-3) / 1e9
    out["bn_training"] = {"ms": ms, "GB/s (x + y once)": gbs,
                          "roofline": s.roof("bn_training", gbs, "hbm"),
                          "note": "x is read three times (mean, variance, output) from L2/HBM"}
    d.close()
    first = out["relu"]
    return {"value": first["GB/s"], "unit": "GB/s", "ms": first["ms"], "dtype": "f32",
            "config": "ReLU 2^28 fp32 (value); maxpool 32x64x112x112 3x3/2; BN 32x64x56x56",
            "roofline": first["roofline"], **out}


def suite_rand_dists(s: Suite) -> dict:
    """Philox log-normal (mean 0, stddev 0.5), Poisson (lambda 4 and 100) and
    uniform-double streams, 2^28 values each, seed 1234."""
    from muda_b200 import capi
    torch = s.torch
    L = capi.curand()
    g = C.c_void_p()
    assert L.curandCreateGenerator(C.byref(g), capi.CURAND_RNG_PSEUDO_PHILOX4_32_10) == 0
    assert L.curandSetPseudoRandomGeneratorSeed(g, 1234) == 0
    assert L.curandSetStream(g, s.sp) == 0
    n = (1 << 28) // s.scale
    buf = torch.empty(2 * n, dtype=torch.float32, device="cuda")
    ptr = C.c_void_p(buf.data_ptr())
    out = {}
    for name, fn, eb in (
            ("lognormal", lambda: L.curandGenerateLogNormal(g, ptr, n, C.c_float(0.0),
                                                            C.c_float(0.5)), 4),
            ("poisson_4", lambda: L.curandGeneratePoisson(g, ptr, n, 4.0), 4),
            ("poisson_100", lambda: L.curandGeneratePoisson(g, ptr, n, 100.0), 4),
            ("uniform_double", lambda: L.curandGenerateUniformDouble(g, ptr, n), 8)):
        ms, _ = s.time(fn)
        out[name] = {"ms": ms, "GB/s": eb * n / (ms * 1e-3) / 1e9}
    assert L.curandDestroyGenerator(g) == 0
    v = out["lognormal"]["GB/s"]
    return {"value": v, "unit": "GB/s", "ms": out["lognormal"]["ms"], "dtype": "f32/u32/f64",
            "config": f"{n} values per call", "roofline": s.roof("philox_fill_kernel<kLogNormal>",
                                                                  v, "hbm"), **out}


def suite_fft(s: Suite) -> dict:
    """C2C N = 4096, batch 65536, normal(0,1) re/im seed 3, forward then
    inverse in place; value = bytes moved (read + write, both directions) per second."""
    from muda_b200 import capi, synth
    torch = s.torch
    n, batch = 4096, 65536 // s.scale // s.shard
    x = synth.normal(torch, 2 * n * batch, seed=3)
    L = capi.cufft()
    p = C.c_void_p()
    nn = (C.c_int * 1)(n)
    assert L.cufftPlanMany(C.byref(p), 1, nn, None, 1, n, None, 1, n, 0x29, batch) == 0
    assert L.cufftSetStream(p, s.sp) == 0
    ptr = C.c_void_p(x.data_ptr())

    def call():
        assert L.cufftExecC2C(p, ptr, ptr, -1) == 0
        assert L.cufftExecC2C(p, ptr, ptr, 1) == 0
    ms, launches = s.time(call, launches_per_call=2)
    per_dir = 2 * 8 * n * batch
    # end to end through the C ABI with host buffers: pinned input copied in, forward
    # then inverse, result copied back, all inside the timed region
    e2e = None
    if s.shard == 1 and s.e2e:
        h_in = torch.empty(2 * n * batch, dtype=torch.float32, pin_memory=True)
        h_in.copy_(x)
        h_out = torch.empty_like(h_in)
        y = torch.empty_like(x)
        py = C.c_void_p(y.data_ptr())

        def e2e_call():
            y.copy_(h_in, non_blocking=True)
            assert L.cufftExecC2C(p, py, py, -1) == 0
            assert L.cufftExecC2C(p, py, py, 1) == 0
            h_out.copy_(y, non_blocking=True)
        steps, warm = s.steps, s.warmup
        s.steps, s.warmup = 3, 1
        e_ms, _ = s.time(e2e_call)
        s.steps, s.warmup = steps, warm
        e2e = {"value": 2 * per_dir / (e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms": e_ms,
               "h2d_bytes_per_step": 8 * n * batch, "d2h_bytes_per_step": 8 * n * batch,
               "path": "pinned host -> device copy, cufftExecC2C forward + inverse in place, "
                       "device -> pinned host copy"}
        del h_in, h_out, y
    assert L.cufftDestroy(p) == 0
    gbs = 2 * per_dir / (ms * 1e-3) / 1e9
    flops = 2 * 5 * n * 12 * batch
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "c64", "e2e": e2e,
           "gflops_5nlogn": flops / (ms * 1e-3) / 1e9,
           "config": f"N {n} x batch {batch}, forward + inverse in place, "
                     f"data {per_dir / 2e9:.2f} GB > L2",
           "roofline": s.roof("stockham_bulk3_kernel<12>", gbs, "hbm"), "launches": launches,
           "algorithmic_bytes_per_launch": per_dir}
    if s.cpu:
        import oracle
        sample = max(1, batch // 64)
        xs = x[: 2 * n * sample].cpu().numpy().view(np.complex64)
        dt = cpu_time(lambda: oracle.fft_c2c(xs, [n], sample, -1, threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": (2 * 8 * n * sample) / dt / 1e9, "unit": "GB/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"forward transform of {sample} of {batch} sequences, "
                                         "oracle/fft.cpp radix-2 Stockham stages"}
    return out


def suite_fft_nonpow2(s: Suite, n: int, kernel: str, how: str) -> dict:
    """C2C of a length that is not a power of two, batch 262144 (N = 1000: mixed radix
    8 x 5 x 5 x 5; N = 1009, a prime: Bluestein with inner length 2048 on chip),
    normal(0,1) re/im seed 4, forward then inverse in place; value = bytes moved (read
    + write, both directions) per second."""
    from muda_b200 import capi, synth
    torch = s.torch
    batch = 262144 // s.scale
    x = synth.normal(torch, 2 * n * batch, seed=4)
    L = capi.cufft()
    p = C.c_void_p()
    nn = (C.c_int * 1)(n)
    assert L.cufftPlanMany(C.byref(p), 1, nn, None, 1, n, None, 1, n, capi.CUFFT_C2C, batch) == 0
    assert L.cufftSetStream(p, s.sp) == 0
    ptr = C.c_void_p(x.data_ptr())

    def call():
        assert L.cufftExecC2C(p, ptr, ptr, -1) == 0
        assert L.cufftExecC2C(p, ptr, ptr, 1) == 0
    ms, launches = s.time(call, launches_per_call=2)
    assert L.cufftDestroy(p) == 0
    per_dir = 2 * 8 * n * batch
    gbs = 2 * per_dir / (ms * 1e-3) / 1e9
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "c64",
           "gflops_5nlogn": 2 * 5 * n * np.log2(n) * batch / (ms * 1e-3) / 1e9,
           "config": f"N {n} x batch {batch}, forward + inverse in place ({how}), "
                     f"data {per_dir / 2e9:.2f} GB > L2",
           "roofline": s.roof(kernel, gbs, "hbm"), "launches": launches,
           "algorithmic_bytes_per_launch": per_dir}
    if s.cpu:
        import oracle
        sample = max(1, batch // 4096)
        xs = x[: 2 * n * sample].cpu().numpy().view(np.complex64)
        dt = cpu_time(lambda: oracle.fft_c2c(xs, [n], sample, -1, threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": (2 * 8 * n * sample) / dt / 1e9, "unit": "GB/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"forward transform of {sample} of {batch} sequences, "
                                         "oracle/fft.cpp direct DFT (the reference's algorithm "
                                         "for this length)"}
    return out


def suite_fft_real(s: Suite) -> dict:
    """R2C then C2R of L = 4096 reals, batch 65536, normal(0,1) seed 5, out of place
    (reals -> half spectrum -> reals); value = algorithmic bytes (reals and half spectrum,
    read + write, both directions) per second."""
    from muda_b200 import capi, synth
    torch = s.torch
    n, batch = 4096, 65536 // s.scale
    h = n // 2 + 1
    x = synth.normal(torch, n * batch, seed=5)
    X = torch.empty(batch * h, dtype=torch.complex64, device="cuda")
    L = capi.cufft()
    fwd, inv = C.c_void_p(), C.c_void_p()
    assert L.cufftPlan1d(C.byref(fwd), n, capi.CUFFT_R2C, batch) == 0
    assert L.cufftPlan1d(C.byref(inv), n, capi.CUFFT_C2R, batch) == 0
    for p in (fwd, inv):
        assert L.cufftSetStream(p, s.sp) == 0
    px, pX = C.c_void_p(x.data_ptr()), C.c_void_p(X.data_ptr())

    y = torch.empty_like(x)
    py = C.c_void_p(y.data_ptr())
    # each direction timed on its own (x -> X, X -> y), so no data grows across steps
    ms_f, lf = s.time(lambda: L.cufftExecR2C(fwd, px, pX))
    ms_i, li = s.time(lambda: L.cufftExecC2R(inv, pX, py))
    assert L.cufftDestroy(fwd) == 0 and L.cufftDestroy(inv) == 0
    per_dir = 4 * n * batch + 8 * h * batch
    ms = ms_f + ms_i
    gbs = 2 * per_dir / (ms * 1e-3) / 1e9
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32/c64",
           "config": f"L {n} x batch {batch}, R2C + C2R out of place, reals "
                     f"{4 * n * batch / 1e9:.2f} GB > L2",
           "r2c": {"ms": ms_f, "GB/s": per_dir / (ms_f * 1e-3) / 1e9},
           "c2r": {"ms": ms_i, "GB/s": per_dir / (ms_i * 1e-3) / 1e9},
           "roofline": s.roof("r2c_bulk_kernel<11> + c2r_bulk_kernel<11>", gbs, "hbm"),
           "launches": lf + li, "algorithmic_bytes_per_direction": per_dir}
    if s.cpu:
        import oracle
        sample = max(1, batch // 64)
        xs = x[: n * sample].cpu().numpy()
        dt = cpu_time(lambda: oracle.fft_r2c(xs, [n], sample, threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": (4 * n + 8 * h) * sample / dt / 1e9, "unit": "GB/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"R2C of {sample} of {batch} rows, oracle/fft.cpp "
                                         "gather + radix-2 Stockham + keep half"}
    return out


def suite_softmax(s: Suite) -> dict:
    """configs[4] softmax: 65536 x 4096 fp32 normal(0, 0.02) seed 11, ACCURATE, INSTANCE."""
    from muda_b200 import capi, synth
    torch = s.torch
    rows, cols = 65536 // s.scale // s.shard, 4096
    x = synth.normal(torch, rows * cols, seed=11, std=0.02)
    y = torch.empty_like(x)
    L = capi.cudnn()
    h, xd = C.c_void_p(), C.c_void_p()
    assert L.cudnnCreate(C.byref(h)) == 0
    assert L.cudnnSetStream(h, s.sp) == 0
    assert L.cudnnCreateTensorDescriptor(C.byref(xd)) == 0
    assert L.cudnnSetTensor4dDescriptor(xd, 0, 0, rows, cols, 1, 1) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    args = (h, 1, 0, C.byref(one), xd, C.c_void_p(x.data_ptr()), C.byref(zero), xd,
            C.c_void_p(y.data_ptr()))
    ms, launches = s.time(lambda: L.cudnnSoftmaxForward(*args))
    assert L.cudnnDestroyTensorDescriptor(xd) == 0
    assert L.cudnnDestroy(h) == 0
    alg = 2 * rows * cols * 4
    gbs = alg / (ms * 1e-3) / 1e9
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32",
           "config": f"{rows} x {cols}, ACCURATE, INSTANCE, data {alg / 2e9:.2f} GB > L2",
           "roofline": s.roof("softmax_block_rows<4,4>", gbs, "hbm"), "launches": launches,
           "algorithmic_bytes_per_launch": alg}
    if s.cpu:
        import oracle
        xs = x.cpu().numpy()
        dt = cpu_time(lambda: oracle.softmax(xs, (rows, cols, 1, 1), algo=1,
                                             threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": alg / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(),
                               "kind": "port", "sample": "full problem, oracle/dnn.cpp"}
    return out


def suite_gemm_bf16(s: Suite) -> dict:
    """configs[4] GEMM: bf16 M = N = K = 8192, batch 8, fp32 accumulate, normal(0, 0.02)
    seed 11, alpha 1, beta 0, through cublasGemmStridedBatchedEx.  The value is the
    N,N call (both operands as stored by a column-major caller, the call a row-major
    caller makes with its operands swapped: A is MN-major, B K-major); T,N (both
    K-major) is timed beside it on the same buffers (N,T and T,T run the same kernel
    with MN-major B; tests cover them)."""
    from muda_b200 import capi, synth
    torch = s.torch
    m = n = k = 8192 // s.scale
    batch = max(1, 8 // s.shard)
    a = synth.normal(torch, m * k * batch, seed=11, std=0.02).to(torch.bfloat16)
    b = synth.normal(torch, n * k * batch, seed=11, std=0.02,
                     offset=(m * k * batch + 3) // 4 * 4).to(torch.bfloat16)
    c = torch.empty(m * n * batch, dtype=torch.bfloat16, device="cuda")
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, s.sp) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)

    def args(ta, tb):
        return (h, ta, tb, m, n, k, C.byref(one), C.c_void_p(a.data_ptr()), 14, k if ta else m,
                m * k, C.c_void_p(b.data_ptr()), 14, n if tb else k, n * k, C.byref(zero),
                C.c_void_p(c.data_ptr()), 14, m, m * n, batch, 68, -1)
    flop = 2.0 * m * n * k * batch
    layouts = {}
    for name, ta, tb in (("NN", 0, 0), ("TN", 1, 0), ("TT", 1, 1), ("NT", 0, 1)):
        a_ = args(ta, tb)
        ms_l, launches_l = s.time(lambda: L.cublasGemmStridedBatchedEx(*a_))
        layouts[name] = {"ms": ms_l, "TFLOP/s": flop / (ms_l * 1e-3) / 1e12,
                         "launches": launches_l}
    # end to end through the C ABI with host buffers (N,N): A and B copied in from pinned
    # host memory, the call, C copied back, all inside the timed region
    e2e = None
    if s.shard == 1 and s.e2e:
        ha, hb = (t.cpu().pin_memory() for t in (a, b))
        hc = torch.empty(m * n * batch, dtype=torch.bfloat16, pin_memory=True)
        da, db = torch.empty_like(a), torch.empty_like(b)
        e_args = list(args(0, 0))
        e_args[7], e_args[11] = C.c_void_p(da.data_ptr()), C.c_void_p(db.data_ptr())

        def e2e_call():
            da.copy_(ha, non_blocking=True)
            db.copy_(hb, non_blocking=True)
            assert L.cublasGemmStridedBatchedEx(*e_args) == 0
            hc.copy_(c, non_blocking=True)
        steps, warm = s.steps, s.warmup
        s.steps, s.warmup = 3, 1
        e_ms, _ = s.time(e2e_call)
        s.steps, s.warmup = steps, warm
        e2e = {"value": flop / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": e_ms,
               "h2d_bytes_per_step": 2 * (m * k + k * n) * batch,
               "d2h_bytes_per_step": 2 * m * n * batch,
               "path": "pinned host -> device copies of A and B, cublasGemmStridedBatchedEx "
                       "(N,N), device -> pinned host copy of C"}
        del ha, hb, hc, da, db
    assert L.cublasDestroy_v2(h) == 0
    ms, launches = layouts["NN"]["ms"], layouts["NN"]["launches"]
    tf = flop / (ms * 1e-3) / 1e12
    out = {"value": tf, "unit": "TFLOP/s", "ms": ms, "dtype": "bf16 (fp32 accumulate)", "e2e": e2e,
           "config": f"{m}x{n}x{k} x batch {batch}, N,N (A MN-major, B K-major), operands "
                     f"{3 * m * k * batch * 2 / 1e9:.1f} GB",
           "roofline": s.roof("tc_gemm_kernel<GemmProblem<bf16,MN,K>>", tf, "tensor"),
           "launches": launches, "layouts": layouts,
           "frac_of_sustained": tf / s.peaks.get("bf16_tflops_sustained", 1391.1)}
    if s.cpu:
        import oracle
        A = a.view(torch.int16).cpu().numpy().view(np.uint16)
        B = b.view(torch.int16).cpu().numpy().view(np.uint16)
        rng = np.random.default_rng(0)
        ne = 4096
        rows = rng.integers(0, m, ne).astype(np.int32)
        cols = (rng.integers(0, batch, ne) * n + rng.integers(0, n, ne)).astype(np.int32)
        Cs = np.zeros(m * n * batch, np.uint16)
        dt = cpu_time(lambda: oracle.gemm("bf16", False, False, m, n, k, 1.0, A, m, B, k, 0.0,
                                          Cs, m, stride_a=m * k, stride_b=n * k,
                                          stride_c=m * n, batch=batch, entries=(rows, cols),
                                          threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": 2.0 * k * ne / dt / 1e12, "unit": "TFLOP/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"{ne} sampled output entries (of {m * n * batch}), "
                                         "oracle/gemm.cpp, rate extrapolated"}
    return out


def suite_conv(s: Suite, dtype: str, krsc: bool = True) -> dict:
    """configs[4] conv: NHWC x 64x56x56x256, KRSC (or KCRS) w 256x3x3x256, pad 1, stride 1,
    normal(0, 0.02) seed 11 (x then w), cross-correlation, alpha 1, beta 0."""
    from muda_b200 import capi, synth
    torch = s.torch
    n, c, hh, ww, kk = max(1, 64 // s.scale // s.shard), 256, 56, 56, 256
    x = synth.normal(torch, n * hh * ww * c, seed=11, std=0.02)
    w = synth.normal(torch, kk * 9 * c, seed=11, std=0.02, offset=(n * hh * ww * c + 3) // 4 * 4)
    if dtype == "bf16":
        x, w = x.to(torch.bfloat16), w.to(torch.bfloat16)
    y = torch.empty(n * hh * ww * kk, dtype=x.dtype, device="cuda")
    dt_code = 9 if dtype == "bf16" else 0
    L = capi.cudnn()
    h, xd, wd, cd, yd = (C.c_void_p() for _ in range(5))
    assert L.cudnnCreate(C.byref(h)) == 0
    assert L.cudnnSetStream(h, s.sp) == 0
    assert L.cudnnCreateTensorDescriptor(C.byref(xd)) == 0
    assert L.cudnnSetTensor4dDescriptor(xd, 1, dt_code, n, c, hh, ww) == 0
    assert L.cudnnCreateTensorDescriptor(C.byref(yd)) == 0
    assert L.cudnnSetTensor4dDescriptor(yd, 1, dt_code, n, kk, hh, ww) == 0
    assert L.cudnnCreateFilterDescriptor(C.byref(wd)) == 0
    assert L.cudnnSetFilter4dDescriptor(wd, dt_code, 1 if krsc else 0, kk, c, 3, 3) == 0
    assert L.cudnnCreateConvolutionDescriptor(C.byref(cd)) == 0
    assert L.cudnnSetConvolution2dDescriptor(cd, 1, 1, 1, 1, 1, 1, 1, 0) == 0
    one, zero = C.c_float(1.0), C.c_float(0.0)
    args = (h, C.byref(one), xd, C.c_void_p(x.data_ptr()), wd, C.c_void_p(w.data_ptr()), cd, 0,
            None, 0, C.byref(zero), yd, C.c_void_p(y.data_ptr()))
    steps, warm = s.steps, s.warmup
    s.steps, s.warmup = max(3, min(steps, 5)), 2
    ms, launches = s.time(lambda: L.cudnnConvolutionForward(*args))
    s.steps, s.warmup = steps, warm
    for fn, d in (("cudnnDestroyTensorDescriptor", xd), ("cudnnDestroyTensorDescriptor", yd),
                  ("cudnnDestroyFilterDescriptor", wd),
                  ("cudnnDestroyConvolutionDescriptor", cd)):
        assert getattr(L, fn)(d) == 0
    assert L.cudnnDestroy(h) == 0
    flop = 2.0 * n * kk * hh * ww * c * 9
    tf = flop / (ms * 1e-3) / 1e12
    if dtype == "bf16":
        bound, kern = "tensor", "tc_gemm_kernel<ConvProblem<bf16,1>,256,4,1>"
    else:
        bound, kern = "tensor-tf32x3", "tc_gemm_split_kernel<ConvProblem<float,2>,256,2,2>"
    return {"value": tf, "unit": "TFLOP/s", "ms": ms,
            "dtype": dtype if dtype == "bf16" else "f32 (split-tf32 on tcgen05)",
            "config": f"NHWC {n}x{hh}x{ww}x{c} -> {kk}, 3x3 pad 1, "
                      f"{'KRSC' if krsc else 'KCRS'} filter",
            "roofline": s.roof(kern, tf, bound), "launches": launches}


def _blas_handle(s):
    from muda_b200 import capi
    L = capi.cublas()
    h = C.c_void_p()
    assert L.cublasCreate_v2(C.byref(h)) == 0
    assert L.cublasSetStream_v2(h, s.sp) == 0
    return L, h


def suite_level1(s: Suite, op: str) -> dict:
    """cuBLAS level 1: saxpy / sdot on 2^28 fp32 elements (1.07 GB per
    vector, larger than L2), uniform[-1, 1] from seed 5."""
    from muda_b200 import synth
    torch = s.torch
    n = (1 << 28) // s.scale
    x = synth.uniform_pm1(torch, n, seed=5)
    y = synth.uniform_pm1(torch, n, seed=5, offset=(n + 3) // 4 * 4)
    L, h = _blas_handle(s)
    px, py = C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr())
    if op == "saxpy":
        a = C.c_float(0.5)
        fn = lambda: L.cublasSaxpy_v2(h, n, C.byref(a), px, 1, py, 1)
        alg, kern = 12 * n, "elementwise<kAxpy, vec>"
    else:
        # device pointer mode keeps the timed call asynchronous (host mode waits)
        assert L.cublasSetPointerMode_v2(h, 1) == 0
        out = torch.zeros(1, dtype=torch.float32, device="cuda")
        fn = lambda: L.cublasSdot_v2(h, n, px, 1, py, 1, C.c_void_p(out.data_ptr()))
        alg, kern = 8 * n, "reduce_kernel<kDot, vec>"
    ms, launches = s.time(fn)
    assert L.cublasDestroy_v2(h) == 0
    gbs = alg / (ms * 1e-3) / 1e9
    out_d = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32",
             "config": f"n = {n}, unit stride, data {alg / 1e9:.2f} GB per call > L2",
             "roofline": s.roof(kern, gbs, "hbm"), "launches": launches,
             "algorithmic_bytes_per_launch": alg}
    if s.cpu:
        import oracle
        xs, ys = x[: 1 << 24].cpu().numpy(), y[: 1 << 24].cpu().numpy()
        if op == "saxpy":
            dt = cpu_time(lambda: oracle.saxpy(1 << 24, 0.5, xs, 1, ys, 1))
            per = 12
        else:
            dt = cpu_time(lambda: oracle.sreduce("dot", 1 << 24, xs, 1, ys, 1))
            per = 8
        out_d["cpu_baseline"] = {"value": per * (1 << 24) / dt / 1e9, "unit": "GB/s", "cores": 1,
                                 "kind": "port",
                                 "sample": "2^24 elements, oracle/blas12.cpp sequential loop"}
    return out_d


def suite_gemv(s: Suite, trans: bool) -> dict:
    """cuBLAS level 2: sgemv on a 16384 x 16384 column-major fp32 matrix
    (1.07 GB), alpha 1, beta 0, uniform[-1, 1] from seed 6."""
    from muda_b200 import synth
    torch = s.torch
    m = n = 16384 // s.scale
    A = synth.uniform_pm1(torch, m * n, seed=6)
    x = synth.uniform_pm1(torch, n, seed=6, offset=(m * n + 3) // 4 * 4)
    y = torch.zeros(m, dtype=torch.float32, device="cuda")
    L, h = _blas_handle(s)
    one, zero = C.c_float(1.0), C.c_float(0.0)
    args = (h, 1 if trans else 0, m, n, C.byref(one), C.c_void_p(A.data_ptr()), m,
            C.c_void_p(x.data_ptr()), 1, C.byref(zero), C.c_void_p(y.data_ptr()), 1)
    ms, launches = s.time(lambda: L.cublasSgemv_v2(*args))
    assert L.cublasDestroy_v2(h) == 0
    alg = 4 * m * n + 4 * n + 4 * m
    gbs = alg / (ms * 1e-3) / 1e9
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32",
           "config": f"{m} x {n}, op {'T' if trans else 'N'}, matrix {4 * m * n / 1e9:.2f} GB > L2",
           "roofline": s.roof("gemv_t_kernel<vec>" if trans else "gemv_n_kernel", gbs, "hbm"),
           "launches": launches, "algorithmic_bytes_per_launch": alg}
    if s.cpu:
        import oracle
        rows = 2048
        Ah = A[: rows * m].cpu().numpy() if not trans else A.cpu().numpy()
        xh, yh = x.cpu().numpy(), np.zeros(max(m, n), np.float32)
        if trans:
            dt = cpu_time(lambda: oracle.sgemv(True, m, rows, 1.0, Ah, m, xh, 1, 0.0, yh, 1,
                                               threads=os.cpu_count() or 1))
        else:
            dt = cpu_time(lambda: oracle.sgemv(False, m, rows, 1.0, Ah, m, xh, 1, 0.0, yh, 1,
                                               threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": 4 * m * rows / dt / 1e9, "unit": "GB/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"{rows} of {n} columns, oracle/blas12.cpp"}
    return out



def suite_geam(s: Suite) -> dict:
    """cuBLAS Sgeam C = A^T + B on 16384 x 16384 column-major fp32 matrices (1.07 GB
    each, larger than L2), alpha 1, beta 1, uniform[-1, 1] from seed 8; the
    transposed operand makes this the staged (shared-memory) form of the kernel."""
    from muda_b200 import synth
    torch = s.torch
    m = n = 16384 // s.scale
    A = synth.uniform_pm1(torch, m * n, seed=8)
    B = synth.uniform_pm1(torch, m * n, seed=8, offset=(m * n + 3) // 4 * 4)
    Cm = torch.empty(m * n, dtype=torch.float32, device="cuda")
    L, h = _blas_handle(s)
    one = C.c_float(1.0)
    args = (h, 1, 0, m, n, C.byref(one), C.c_void_p(A.data_ptr()), n, C.byref(one),
            C.c_void_p(B.data_ptr()), m, C.c_void_p(Cm.data_ptr()), m)
    ms, launches = s.time(lambda: L.cublasSgeam(*args))
    # the untransposed form (both operands read straight into registers), same bytes
    args_nn = args[:1] + (0,) + args[2:7] + (m,) + args[8:]
    ms_nn, _ = s.time(lambda: L.cublasSgeam(*args_nn))
    assert L.cublasDestroy_v2(h) == 0
    alg = 12 * m * n
    gbs = alg / (ms * 1e-3) / 1e9
    out = {"value": gbs, "unit": "GB/s", "ms": ms, "dtype": "f32",
           "op_n_n": {"value": alg / (ms_nn * 1e-3) / 1e9, "unit": "GB/s", "ms": ms_nn},
           "config": f"{m} x {n}, op(A) T, op(B) N, {alg / 1e9:.2f} GB per call > L2",
           "roofline": s.roof("geam_kernel_db<float,1>", gbs, "hbm"), "launches": launches,
           "algorithmic_bytes_per_launch": alg}
    if s.cpu:
        import oracle
        Ah = A.cpu().numpy()
        Bh = B.cpu().numpy()
        Ch = np.zeros(m * n, np.float32)
        Ch.fill(1.0)
        cores = os.cpu_count() or 1
        dt = cpu_time(lambda: oracle.geam(np.float32, True, False, m, n, 1.0, Ah, n, 1.0,
                                          Bh, m, Ch, m, threads=cores))
        out["cpu_baseline"] = {"value": alg / dt / 1e9, "unit": "GB/s", "cores": cores,
                               "kind": "port",
                               "sample": "full problem, oracle/blas12.cpp column loop split over "
                                         "host threads"}
    return out

def suite_dgemm(s: Suite) -> dict:
    """cublasDgemm fp64 M = N = K = 4096 (column-major, N,N), alpha 1, beta 0,
    uniform[-1, 1] from seed 21, through the fp64 tensor-core MMA kernel."""
    from muda_b200 import synth
    torch = s.torch
    m = n = k = 4096 // s.scale
    a = synth.uniform_pm1(torch, m * k, seed=21).double()
    b = synth.uniform_pm1(torch, k * n, seed=21, offset=(m * k + 3) // 4 * 4).double()
    c = torch.empty(m * n, dtype=torch.float64, device="cuda")
    L, h = _blas_handle(s)
    one, zero = C.c_double(1.0), C.c_double(0.0)
    args = (h, 0, 0, m, n, k, C.byref(one), C.c_void_p(a.data_ptr()), m,
            C.c_void_p(b.data_ptr()), k, C.byref(zero), C.c_void_p(c.data_ptr()), m)
    ms, launches = s.time(lambda: L.cublasDgemm_v2(*args), flush=True)
    assert L.cublasDestroy_v2(h) == 0
    flop = 2.0 * m * n * k
    tf = flop / (ms * 1e-3) / 1e12
    out = {"value": tf, "unit": "TFLOP/s", "ms": ms, "dtype": "f64",
           "config": f"{m}x{n}x{k} fp64 N,N, L2 flushed before each call",
           "roofline": s.roof("dgemm_kernel<128,false,false> (fp64 MMA)", tf, "fp64"),
           "launches": launches}
    if s.cpu:
        import oracle
        A = a.cpu().numpy()
        B = b.cpu().numpy()
        rng = np.random.default_rng(0)
        ne = 8192
        pick = rng.choice(m * n, ne, replace=False)
        rows, cols = (pick % m).astype(np.int32), (pick // m).astype(np.int32)
        dt = cpu_time(lambda: oracle.dgemm(False, False, m, n, k, 1.0, A, m, B, k, 0.0,
                                           np.zeros(m * n), m, entries=(rows, cols),
                                           threads=os.cpu_count() or 1))
        out["cpu_baseline"] = {"value": 2.0 * k * ne / dt / 1e12, "unit": "TFLOP/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"{ne} sampled output entries (of {m * n}), "
                                         "oracle/blas64.cpp extended-precision dot products, "
                                         "rate extrapolated"}
    return out


SUITE = {
    "sgemm": suite_sgemm,
    "spmv": suite_spmv,
    "spmv_t": suite_spmv_t,
    "spmm": suite_spmm,
    "fft": suite_fft,
    "fft_real": suite_fft_real,
    "fft_mixed": lambda s: suite_fft_nonpow2(s, 1000, "mixed_radix_kernel", "mixed radix"),
    "fft_bluestein": lambda s: suite_fft_nonpow2(s, 1009, "bluestein_kernel<11>",
                                                 "Bluestein"),
    "conv_bwd": suite_conv_bwd,
    "dnn_elementwise": suite_dnn_elementwise,
    "rand_dists": suite_rand_dists,
    "softmax": suite_softmax,
    "gemm_bf16": suite_gemm_bf16,
    "conv_bf16": lambda s: suite_conv(s, "bf16"),
    "conv_f32": lambda s: suite_conv(s, "f32"),
    "conv_f32_kcrs": lambda s: suite_conv(s, "f32", krsc=False),
    "saxpy": lambda s: suite_level1(s, "saxpy"),
    "sdot": lambda s: suite_level1(s, "sdot"),
    "sgemv_n": lambda s: suite_gemv(s, False),
    "sgemv_t": lambda s: suite_gemv(s, True),
    "sgeam": suite_geam,
    "dgemm": suite_dgemm,
}


SUITE_GAP_S = 0.5  # idle time between routines, so that no routine inherits another's power state


def run_suite(names, args, torch) -> dict:
    out = {}
    for name in names:
        time.sleep(SUITE_GAP_S)
        s = Suite(torch, max(3, args.steps // 4), args.warmup, not args.no_cpu, args.scale)
        s.e2e = not args.no_e2e
        try:
            out[name] = SUITE[name](s)
        except Exception as e:  # one failing routine must not hide the others
            out[name] = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()
    return out


def _cpu_generator():
    """The reference's host generator for the CPU legs: its own curand_context.mm
    compiled by oracle/ref/build.py ("reference"), else the oracle's restatement of it
    ("port").  Returns (kind, description, uniform(out, offset), normal(out, offset))."""
    threads = os.cpu_count() or 1
    import oracle.ref as ref
    if ref.available():
        def uni(out, offset):
            ref.generate_parallel(ref.UNIFORM, SEED, offset, len(out), threads=threads, out=out)

        def nor(out, offset):
            ref.generate_parallel(ref.NORMAL, SEED, offset, len(out), 0.0, 1.0, threads=threads,
                                  out=out)
        return ("reference", "the reference's GenerateHostUniform / GenerateHostNormal "
                "(libraries/rand/src/curand_context.mm, compiled unmodified by "
                "oracle/ref/build.py), one generator per host thread on consecutive "
                "Philox-block slices of the call", uni, nor)
    import oracle

    def uni_p(out, offset):
        out[:] = oracle.generate_uniform(SEED, offset, len(out), threads=threads)[0]

    def nor_p(out, offset):
        out[:] = oracle.generate_normal(SEED, offset, len(out), 0.0, 1.0, threads=threads)[0]
    return ("port", "oracle/philox.cpp, the restatement of "
            "libraries/rand/src/curand_context.mm:42-185", uni_p, nor_p)


def cpu_baseline() -> dict:
    """The reference's host generator path on all host cores, the config's two calls."""
    threads = os.cpu_count() or 1
    kind, what, uni, nor = _cpu_generator()
    hu = np.empty(CPU_SAMPLE_WORDS, np.float32)
    hn = np.empty(CPU_SAMPLE_WORDS, np.float32)
    uni(hu[: 1 << 20], 0)  # touch the code paths once
    hu.fill(0.0)
    hn.fill(0.0)
    t0 = time.perf_counter()
    uni(hu, 0)
    nor(hn, CPU_SAMPLE_WORDS)
    dt = time.perf_counter() - t0
    return {"value": 2 * 4 * CPU_SAMPLE_WORDS / dt / 1e9, "unit": UNIT, "cores": threads,
            "kind": kind, "seconds": dt,
            "sample": f"uniform + normal, 2^{CPU_SAMPLE_WORDS.bit_length() - 1} words each "
                      f"(1/{N_WORDS // CPU_SAMPLE_WORDS} of the config), {what}"}


def run_reference(args) -> None:
    """Reference arm: the reference's CPU path for this workload, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    kind, what, uni, nor = _cpu_generator()
    hu = np.empty(CPU_SAMPLE_WORDS, np.float32)
    hn = np.empty(CPU_SAMPLE_WORDS, np.float32)
    hu.fill(0.0)  # fault the pages in before the timed region
    hn.fill(0.0)
    for _ in range(args.warmup):
        uni(hu[: CPU_SAMPLE_WORDS // 8], 0)
        nor(hn[: CPU_SAMPLE_WORDS // 8], CPU_SAMPLE_WORDS)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        uni(hu, 0)
        nor(hn, CPU_SAMPLE_WORDS)
    dt = (time.perf_counter() - t0) / args.steps
    value = 2 * 4 * CPU_SAMPLE_WORDS / dt / 1e9
    sample = (f"per step uniform + normal of 2^{CPU_SAMPLE_WORDS.bit_length() - 1} words each "
              f"(1/{N_WORDS // CPU_SAMPLE_WORDS} of the config)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32->f32",
        "data": "synthetic (counter-based RNG output)",
        "config": {"workload": "configs[1]: Philox4x32-10 uniform 2^30 + normal(0,1) 2^30, "
                               "seed 1234, offset 0, same generator and stream",
                   "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": sample + "; " + what},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_spmv_dist(args) -> None:
    """`--routine spmv_dist` under torchrun: spmv_dist_measure's line on rank 0."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    res = spmv_dist_measure(args, torch, dist if world > 1 else None, world, rank, local)
    if rank == 0:
        print(json.dumps({"routine": "spmv_dist", **res}), flush=True)
    if world > 1:
        dist.destroy_process_group()
    if not res["y_check"]:
        raise SystemExit("distributed SpMV arms disagree (peer vs NCCL bit for bit, "
                         "overlapped vs sequential within the summation bound)")


def spmv_dist_measure(args, torch, dist, world: int, rank: int, local: int) -> dict:
    """configs[2] SpMV across the ranks of torchrun (strong scaling: the 4M x 4M matrix
    is fixed, its rows split into nnz-balanced blocks).  Each step gathers x into
    local HBM and runs the local cusparseSpMV.  Two exchanges are timed on the same
    blocks: the NVLink peer-memory pull of libmuda_peer and NCCL's
    all_gather_into_tensor; both must give the same y, bit for bit.  Each is timed twice:
    exchange then product, and overlapped (DistSpMV overlap=True: the product over this
    rank's own x block runs on a side stream during the exchange, the rest after it;
    the overlapped y must match the sequential one within the float32 summation bound).
    The value is the fastest of the four (named in config.exchange), the others are
    reported beside it.  Reported are the step time (max over ranks) with and without
    the exchange.  `dist` is None on one rank."""
    from muda_b200 import synth
    from muda_b200.dist_spmv import DistSpMV
    group = None
    rows = (1 << 22) // args.scale
    mtx = synth.powerlaw_csr(torch, rows, rows, seed=7)
    nnz = mtx["nnz"]
    names = ("peer", "nccl", "peer+overlap", "nccl+overlap")
    arms = {nm: DistSpMV.from_full(torch, dist, group, mtx["row_offsets"], mtx["col_ind"],
                                   mtx["values"], rows, exchange=nm.split("+")[0],
                                   overlap=nm.endswith("overlap")) for nm in names}
    d = arms["peer"]
    x_local = d.x_slice(mtx["x"])
    ys = {ex: torch.zeros(max(d.rows, 1), dtype=torch.float32, device="cuda") for ex in arms}
    # |A| |x| per local row, for the bound on the overlapped (two-part) row sums
    o64 = mtx["row_offsets"][d.row_begin:d.row_end + 1].to(torch.int64)
    e0, e1 = int(o64[0].item()), int(o64[-1].item())
    ax = (mtx["values"][e0:e1].abs() * mtx["x"][mtx["col_ind"][e0:e1].to(torch.int64)].abs())
    row_id = torch.repeat_interleave(torch.arange(d.rows, device="cuda"), o64[1:] - o64[:-1])
    mag = torch.zeros(max(d.rows, 1), dtype=torch.float64, device="cuda")
    mag.index_add_(0, row_id, ax.double())
    row_len = torch.zeros(max(d.rows, 1), dtype=torch.float64, device="cuda")
    row_len[:d.rows] = (o64[1:] - o64[:-1]).double()
    del o64, ax, row_id
    del mtx
    torch.cuda.empty_cache()
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB > L2
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    times = {ex: ([], [], []) for ex in arms}
    for it in range(args.warmup + args.steps):
        for ex, arm in arms.items():
            flush.fill_(float(it))
            barrier()
            ev[0].record()
            if arm.overlap:
                arm.spmv(1.0, x_local, 0.0, ys[ex])
                ev[1].record()
            else:
                arm.gather_x(x_local)
                ev[1].record()
                arm.local(1.0, 0.0, ys[ex])
            ev[2].record()
            torch.cuda.synchronize()
            if it >= args.warmup:
                full_ms, local_ms, gather_ms = times[ex]
                gather_ms.append(ev[0].elapsed_time(ev[1]) if not arm.overlap else 0.0)
                local_ms.append(ev[1].elapsed_time(ev[2]) if not arm.overlap else 0.0)
                full_ms.append(ev[0].elapsed_time(ev[2]))
    barrier()
    status = d._peer.take_status() | arms["peer+overlap"]._peer.take_status()
    bound = (row_len + 3) * 2.0 ** -24 * mag + 1e-30
    within = bool((ys["peer+overlap"].double() - ys["peer"].double()).abs()
                  .le(2 * bound).all().item())
    same = (bool(torch.equal(ys["peer"], ys["nccl"])) and status == 0 and
            bool(torch.equal(ys["peer+overlap"], ys["nccl+overlap"])) and within)
    check = torch.tensor([0 if same else 1], dtype=torch.int32, device="cuda")
    stats = torch.tensor([float(np.mean(v)) for ex in names for v in times[ex]],
                         device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(check, op=dist.ReduceOp.MAX)
    shares = torch.tensor([d.nnz], dtype=torch.int64, device="cuda")
    if world > 1:
        parts = [torch.zeros_like(shares) for _ in range(world)]
        dist.all_gather(parts, shares)
        shares = torch.cat(parts)
    st = [float(v) for v in stats.cpu()]
    per = {nm: st[3 * i:3 * i + 3] for i, nm in enumerate(names)}  # full, local, gather
    alg_bytes = nnz * 8 + (rows + 1) * 4 + rows * 4 + rows * 4
    ok = int(check.item()) == 0
    best = min(names, key=lambda nm: per[nm][0])
    full = per[best][0]
    # the exchange's own time and the kernel-only time come from the sequential arm
    # of the same exchange
    _, loc, gat = per[best.split("+")[0]]
    exchange_name = {"peer": "peer-memory pull over NVLink (libmuda_peer)",
                     "nccl": "NCCL all_gather_into_tensor"}[best.split("+")[0]]
    if best.endswith("overlap"):
        exchange_name += ", overlapped with the own-block product"
    nz = shares.cpu().numpy()
    res = {
        "metric": "SpMV GB/s (algorithmic bytes of the whole matrix / step time, max over "
                  "ranks)", "value": alg_bytes / (full * 1e-3) / 1e9,
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms": full, "ms_per_step": full, "scaling": "strong", "higher_is_better": True,
        "dtype": "f32/i32", "data": "synthetic power-law CSR (configs[2])",
        "config": {"workload": f"{rows} x {rows}, nnz {nnz}, rows split into "
                               f"{world} nnz-balanced blocks", "l2": "256 MB flush "
                               "before each step",
                   "exchange": exchange_name},
        "kernel_only": {"ms": loc, "GB/s": alg_bytes / (loc * 1e-3) / 1e9},
        "exchange_ms": gat,
        # the part of the step the exchange adds over the product alone
        "exchange_share": max(full - loc, 0.0) / full if full > 0 else None,
        "arms": {nm: {"ms_per_step": per[nm][0], "GB/s": alg_bytes / (per[nm][0] * 1e-3) / 1e9,
                      **({"exchange_ms": per[nm][2]} if not nm.endswith("overlap") else {})}
                 for nm in names},
        "y_check": ok, "nnz_per_rank": [int(v) for v in nz],
        "imbalance": float(nz.max() / max(float(nz.mean()), 1.0)),
        "roofline": {"bound": "hbm", "kernel": "spmv_csr_ranges (per rank) + x exchange",
                     "frac": alg_bytes / (full * 1e-3) / 1e9 / world / _peaks()["hbm_gbs"],
                     "peak": _peaks()["hbm_gbs"], "unit": "GB/s",
                     "note": "whole-job GB/s / N / per-GPU measured HBM"}}
    for arm in arms.values():
        arm.close()
    return res


def summarize(suite: dict | None) -> dict | None:
    """{routine: [value, unit, roofline frac, ms per call]} for the final line."""
    if not suite:
        return None
    out = {}
    for name, r in suite.items():
        if "error" in r:
            out[name] = ["error", r["error"][:120]]
            continue
        frac = (r.get("roofline") or {}).get("frac")
        out[name] = [float(f"{r['value']:.5g}"), r["unit"],
                     None if frac is None else round(float(frac), 3),
                     None if r.get("ms") is None else float(f"{r['ms']:.4g}")]
        if r.get("exchange_share") is not None:  # the x exchange's share of the SpMV step
            out[name].append({"exchange_share": round(float(r["exchange_share"]), 3)})
        if r.get("e2e"):  # the same metric through host buffers
            out[name].append({"e2e": float(f"{r['e2e']['value']:.4g}")})
        if (r.get("gather_ceiling") or {}).get("spmv_frac_of_ceiling") is not None:
            out[name].append({"frac_of_gather_ceiling":
                              round(float(r["gather_ceiling"]["spmv_frac_of_ceiling"]), 3)})
        if (r.get("row_gather_ceiling") or {}).get("spmm_frac_of_ceiling") is not None:
            out[name].append({"frac_of_row_gather_ceiling":
                              round(float(r["row_gather_ceiling"]["spmm_frac_of_ceiling"]), 3)})
        if (r.get("scatter_ceiling") or {}).get("spmv_t_frac_of_ceiling") is not None:
            out[name].append({"frac_of_scatter_ceiling":
                              round(float(r["scatter_ceiling"]["spmv_t_frac_of_ceiling"]), 3)})
    return out


def run_suite_sharded(names, args, torch, dist, world: int, rank: int, local: int) -> dict:
    """The multi-GPU paths at N > 1, every rank in the same order: each batch-sharded
    routine (1/N of the batch per rank, no collective on the data path) and the
    row-block SpMV with its x exchange."""
    out = {}
    for name in names:
        time.sleep(SUITE_GAP_S)
        try:
            if name == "spmv_dist":
                out[name] = spmv_dist_measure(args, torch, dist, world, rank, local)
            else:
                out[name] = sharded_measure(name, args, torch, dist, world)
        except Exception as e:  # recorded; the other routines still run
            out[name] = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()
    return out


SHARDED = ("fft", "gemm_bf16", "conv_bf16", "conv_f32", "softmax")


def sharded_measure(name: str, args, torch, dist, world: int) -> dict:
    """A batch-sharded suite routine across the ranks (strong scaling): each rank runs
    1/world of the batch (FFT transforms, GEMM batch entries, conv images, softmax rows)
    on its own GPU with no collective on the data path; every rank's timed region is
    bracketed by a barrier, the step time is the max over ranks and the value is the
    whole job's work over that time."""
    def barrier():
        dist.barrier()
        torch.cuda.synchronize()

    s = Suite(torch, max(3, args.steps // 4), args.warmup, False, args.scale)
    s.shard, s.barrier = world, barrier
    res = SUITE[name](s)
    ms = torch.tensor([res["ms"]], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_max = float(ms.item())
    total = res["value"] * res["ms"] / ms_max * world
    roof = res.get("roofline") or {}
    peak = roof.get("peak")
    return {"value": total, "unit": res["unit"], "ms": ms_max, "n_gpus": world,
            "per_rank_value": res["value"], "scaling": "strong", "config": res.get("config"),
            "sharding": f"batch / {world} per rank", "dtype": res.get("dtype"),
            "roofline": {"kernel": roof.get("kernel"), "bound": roof.get("bound"),
                         "per_gpu_achieved": total / world, "peak": peak,
                         "unit": roof.get("unit"),
                         "frac": total / world / peak if peak else None}}


def run_sharded(args) -> None:
    """`--routine NAME` under torchrun for a batch-sharded routine: its line on rank 0."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    res = sharded_measure(args.routine, args, torch, dist, world)
    if rank == 0:
        print(json.dumps({"routine": args.routine, **res}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--words", type=int, default=None,
                    help="override words per call (smaller cases for profiling)")
    ap.add_argument("--suite", default="all",
                    help="comma list of other routines to measure at N=1 "
                         f"({','.join(SUITE)}), 'all' or 'none'")
    ap.add_argument("--routine", default=None, choices=list(SUITE) + ["spmv_dist"],
                    help="measure only this routine and print its line (profiling); "
                         "spmv_dist runs under torchrun across the ranks")
    ap.add_argument("--scale", type=int, default=1,
                    help="divide the routine's batch/size by this factor (profiling)")
    args = ap.parse_args()
    if args.routine == "spmv_dist":
        run_spmv_dist(args)
        return
    if args.routine in SHARDED and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_sharded(args)
        return
    if args.routine:
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        res = run_suite([args.routine], args, torch)
        print(json.dumps({"routine": args.routine, **res[args.routine]}), flush=True)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.words:
        global N_WORDS, BYTES_PER_CALL, BYTES_PER_STEP
        N_WORDS = args.words
        BYTES_PER_CALL = 4 * N_WORDS
        BYTES_PER_STEP = 2 * BYTES_PER_CALL
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
