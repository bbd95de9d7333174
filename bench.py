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

``--impl reference`` times the reference's CPU path for the same workload: the
reference cannot be built off macOS, so it runs the oracle's restatement of its
host generator (oracle/philox.cpp) on all host cores, each step a bounded sample.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_WORDS = 1 << 30          # per call, per rank
SEED = 1234
BYTES_PER_CALL = 4 * N_WORDS
BYTES_PER_STEP = 2 * BYTES_PER_CALL
METRIC = ("RNG HBM GB/s: Philox4x32-10 curandGenerateUniform + curandGenerateNormal, "
          "2^30 fp32 each, seed 1234")
UNIT = "GB/s"
CPU_SAMPLE_WORDS = 1 << 30  # per call: the full config size (about 1.5 s on 16 host cores)


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


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
    base_offset = rank * 2 * N_WORDS
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

    assert L.curandDestroyGenerator(gen) == 0
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
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline() -> dict:
    """The reference's host generator path (oracle restatement), all host cores."""
    import oracle
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    oracle.generate_uniform(SEED, 0, CPU_SAMPLE_WORDS, threads=threads)
    oracle.generate_normal(SEED, 4 * CPU_SAMPLE_WORDS, CPU_SAMPLE_WORDS, 0.0, 1.0, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": 2 * 4 * CPU_SAMPLE_WORDS / dt / 1e9, "unit": UNIT, "cores": threads,
            "kind": "port", "seconds": dt,
            "sample": f"uniform + normal, 2^{CPU_SAMPLE_WORDS.bit_length() - 1} words each "
                      f"(1/{N_WORDS // CPU_SAMPLE_WORDS} of the config), oracle/philox.cpp"}


def run_reference(args) -> None:
    """Reference arm: the reference's CPU path for this workload, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        oracle.generate_uniform(SEED, 0, CPU_SAMPLE_WORDS // 8, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.generate_uniform(SEED, 0, CPU_SAMPLE_WORDS, threads=threads)
        oracle.generate_normal(SEED, 4 * CPU_SAMPLE_WORDS, CPU_SAMPLE_WORDS, 0.0, 1.0,
                               threads=threads)
    dt = (time.perf_counter() - t0) / args.steps
    value = 2 * 4 * CPU_SAMPLE_WORDS / dt / 1e9
    sample = (f"per step uniform + normal of 2^{CPU_SAMPLE_WORDS.bit_length() - 1} words each "
              f"(1/{N_WORDS // CPU_SAMPLE_WORDS} of the config)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32->f32",
        "data": "synthetic (counter-based RNG output)",
        "config": {"workload": "configs[1]: Philox4x32-10 uniform 2^30 + normal(0,1) 2^30, seed 1234",
                   "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample + "; oracle/philox.cpp restates "
                                   "libraries/rand/src/curand_context.mm:42-185 (the reference "
                                   "builds only on macOS/Metal)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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
    args = ap.parse_args()
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
