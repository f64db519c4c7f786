#!/usr/bin/env python3
"""Benchmark driver: GEMM TFLOPS and % of the measured UMMA dense peak on B200.

Default workload (BASELINE config 2's problem, the metric's configuration): bf16
GEMM M = N = K = 8192, A row-major, B N x K, D column-major bf16, seeded
uniform[-1,1) inputs, fp32 accumulation, CTA-pair (cta_group::2) 256x256x64
tiles, tile groups of 4 M-tiles.  One step = one GEMM (one launch of the library
kernel through the C ABI).  At N GPUs the GEMM is N-split with a fixed
8192-column slab per GPU (A replicated, B and D column-sliced, no collective on
the data path): weak scaling, value = total FLOPs / max-over-ranks time.

Beside the headline the line carries: the other BASELINE configurations (3-5,
fp8 at 8192^3, config 5 strong-scaled over the ranks with its all-gather and the
fused GEMM+gather timed separately), config 2 exactly as stated (the 1-SM
128x256x64 tile, stages 2..8), config 1 against the measured TMA/HBM read roof,
the reference's CUTLASS kernel family on the same operands, the reference's
single-CTA experiment, and the CPU baseline.

``--impl reference`` times the CPU path the reference lacks and the benchmark
plan names as its stand-in: the OpenMP fp32-accumulate host GEMM of oracle/
(cpu_gemm.c), on a bounded slab of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "microbench-blackwell_b200"

# Reference figures used in derived keys (cited, not measured here).
REF_UMMA_FLOP_PER_CLK_SM = {  # umma_throughput/tput_results_max.csv:13,49,175 (1SM M128 N256 SS; nvfp4 = MXF4 row)
    "bf16": 8152.85, "e4m3": 16344.5, "nvfp4": 32721.3}
DENSE_RATE_VS_BF16 = {"bf16": 1.0, "e4m3": 2.0, "nvfp4": 4.0}     # tcgen05 dense rates per SM per clock
REF_SINGLE_CTA_TFLOPS = {"bf16": 10.4596, "e4m3": 20.6377}  # cutlass_gemm_mainloop/results.csv:461,938

WORKLOADS = {
    # name: dtype, M, N (per GPU), K, knobs, inputs.  Knobs are the fastest measured on
    # B200 under the power cap (interleaved with CUTLASS's 2SM kernel, medians).
    "bf16_8192": dict(dtype="bf16", m=8192, n=8192, k=8192,
                      knobs=dict(tile_n=256, tile_k=64, stages=0, cta_group=2, raster_group=4),
                      a=("uniform", 1.0), b=("uniform", 1.0), config=2),
    "bf16_8192_1sm": dict(dtype="bf16", m=8192, n=8192, k=8192,
                          knobs=dict(tile_n=256, tile_k=64, stages=4, cta_group=1, raster_group=1),
                          a=("uniform", 1.0), b=("uniform", 1.0), config=2),
    "e4m3_16384_2sm": dict(dtype="e4m3", m=16384, n=16384, k=16384,
                           knobs=dict(tile_n=256, tile_k=128, stages=0, cta_group=2, raster_group=4),
                           a=("normal", 0.25), b=("normal", 0.25), config=3),
    "e4m3_8192": dict(dtype="e4m3", m=8192, n=8192, k=8192,
                      knobs=dict(tile_n=256, tile_k=128, stages=0, cta_group=2, raster_group=4),
                      a=("normal", 0.25), b=("normal", 0.25), config=3),
    "nvfp4_mlp": dict(dtype="nvfp4", m=8192, n=28672, k=8192,
                      knobs=dict(tile_n=256, tile_k=256, stages=0, cta_group=2, raster_group=-16),
                      a=("normal", 1.0), b=("normal", 1.0), config=4),
    # config 5: N is the whole problem's (57344); bench.py splits it over the ranks (strong scaling)
    "e4m3_nsplit": dict(dtype="e4m3", m=16384, n=57344, k=8192,
                        knobs=dict(tile_n=256, tile_k=128, stages=0, cta_group=2, raster_group=4),
                        a=("normal", 0.25), b=("normal", 0.02), config=5, split="strong"),
    "bf16_256": dict(dtype="bf16", m=256, n=256, k=256,
                     knobs=dict(tile_n=256, tile_k=64, stages=4, cta_group=1),
                     a=("uniform", 1.0), b=("uniform", 1.0), config=1),
}


def interleaved(stream, fns: dict, flop: float, rounds: int = 6, burst_s: float = 0.02, settle_s: float = 0.3):
    """Time callables (each enqueues one launch on `stream`) in alternating bursts of about
    burst_s, after a settle, so all see the same power-capped clock state.  Returns per name
    the median TFLOP/s and, against the first name, the median of the per-round ratios."""
    import torch
    names = list(fns)
    t0 = time.perf_counter()
    n_settle = 0
    while time.perf_counter() - t0 < settle_s or n_settle < 3:
        for f in fns.values():
            if f() != 0:
                return None
        stream.synchronize()
        n_settle += 1
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for f in fns.values():
        f()
    e1.record(stream)
    e1.synchronize()
    reps = max(2, int(burst_s * 1e3 / max(e0.elapsed_time(e1) / len(fns), 1e-3)))
    res = {k: [] for k in names}
    for _ in range(rounds):
        for k in names:
            e0.record(stream)
            for _ in range(reps):
                fns[k]()
            e1.record(stream)
            e1.synchronize()
            res[k].append(flop / (e0.elapsed_time(e1) / reps * 1e-3) / 1e12)
    first = names[0]
    return {k: {"tflops": statistics.median(v),
                "ratio_to_" + first: statistics.median(a / b for a, b in zip(v, res[first]))}
            for k, v in res.items()} | {"_rounds": rounds, "_launches_per_burst": reps}


def load_pkg():
    name = "microbench_blackwell_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "sm_max_mhz": 1965.0, "source": "fallback"}


def ncu_traffic(workload: str):
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(workload)
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Polls NVML (read-only) every few ms on this rank's GPU during the timed region."""

    REASONS = {"sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
               "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "hw_power_brake_slowdown": "nvmlClocksEventReasonHwPowerBrakeSlowdown"}

    def __init__(self, torch_device_index: int, period_s: float = 0.005):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml as N
            import torch
            N.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device_index).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self.h = N.nvmlDeviceGetHandleByUUID(uuid.encode() if isinstance(uuid, str) else uuid)
            self.N = N
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report no clocks rather than guess
            self.err = repr(e)
            self.max_mhz = None

    def _run(self):
        N = self.N
        masks = {k: getattr(N, v) for k, v in self.REASONS.items() if hasattr(N, v)}
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
                r = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, m in masks.items():
                    if r & m:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self) -> dict:
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ helpers
def dist_code(pkg, name: str) -> int:
    return pkg.UNIFORM if name == "uniform" else pkg.NORMAL


def dtype_code(pkg, name: str) -> int:
    return {"bf16": pkg.BF16, "e4m3": pkg.FP8_E4M3, "nvfp4": pkg.NVFP4}[name]


def elem_bytes(name: str) -> float:
    return {"bf16": 2.0, "e4m3": 1.0, "nvfp4": 0.5}[name]


class CpuGemm:
    """The oracle's OpenMP fp32-accumulate GEMM (oracle/cpu_gemm.c) on a slab of
    rows of A against B (dequantised fp32).  B is capped at 8192 rows so set-up
    stays bounded; the slab height is chosen once so one timed call takes
    about `target_s` seconds."""

    def __init__(self, wl: dict, seed: int = 0, target_s: float = 1.0):
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O
        self.O = O
        m, n, k, dt = wl["m"], wl["n"], wl["k"], wl["dtype"]
        self.m, self.k, self.dt = m, k, dt
        self.nb = min(n, 8192)
        self.wl = wl
        rows_max = min(m, 1024)
        if dt == "nvfp4":
            pb, sb = O.generate_nvfp4(self.nb, k, wl["b"][1], seed, 1)
            self.B = O.dequant_nvfp4(pb, sb, k)
            pa, sa = O.generate_nvfp4(max(128, (rows_max + 127) // 128 * 128), k, wl["a"][1], seed, 0)
            self.A = O.dequant_nvfp4(pa, sa, k)[:rows_max]
        else:
            odt = O.BF16 if dt == "bf16" else O.FP8_E4M3
            self.B = O.dequant(O.generate(self.nb, k, odt, 0 if wl["b"][0] == "uniform" else 1, wl["b"][1], seed, 1), odt)
            self.A = O.dequant(O.generate(rows_max, k, odt, 0 if wl["a"][0] == "uniform" else 1, wl["a"][1], seed, 0), odt)
        rows = 16
        while True:
            t = self._time(rows)
            if t * 2 > target_s or rows >= rows_max:
                break
            rows = min(rows_max, rows * 2)
        self.rows = rows

    def _time(self, rows: int) -> float:
        import numpy as np
        A = np.ascontiguousarray(self.A[:rows])
        t0 = time.perf_counter()
        self.O.gemm_omp_f32(A, self.B)
        return time.perf_counter() - t0

    def step(self) -> float:
        """TFLOPS of one timed slab."""
        t = self._time(self.rows)
        return 2.0 * self.rows * self.nb * self.k / t / 1e12

    def describe(self, secs: float) -> dict:
        return {"unit": "TFLOPS", "cores": self.O.num_threads(), "kind": "port",
                "sample": f"{self.rows} x {self.nb} x {self.k} row slab of the {self.m}x{self.wl['n']}x{self.k} "
                          f"{self.dt} GEMM (oracle/cpu_gemm.c, OpenMP fp32 accumulate over dequantised inputs), "
                          f"{secs:.1f} s of timed CPU work"}


def cpu_gemm_sample(wl: dict, budget_s: float, seed: int = 0):
    g = CpuGemm(wl, seed=seed, target_s=1.0)
    vals = []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or not vals:
        vals.append(g.step())
    info = g.describe(time.perf_counter() - t0)
    info["value"] = statistics.median(vals)
    return info, time.perf_counter() - t0


def host_note_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ reference arm
def run_reference(args, wl, rank: int, world: int):
    if rank != 0:
        return
    g = CpuGemm(wl, seed=args.seed, target_s=1.0)
    per_step = []
    t0 = time.perf_counter()
    for i in range(args.warmup + args.steps):
        v = g.step()
        if i >= args.warmup:
            per_step.append(v)
    value = statistics.median(per_step)
    info = g.describe(time.perf_counter() - t0)
    info["value"] = value
    line = {"metric": "GEMM TFLOPS", "impl": "reference", "value": value, "unit": "TFLOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": wl["dtype"], "data": "synthetic (seeded)",
            "config": config_block(wl, world, args),
            "cpu_baseline": info,
            "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_cutlass_single_cta": run_reference_cutlass_single_cta(wl),
            "note": "the reference has no CPU GEMM; this arm times oracle/cpu_gemm.c (OpenMP host GEMM) "
                    "on a row slab, host cores only"}
    print(json.dumps(line), flush=True)


def effective_knobs(wl, args) -> dict:
    knobs = dict(wl["knobs"])
    for key in ("stages", "tile_n", "tile_k", "cta_group", "raster_group"):
        v = getattr(args, key, None)
        if v is not None:
            knobs[key] = v
    return knobs


def config_block(wl, world, args):
    strong = wl.get("split") == "strong"
    return {"workload": args.workload, "baseline_config": wl["config"],
            "m": wl["m"], "n_per_gpu": wl["n"] // world if strong else wl["n"],
            "n_total": wl["n"] if strong else wl["n"] * world, "k": wl["k"],
            "dtype": wl["dtype"], **effective_knobs(wl, args),
            "parallelism": f"nsplit{world}" if world > 1 else "single",
            "layout": "A row-major MxK, B NxK (K-major), D column-major bf16",
            "l2": "inputs larger than L2 (126 MB), no flush" if wl["m"] * wl["k"] * elem_bytes(wl["dtype"]) +
                  wl["n"] * wl["k"] * elem_bytes(wl["dtype"]) > 126e6 else "inputs fit in L2 (latency-bound KAT)"}


# ------------------------------------------------------------------ our arm
def slab_for(wl, knobs, world, rank):
    """N-split slab of this rank: strong-scaled workloads split their own N over the ranks,
    the others give every rank a slab of the per-GPU N (weak scaling)."""
    from microbench_blackwell_b200 import nsplit
    n_total = wl["n"] if wl.get("split") == "strong" else wl["n"] * world
    return nsplit.partition(n_total, world, rank, align=knobs.get("tile_n", 256))


def make_gemm(pkg, wl, knobs, slab, dev, stream, seed):
    import torch
    dt = dtype_code(pkg, wl["dtype"])
    with torch.cuda.stream(stream):
        ops = pkg.make_operands(dt, wl["m"], slab.n_local, wl["k"], seed=seed,
                                a_dist=dist_code(pkg, wl["a"][0]), a_scale=wl["a"][1],
                                b_dist=dist_code(pkg, wl["b"][0]), b_scale=wl["b"][1],
                                n0=slab.n0, device=dev, stream=stream.cuda_stream)
    clock_buf = torch.zeros(2, dtype=torch.int64, device=dev)     # [cycles, ns] summed over CTAs and launches
    g = pkg.make_args(dtype=dt, m=ops.m, n=ops.n, k=ops.k, a=ops.a.data_ptr(), b=ops.b.data_ptr(),
                      d=ops.d.data_ptr(), sfa=None if ops.sfa is None else ops.sfa.data_ptr(),
                      sfb=None if ops.sfb is None else ops.sfb.data_ptr(), clock_out=clock_buf.data_ptr(), **knobs)
    rc, info = pkg.query(g)
    if rc != pkg.OK:
        raise SystemExit(f"cannot implement: {info.reason.decode()}")
    return ops, g, clock_buf, info


def run_ours(args, wl, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist
    pkg = load_pkg()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    st = stream.cuda_stream
    knobs = effective_knobs(wl, args)
    slab = slab_for(wl, knobs, world, rank)
    ops, gargs, clock_buf, info = make_gemm(pkg, wl, knobs, slab, dev, stream, args.seed)
    m, n, k = ops.m, ops.n, ops.k
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    gargs.status = status.data_ptr()
    L = pkg.lib()
    launch = L.gemm_sm100a_launch
    argp = C.byref(gargs)
    sp = C.c_void_p(st)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # warm-up
    for _ in range(args.warmup):
        if launch(argp, sp) != 0:
            raise SystemExit("launch failed")
    stream.synchronize()
    rc, detail = pkg.read_status(status.data_ptr(), st)
    if rc != 0:
        raise SystemExit(f"device status error 0x{detail & 0xffffffff:08x}")

    # timed region: K launches bracketed by barrier + synchronize, events on the launching stream
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize(dev)
    step_clocks = torch.zeros((args.steps, 2), dtype=torch.int64, device=dev)
    with sampler:
        start.record(stream)
        launch_recording_clocks(launch, gargs, sp, args.steps, step_clocks)
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(dev)
    barrier()
    ms = start.elapsed_time(end)
    from microbench_blackwell_b200 import nsplit
    ms_max = nsplit.max_over_ranks(ms, device=dev)
    rc, detail = pkg.read_status(status.data_ptr(), st)
    if rc != 0:
        raise SystemExit(f"device status error 0x{detail & 0xffffffff:08x}")
    flop = pkg.flops(m, n, k)
    ms_per_step = ms_max / args.steps
    value = flop * world / (ms_per_step * 1e-3) / 1e12
    achieved = flop / (ms / args.steps * 1e-3) / 1e12          # this rank's kernel, per launch
    clocks = sampler.summary()
    clocks["kernel_sm_mhz"] = kernel_mhz(step_clocks)
    gargs.status = None
    gargs.clock_out = None

    # ---------------------------------------------------------- the reference's kernel family, same box
    ref_full = run_reference_cutlass_full(pkg, ops, gargs, stream, wl["dtype"], args.steps) if world == 1 else None

    # ---------------------------------------------------------- end to end (host buffers)
    e2e = run_e2e(pkg, ops, gargs, dev, stream, args, world, local_rank)
    del ops
    torch.cuda.empty_cache()

    # ---------------------------------------------------------- the other BASELINE configurations
    per_dtype = None
    if not args.no_per_dtype:
        per_dtype = run_per_dtype(pkg, args, dev, stream, world, rank, local_rank)

    extras = {}
    if world == 1 and not args.no_per_dtype:
        extras["config2_stage_sweep"] = run_stage_sweep(pkg, args, dev, stream)
        extras["tma_hbm_probe"] = run_tma_probe(pkg, dev, stream)
        extras["config1_bf16_256"] = run_config1(pkg, args, dev, stream, extras["tma_hbm_probe"])

    # ---------------------------------------------------------- single-CTA mainloop (reference experiment)
    single = run_single_cta(pkg, wl, dev, stream) if (rank == 0 and wl["dtype"] in SINGLE_CTA_CFG) else None

    if rank != 0:
        return
    peaks = measured_peaks()
    umma_peak = measured_umma_peak(pkg, wl["dtype"], dev)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu, _ = cpu_gemm_sample(wl, budget_s=12.0, seed=args.seed)
    peak = peaks["bf16_tflops"] * DENSE_RATE_VS_BF16[wl["dtype"]]
    peak_src = f"{peaks['source']} cuBLAS bf16 burst (MEASURED_PEAKS.json)" + (
        "" if wl["dtype"] == "bf16" else f" x {DENSE_RATE_VS_BF16[wl['dtype']]:.0f} (dense {wl['dtype']} rate), derived")
    line = {
        "metric": "GEMM TFLOPS", "value": value, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "strong" if wl.get("split") == "strong" else "weak",
        "vs_baseline": None,
        "dtype": wl["dtype"], "data": "synthetic (seeded, generated on device)",
        "config": config_block(wl, world, args),
        "roofline": {"bound": "tensor", "achieved": achieved,
                     "peak": peak,
                     "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "peak_source": peak_src,
                     "traffic": ncu_traffic(args.workload),
                     "algorithmic_bytes": m * k * elem_bytes(wl["dtype"]) + n * k * elem_bytes(wl["dtype"]) + m * n * 2},
        "sol_umma": sol_block(achieved, umma_peak, clocks["kernel_sm_mhz"], wl["dtype"]),
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "cpu_baseline": cpu,
        "single_cta": single,
        "reference_cutlass_full": ref_full,
        "per_dtype": per_dtype,
        **extras,
        "kernel": {"grid": info.grid_ctas, "stages": info.stages, "tile": [info.tile_m, info.tile_n, info.tile_k],
                   "smem_bytes": info.smem_bytes, "tmem_columns": info.tmem_columns,
                   "epilogue_staging_buffers": info.epilogue_staging_buffers},
    }
    print(json.dumps(line), flush=True)


PER_DTYPE = [
    # (label, workload): configs 3-5 and fp8 at 8192^3 (north_star's >= 90 % target)
    ("e4m3_config3", "e4m3_16384_2sm"),
    ("e4m3_8192", "e4m3_8192"),
    ("nvfp4_config4", "nvfp4_mlp"),
    ("e4m3_nsplit_config5", "e4m3_nsplit"),
]


def kernel_mhz(clock_buf):
    """Effective SM clock over the launches that recorded into clock_buf ([n, 2]: the cycles
    and ns every CTA of a launch adds, the kernel's own clock64 / %globaltimer record): sum of
    cycles over sum of time.  Sampled NVML clocks miss power-cap throttling."""
    v = clock_buf.view(-1, 2).cpu().double()
    cyc, ns = float(v[:, 0].sum()), float(v[:, 1].sum())
    return 1000.0 * cyc / ns if ns > 0 else None


def launch_recording_clocks(launch, g, sp, steps, clock_buf):
    """Enqueue `steps` launches of `g`, each adding its CTAs' cycles and ns into its own
    (zeroed) row of clock_buf ([steps, 2] int64): the timed launches' mean clock."""
    base = clock_buf.data_ptr()
    for i in range(steps):
        g.clock_out = base + 16 * i
        launch(C.byref(g), sp)


def pct_at_clock(tflops, umma_peak, mhz):
    """% of the probe's FLOP/clk/SM x 148 SMs at the GEMM's own clock: the per-clock efficiency."""
    if not mhz:
        return None
    return 100.0 * tflops / (umma_peak["flop_per_clk_per_sm"] * 148 * mhz * 1e6 / 1e12)


def sol_block(tflops_per_gpu, umma_peak, gemm_mhz, dtype):
    """SOL against the own tcgen05 probe.  Primary: the per-clock efficiency (TFLOP/s over
    the probe's FLOP/clk/SM x 148 SMs at the GEMM's own measured clock), which cannot exceed
    100 %.  The ratio to the whole-GPU probe at the probe's clock is secondary: the probe,
    a pure tensor load, is power-capped to a different clock than a GEMM."""
    return {"pct_umma_peak_at_gemm_clock": pct_at_clock(tflops_per_gpu, umma_peak, gemm_mhz),
            "gemm_sm_mhz": gemm_mhz,
            "umma_flop_per_clk_per_sm": umma_peak["flop_per_clk_per_sm"],
            "reference_flop_per_clk_per_sm": REF_UMMA_FLOP_PER_CLK_SM[dtype],
            "pct_umma_peak_at_max_clock": 100.0 * tflops_per_gpu / (umma_peak["flop_per_clk_per_sm"] * 148 * SM_MAX_MHZ * 1e6 / 1e12),
            "secondary_pct_of_whole_gpu_probe": 100.0 * tflops_per_gpu / umma_peak["tflops"],
            "whole_gpu_probe_tflops": umma_peak["tflops"], "whole_gpu_probe_sm_mhz": umma_peak["sm_mhz"],
            "probe": umma_peak["source"]}


def measured_umma_peak(pkg, dtype_name: str, dev) -> dict:
    """Whole-GPU tcgen05 dense peak of this GPU for one dtype (CTA pairs on every SM,
    non-zero operands), from the library's probe -- the SOL denominator."""
    import torch
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    r = pkg.umma_peak(dtype_code(pkg, dtype_name), cta_group=2, num_ctas=sms - sms % 2, depth=256, iters=1500,
                      device=dev)
    r["source"] = "gemm_sm100a_umma_peak, whole GPU, M256 N256 pairs, non-zero operands"
    return r


def run_per_dtype(pkg, args, dev, stream, world, rank, local_rank):
    """Time the other BASELINE configurations (fewer steps) for the per-dtype metric."""
    import torch
    import torch.distributed as dist
    from microbench_blackwell_b200 import nsplit
    out = {}
    steps = max(5, min(args.steps, 20))
    L = pkg.lib()
    sp = C.c_void_p(stream.cuda_stream)
    for label, name in PER_DTYPE:
        wl = WORKLOADS[name]
        knobs = dict(wl["knobs"])
        slab = slab_for(wl, knobs, world, rank)
        ops, g, clock_buf, _ = make_gemm(pkg, wl, knobs, slab, dev, stream, args.seed)
        # Untimed settle (>= 3 launches, ~0.25 s): the clock reaches this configuration's
        # own power-capped steady state instead of the previous configuration's.
        settle_end = time.perf_counter() + 0.25
        n_settle = 0
        while n_settle < 3 or time.perf_counter() < settle_end:
            for _ in range(4):
                L.gemm_sm100a_launch(C.byref(g), sp)
            n_settle += 4
            stream.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        step_clocks = torch.zeros((steps, 2), dtype=torch.int64, device=dev)
        s0.record(stream)
        launch_recording_clocks(L.gemm_sm100a_launch, g, sp, steps, step_clocks)
        s1.record(stream)
        s1.synchronize()
        ms = nsplit.max_over_ranks(s0.elapsed_time(s1) / steps, device=dev)
        gemm_mhz = kernel_mhz(step_clocks)
        flop_total = pkg.flops(ops.m, ops.n, ops.k) * world
        tf = flop_total / (ms * 1e-3) / 1e12
        per_gpu = tf / world
        rec = {"workload": name, "baseline_config": wl["config"],
               "scaling": "strong" if wl.get("split") == "strong" else "weak",
               "m": ops.m, "n_total": slab.n_total, "n_per_gpu": ops.n, "k": ops.k, "knobs": knobs, "steps": steps,
               "ms_per_step": ms, "tflops": tf, "tflops_per_gpu": per_gpu}
        g.clock_out = None
        rec["reference_cutlass_full"] = run_reference_cutlass_full(pkg, ops, g, stream, wl["dtype"], steps) if world == 1 else None
        if wl.get("split") == "strong" and world > 1:
            rec["gather"] = run_nsplit_gather(pkg, ops, g, slab, dev, stream, world, rank, local_rank, ms)
        peak = measured_umma_peak(pkg, wl["dtype"], dev)
        rec["sol_umma"] = sol_block(per_gpu, peak, gemm_mhz, wl["dtype"])
        rec["pct_umma_peak_at_gemm_clock"] = rec["sol_umma"]["pct_umma_peak_at_gemm_clock"]
        out[label] = rec
        del ops
        torch.cuda.empty_cache()
    return out


def run_nsplit_gather(pkg, ops, g, slab, dev, stream, world, rank, local_rank, gemm_ms):
    """Config 5's optional output gather, timed three ways at N GPUs (max over ranks):
    the GEMM alone (gemm_ms), ncclAllGather of this configuration's own bf16 D slices,
    and the fused GEMM + gather (gemm_sm100a_launch_gather: the epilogue also stores each
    staged block into every other GPU's full D, reached by CUDA IPC over NVLink).  The
    fused result is checked bit for bit against the NCCL-gathered D."""
    import torch
    import torch.distributed as dist
    from microbench_blackwell_b200 import nsplit
    out = {"gemm_ms": gemm_ms}
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        full = nsplit.gather_columns(ops.d, slab.n_total)                 # warm-up
        stream.synchronize()
        times = []
        for _ in range(3):
            dist.barrier(device_ids=[local_rank])
            ev0.record(stream)
            full = nsplit.gather_columns(ops.d, slab.n_total)
            ev1.record(stream)
            ev1.synchronize()
            times.append(ev0.elapsed_time(ev1))
    ag_ms = nsplit.max_over_ranks(min(times), device=dev)
    recv = (world - 1) * ops.d.numel() * ops.d.element_size()
    out["nccl_allgather"] = {"ms": ag_ms, "bytes_received_per_rank": recv,
                             "GBps_per_rank": recv / (ag_ms * 1e-3) / 1e9,
                             "gemm_plus_allgather_ms": gemm_ms + ag_ms}
    try:
        out["fused"] = nsplit.fused_gather_timing(pkg, g, ops, slab, full, stream, dev, local_rank)
    except Exception as e:       # a box without peer access between the ranks' GPUs
        out["fused"] = {"unavailable": repr(e)[:200]}
        dist.barrier(device_ids=[local_rank])
    del full
    return out


def run_stage_sweep(pkg, args, dev, stream):
    """BASELINE config 2 exactly as stated: the 1-SM 128x256x64 tile at 8192^3 with stages
    swept 2..8 (interleaved bursts, medians).  Stages that do not fit in shared memory are
    reported as the can't-implement rows of the reference's sweep (results.csv:462-465)."""
    import torch
    from microbench_blackwell_b200 import nsplit
    wl = WORKLOADS["bf16_8192_1sm"]
    slab = nsplit.partition(wl["n"], 1, 0)
    ops, g0, _, _ = make_gemm(pkg, wl, dict(wl["knobs"]), slab, dev, stream, args.seed)
    L = pkg.lib()
    sp = C.c_void_p(stream.cuda_stream)
    rows, fns, keep = [], {}, []
    for s in range(2, 9):
        g = pkg.make_args(dtype=ops.dtype, m=ops.m, n=ops.n, k=ops.k, a=ops.a.data_ptr(), b=ops.b.data_ptr(),
                          d=ops.d.data_ptr(), **dict(wl["knobs"], stages=s))
        rc, info = pkg.query(g)
        if rc != pkg.OK:
            rows.append({"stages": s, "cannot_implement": info.reason.decode()})
            continue
        keep.append(g)
        fns[f"S{s}"] = (lambda g=g: L.gemm_sm100a_launch(C.byref(g), sp))
        rows.append({"stages": s})
    res = interleaved(stream, fns, pkg.flops(ops.m, ops.n, ops.k), rounds=4)
    for r in rows:
        key = f"S{r['stages']}"
        if res and key in res:
            r["tflops"] = res[key]["tflops"]
    del ops
    torch.cuda.empty_cache()
    return {"tile": [128, 256, 64], "cta_group": 1, "rows": rows}


def run_tma_probe(pkg, dev, stream):
    """The TMA-2D HBM read roof (the reference's tma2d_throughput sweep points, 2 GiB read
    once after an L2 flush): the memory-side denominator for config 1 and skinny shapes."""
    import torch
    buf = torch.empty(2 << 30, dtype=torch.uint8, device=dev)
    flush = torch.empty(pkg.L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    pts = []
    with torch.cuda.stream(stream):
        for rows, stages in ((256, 1), (128, 1), (64, 2), (32, 4), (16, 4)):
            best = max((pkg.tma_read_probe(buf, box_rows=rows, stages=stages, flush=flush, device=dev)
                        for _ in range(2)), key=lambda r: r["GBps"])
            pts.append({"box": [128, rows], "stages": stages, "bytes_in_flight_per_sm": best["bytes_in_flight_per_sm"],
                        "GBps": best["GBps"], "cycles_per_tma": best["cycles_per_tma"]})
    # L2-resident read rate of the probe (one warp per SM): a 96 MiB tensor (under the
    # 126 MB L2) read three times without a flush, the last pass timed by the CTAs' own
    # counters.  One warp does not saturate L2 (NVFP4 config 4 moves more under ncu at 57 %
    # of L2 throughput), so this is a lower bound on the L2 roof, not the roof.
    l2buf = torch.randint(0, 255, (96 << 20,), dtype=torch.uint8, device=dev)
    l2pts = []
    with torch.cuda.stream(stream):
        for rows, stages in ((128, 3), (64, 6)):
            r = [pkg.tma_read_probe(l2buf, box_rows=rows, stages=stages, device=dev) for _ in range(3)][-1]
            l2pts.append({"box": [128, rows], "stages": stages, "bytes_per_clk_per_sm": r["bytes_per_clk_per_cta"],
                          "sm_mhz": r["sm_mhz"], "GBps": r["GBps_in_kernel"]})
    del buf, flush, l2buf
    torch.cuda.empty_cache()
    top = max(pts, key=lambda r: r["GBps"])
    return {"points": pts, "roof_GBps": top["GBps"], "l2_resident_one_warp": l2pts,
            "reference_roof_GBps": 7260.0, "reference_source": "tma2d_throughput/tma2d_tput_results.csv:25 (ncu DRAM counter)",
            "method": "bytes / CUDA-event time of one probe launch over 2 GiB after an L2 flush"}


def run_config1(pkg, args, dev, stream, probe):
    """BASELINE config 1 (bf16 256^3), latency-bound: per-launch device time from a
    stream of back-to-back launches and from a CUDA graph of them, against the time the
    384 KiB of A, B and D take at the measured TMA read roof."""
    import torch
    from microbench_blackwell_b200 import nsplit
    wl = WORKLOADS["bf16_256"]
    ops, g, _, _ = make_gemm(pkg, wl, dict(wl["knobs"]), nsplit.partition(256, 1, 0), dev, stream, args.seed)
    L = pkg.lib()
    sp = C.c_void_p(stream.cuda_stream)
    n = 2000
    for _ in range(20):
        L.gemm_sm100a_launch(C.byref(g), sp)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        L.gemm_sm100a_launch(C.byref(g), sp)
    e1.record(stream)
    e1.synchronize()
    us_stream = e0.elapsed_time(e1) / n * 1e3
    out = {"us_per_launch_stream": us_stream}
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="relaxed"):
            for _ in range(100):
                L.gemm_sm100a_launch(C.byref(g), C.c_void_p(torch.cuda.current_stream().cuda_stream))
        with torch.cuda.stream(stream):              # replay() launches on the current stream
            graph.replay()
            stream.synchronize()
            e0.record(stream)
            for _ in range(n // 100):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
        out["us_per_launch_graph"] = e0.elapsed_time(e1) / n * 1e3
        del graph
    except Exception as e:
        out["graph"] = {"unavailable": repr(e)[:200]}
    us = min(v for k, v in out.items() if k.startswith("us_per"))
    bytes_moved = 3 * 256 * 256 * 2
    out.update({"tflops": pkg.flops(256, 256, 256) / (us * 1e-6) / 1e12,
                "bytes_moved": bytes_moved, "GBps": bytes_moved / (us * 1e-6) / 1e9,
                "memory_roof_us": bytes_moved / (probe["roof_GBps"] * 1e9) * 1e6,
                "note": "2 output tiles on 2 SMs: bound by launch and pipeline latency, not by HBM or tensor throughput"})
    del ops
    torch.cuda.empty_cache()
    return out


def run_e2e(pkg, ops, gargs, dev, stream, args, world, local_rank):
    """The same GEMM through the C ABI with host buffers: every step copies its A and B
    from pinned host memory and reads its D back.  Two device buffer sets and separate
    copy streams let step i's upload overlap step i-1's GEMM and step i-2's download
    (the copy engines and the SMs work concurrently); every copy is inside the timed
    region."""
    import torch
    import torch.distributed as dist
    steps = max(4, min(args.steps, 12))
    ha = torch.empty_like(ops.a, device="cpu").pin_memory()
    hb = torch.empty_like(ops.b, device="cpu").pin_memory()
    ha.copy_(ops.a); hb.copy_(ops.b)
    hsa = hsb = None
    if ops.sfa is not None:
        hsa = torch.empty_like(ops.sfa, device="cpu").pin_memory(); hsa.copy_(ops.sfa)
        hsb = torch.empty_like(ops.sfb, device="cpu").pin_memory(); hsb.copy_(ops.sfb)
    hd = [torch.empty_like(ops.d, device="cpu").pin_memory() for _ in range(2)]
    # Two device buffer sets (set 0 reuses the bench's operands).
    sets = [(ops.a, ops.b, ops.sfa, ops.sfb, ops.d),
            (torch.empty_like(ops.a), torch.empty_like(ops.b),
             None if ops.sfa is None else torch.empty_like(ops.sfa),
             None if ops.sfb is None else torch.empty_like(ops.sfb), torch.empty_like(ops.d))]
    args_ = []
    for a, b, sa, sb, d in sets:
        g = pkg.make_args(dtype=ops.dtype, m=ops.m, n=ops.n, k=ops.k, a=a.data_ptr(), b=b.data_ptr(), d=d.data_ptr(),
                          sfa=None if sa is None else sa.data_ptr(), sfb=None if sb is None else sb.data_ptr(),
                          **{f: getattr(gargs, f) for f in ("tile_n", "tile_k", "stages", "cta_group", "raster_group")})
        args_.append(g)
    h2d_bytes = ha.numel() * ha.element_size() + hb.numel() * hb.element_size() + \
        (0 if hsa is None else hsa.numel() + hsb.numel())
    d2h_bytes = hd[0].numel() * hd[0].element_size()
    L = pkg.lib()
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    loaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    drained = [torch.cuda.Event() for _ in range(2)]
    for e in drained:
        e.record(down)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize(dev)
    start.record(stream)
    up.wait_event(start)
    for i in range(steps):
        j = i % 2
        a, b, sa, sb, d = sets[j]
        with torch.cuda.stream(up):
            up.wait_event(computed[j]) if i >= 2 else None       # set j free of step i-2's GEMM
            a.copy_(ha, non_blocking=True)
            b.copy_(hb, non_blocking=True)
            if sa is not None:
                sa.copy_(hsa, non_blocking=True)
                sb.copy_(hsb, non_blocking=True)
            loaded[j].record(up)
        stream.wait_event(loaded[j])
        stream.wait_event(drained[j])                             # D of step i-2 read back
        L.gemm_sm100a_launch(C.byref(args_[j]), C.c_void_p(stream.cuda_stream))
        computed[j].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(computed[j])
            hd[j].copy_(d, non_blocking=True)
            drained[j].record(down)
    stream.wait_stream(down)
    stream.wait_stream(up)
    end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / steps
    flop = pkg.flops(ops.m, ops.n, ops.k) * world
    ok = torch.equal(hd[(steps - 1) % 2].to(dev), sets[(steps - 1) % 2][4])
    return {"value": flop / (ms_step * 1e-3) / 1e12, "unit": "TFLOPS", "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes, "steps": steps, "ms_per_step": ms_step, "readback_matches_device": ok,
            "path": "pinned host A,B -> gemm_sm100a_launch -> pinned host D; upload, GEMM and download on "
                    "three streams with two device buffer sets (overlapped, all copies timed)"}


SINGLE_CTA_CFG = {"bf16": (128, 256, 64, 4, 0), "e4m3": (128, 256, 128, 0, 1)}


def parse_csv_line(text: str):
    line = [l for l in text.strip().splitlines() if l and not l.startswith("#")][-1]
    f = line.split(",")
    return {"M": int(f[0]), "N": int(f[1]), "K": int(f[2]), "tile": [int(f[3]), int(f[4]), int(f[5])],
            "stages": int(f[6]), "dtype": f[7], "time_ms": float(f[8]), "tflops": float(f[9])}


def run_single_cta(pkg, wl, dev, stream):
    """The reference experiment through our drop-in harness binary, run exactly as
    the reference runs its own: no argv, one CTA, M=TILE_M, N=TILE_N, K=131072,
    zero-filled inputs, 1 warm-up + 20 timed (cutlass_gemm_bench.cu:158-257)."""
    import subprocess
    cfg = SINGLE_CTA_CFG[wl["dtype"]]
    binp = PKG_DIR / "harness" / "bin" / ("gemm_bench_%d_%d_%d_s%d_d%d" % cfg)
    if not binp.exists():
        return {"error": f"{binp.name} not built"}
    r = subprocess.run([str(binp)], capture_output=True, text=True, timeout=120)
    if r.returncode != 0:
        return {"error": r.stderr.strip()[-200:]}
    out = parse_csv_line(r.stdout)
    out["reference_published_tflops"] = REF_SINGLE_CTA_TFLOPS[wl["dtype"]]
    out["ratio_vs_published"] = out["tflops"] / REF_SINGLE_CTA_TFLOPS[wl["dtype"]]
    out["binary"] = binp.name
    return out


SM_MAX_MHZ = 1965.0   # B200 clocks.max.sm

# Kernels of oracle/_ref/libcutlass_ref.so (oracle/cutlass_ref.cu) timed beside ours, per dtype.
CUTLASS_REF_KERNELS = {
    "bf16": {0: "CUTLASS SM100 1SM 128x256x64, 4 stages (the reference's best point, cutlass_gemm_mainloop/results.csv:461)"},
    "e4m3": {1: "CUTLASS SM100 1SM 128x256x128, auto stages (cutlass_gemm_mainloop/results.csv:938)"},
    "nvfp4": {4: "CUTLASS SM100 1SM Nvf4 128x256x256, auto stages"},
}


def run_reference_cutlass_full(pkg, ops, gargs, stream, dtype, steps):
    """The reference's own CUTLASS kernel family (oracle/_ref/libcutlass_ref.so, the
    cutlass_gemm_bench.cu:101-156 type chain, 1SM schedule, plus its Nvf4 form) on the same
    operands over the whole GPU, interleaved with ours in alternating bursts (6 rounds,
    medians) so every kernel sees the same power-capped clock state.  For bf16 the vendor
    GEMM (cuBLAS through torch.mm) joins the same bursts (`vendor_cublas`).  Informational:
    the reference itself runs one CTA."""
    import torch
    kernels = CUTLASS_REF_KERNELS.get(dtype)
    lib = ROOT / "oracle" / "_ref" / "libcutlass_ref.so"
    if kernels is None:
        return None
    if not lib.exists():
        return {"unavailable": "oracle/_ref/libcutlass_ref.so not built (oracle/ref_build.sh)"}
    R = C.CDLL(str(lib))
    R.cutlass_ref_run.restype = C.c_int
    R.cutlass_ref_run.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
    L = pkg.lib()
    sp = C.c_void_p(stream.cuda_stream)
    d_ref = torch.empty_like(ops.d)
    sfa = None if ops.sfa is None else ops.sfa.data_ptr()
    sfb = None if ops.sfb is None else ops.sfb.data_ptr()
    fns = {"ours": lambda: L.gemm_sm100a_launch(C.byref(gargs), sp)}
    out = {"kernels": {}}
    for kid, desc in kernels.items():
        def cut(kid=kid):
            return R.cutlass_ref_run(kid, ops.a.data_ptr(), ops.b.data_ptr(), sfa, sfb, d_ref.data_ptr(),
                                     ops.m, ops.n, ops.k, 0, sp)
        rc = cut()
        if rc != 0:
            out["kernels"][desc] = {"unavailable": f"cutlass_ref_run returned {rc}"}
            continue
        fns[desc] = cut
    cublas = "cuBLAS (torch.mm, bf16)"
    if dtype == "bf16":
        # The vendor GEMM on the same operands, as a comparison only: D^T = B . A^T
        # in D's own layout (ops.d is N x M row-major, i.e. M x N column-major).
        d_blas = torch.empty_like(ops.d)

        def vendor():
            with torch.cuda.stream(stream):
                torch.mm(ops.b, ops.a.t(), out=d_blas)
            return 0
        fns[cublas] = vendor
    stream.synchronize()
    res = interleaved(stream, fns, pkg.flops(ops.m, ops.n, ops.k))
    if res is None:
        return {"unavailable": "launch failed"}
    if cublas in fns:
        out["vendor_cublas"] = {"tflops": res[cublas]["tflops"], "ours_over_cublas": 1.0 / res[cublas]["ratio_to_ours"]}
        del fns[cublas]
    out["rounds"] = res["_rounds"]
    out["launches_per_burst"] = res["_launches_per_burst"]
    out["tflops_ours_interleaved"] = res["ours"]["tflops"]
    best = None
    for desc in fns:
        if desc == "ours":
            continue
        rec = {"tflops_cutlass": res[desc]["tflops"], "ours_over_cutlass": 1.0 / res[desc]["ratio_to_ours"]}
        out["kernels"][desc] = rec
        if best is None or rec["tflops_cutlass"] > best[1]["tflops_cutlass"]:
            best = (desc, rec)
    if best is not None:
        out["best_cutlass_kernel"] = best[0]
        out["tflops_cutlass"] = best[1]["tflops_cutlass"]
        out["ours_over_best_cutlass"] = best[1]["ours_over_cutlass"]
    return out


def run_reference_cutlass_single_cta(wl):
    """The reference's own benchmark binary (oracle/_ref, built from
    cutlass_gemm_mainloop/cutlass_gemm_bench.cu) on this box, same config."""
    import subprocess
    cfg = SINGLE_CTA_CFG.get(wl["dtype"])
    if cfg is None:
        return None
    binp = ROOT / "oracle" / "_ref" / ("cutlass_bench_%d_%d_%d_s%d_d%d" % cfg)
    if not binp.exists():
        return {"unavailable": f"{binp.name} not built (oracle/ref_build.sh needs the reference tree)"}
    try:
        r = subprocess.run([str(binp)], capture_output=True, text=True, timeout=120)
    except Exception as e:  # no GPU on this host, etc.
        return {"unavailable": repr(e)[:200]}
    if r.returncode != 0:
        return {"unavailable": (r.stderr or r.stdout).strip()[-200:]}
    out = parse_csv_line(r.stdout)
    out["binary"] = binp.name
    out["reference_published_tflops"] = REF_SINGLE_CTA_TFLOPS[wl["dtype"]]
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="bf16_8192")
    ap.add_argument("--stages", type=int, default=None)
    ap.add_argument("--tile-n", type=int, default=None)
    ap.add_argument("--tile-k", type=int, default=None)
    ap.add_argument("--cta-group", type=int, default=None, choices=[1, 2])
    ap.add_argument("--raster-group", type=int, default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-dtype", action="store_true", help="skip the other BASELINE configurations")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}; using WORLD_SIZE", file=sys.stderr)

    if args.impl == "reference":
        run_reference(args, wl, rank, world)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, wl, rank, world, local_rank)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
