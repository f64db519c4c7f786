#!/usr/bin/env python3
"""Mainloop sweep of the sm_100a GEMM library, written to results.csv in the
reference's schema so cutlass_gemm_mainloop/plot_results.py (and
sol_table.py here) read it unchanged.

Replaces cutlass_gemm_mainloop/sweep.sh: same header (:21), the same stage list
(:23) and tile lists (:28-65) plus NVFP4 (DTYPE_ID 2) and CTA-pair (TILE_M 256)
tiles, and the same comment rows for points that fail ("# FAILED: cfg") or
cannot be built ("# BUILD_FAILED: cfg"; here: rejected by the library's
can-implement check, e.g. a ring deeper than shared memory, which is what the
reference's BUILD_FAILED rows are, results.csv:462-465).

Every point is the reference experiment (cutlass_gemm_bench.cu:52-55,158-257):
one CTA (one CTA pair for TILE_M 256), M = TILE_M, N = TILE_N, K = 131072,
zero-filled operands, one warm-up launch, then 20 launches between CUDA events;
the line is M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS with
TFLOPS = 2*M*N*K / time, followed in-process by sm_mhz, the mean effective SM
clock of the timed launches (the kernel's own clock64 / %globaltimer record), which
readers that select columns by name (the reference's plot script) ignore.

Two ways to run the points:
  default      all points in this process, through the library's C ABI (the
               knobs are run-time arguments of the kernels, so nothing is
               compiled per point and the whole sweep takes minutes);
  --binaries   the process-level drop-in the reference uses: one harness
               binary per point (make with the -D knobs, built in parallel),
               then each binary run on its own with no arguments.

Usage: sweep.py [--scope focus|full] [--out results.csv] [--binaries] [--jobs N]
(environment: SWEEP, OUTFILE, MAX_JOBS, as the reference's script reads them).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import datetime
import importlib.util
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG_DIR = HERE.parent
HEADER = "M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS"
EXTRA_COLUMNS = ",sm_mhz"    # in-process runs: the SM clock the point ran at (read by sol_table.py)
DTYPE_NAMES = {0: "BF16", 1: "FP8_E4M3", 2: "NVFP4"}
K_EXPERIMENT = 131072
WARMUP, TIMED = 1, 20

STAGE_LIST = (0, 2, 3, 4, 5, 6, 7, 8)
TILE_N = (16, 32, 64, 128, 192, 256)
REF_TILES = {   # the reference's lists, per DTYPE_ID
    0: [(tm, tn, tk) for tm in (64, 128) for tn in TILE_N for tk in (16, 32, 64, 128, 256)],
    1: [(tm, tn, tk) for tm in (64, 128) for tn in TILE_N for tk in (32, 64, 128, 256, 512)],
}
FOCUS_TILES = {
    0: [(128, 128, 64), (128, 192, 64), (128, 256, 64), (128, 256, 128)],
    1: [(128, 128, 128), (128, 192, 128), (128, 256, 128), (128, 256, 256)],
}
EXTRA_TILES = {   # beyond the reference: CTA pairs and NVFP4
    0: [(256, 256, 64), (256, 512, 64), (256, 256, 128)],
    1: [(256, 256, 128), (256, 512, 128), (256, 256, 256)],
    2: [(128, 128, 256), (128, 256, 256), (256, 128, 256), (256, 256, 256)],
}


def sweep_points(scope: str):
    """(TILE_M, TILE_N, TILE_K, STAGES, DTYPE_ID) in the order the CSV lists them."""
    tiles = REF_TILES if scope == "full" else FOCUS_TILES
    out = []
    for dt in (0, 1, 2):
        for tm, tn, tk in tiles.get(dt, []) + EXTRA_TILES.get(dt, []):
            out += [(tm, tn, tk, s, dt) for s in STAGE_LIST]
    return out


def csv_line(tm, tn, tk, s, dt, ms, sm_mhz=None):
    flop = 2.0 * tm * tn * K_EXPERIMENT
    line = f"{tm},{tn},{K_EXPERIMENT},{tm},{tn},{tk},{s},{DTYPE_NAMES[dt]},{ms:.6g},{flop / (ms * 1e-3) / 1e12:.6g}"
    return line + ("" if sm_mhz is None else f",{sm_mhz:.1f}")


def cfg_text(p):
    return ",".join(str(v) for v in p)


# ---------------------------------------------------------------- in process
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


def run_in_process(points, emit):
    import ctypes as C
    import torch
    pkg = load_pkg()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    L = pkg.lib()
    bufs = {}

    def zeros(key, nbytes):
        t = bufs.get(key)
        if t is None or t.numel() < nbytes:
            t = bufs[key] = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        return t.data_ptr()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clock = torch.zeros(2, dtype=torch.int64, device=dev)
    for p in points:
        tm, tn, tk, s, dt = p
        bits = {0: 16, 1: 8, 2: 4}[dt]
        cg = 2 if tm > 128 else 1
        kw = {}
        if dt == 2:
            kw = dict(sfa=zeros("sfa", pkg.sf_bytes(tm, K_EXPERIMENT)), sfb=zeros("sfb", pkg.sf_bytes(tn, K_EXPERIMENT)))
        args = pkg.make_args(dtype=dt, m=tm, n=tn, k=K_EXPERIMENT,
                             a=zeros("a", tm * K_EXPERIMENT * bits // 8), b=zeros("b", tn * K_EXPERIMENT * bits // 8),
                             d=zeros("d", tm * tn * 2), tile_m=tm, tile_n=tn, tile_k=tk, stages=s,
                             cta_group=cg, max_ctas=cg, clock_out=clock.data_ptr(), **kw)
        rc, info = pkg.query(args)
        if rc != pkg.OK:
            emit(f"# BUILD_FAILED: {cfg_text(p)}", f"cannot implement: {info.reason.decode()}")
            continue
        sp = C.c_void_p(stream.cuda_stream)
        ok = all(L.gemm_sm100a_launch(C.byref(args), sp) == 0 for _ in range(WARMUP))
        clock.zero_()                  # the timed launches add their cycles and ns
        e0.record(stream)
        ok = ok and all(L.gemm_sm100a_launch(C.byref(args), sp) == 0 for _ in range(TIMED))
        e1.record(stream)
        try:
            e1.synchronize()
        except RuntimeError as e:      # a launch error surfaces here; the context is lost
            emit(f"# FAILED: {cfg_text(p)}", repr(e)[:120])
            raise
        if not ok:
            emit(f"# FAILED: {cfg_text(p)}", "launch failed")
            continue
        cyc, ns = (int(v) for v in clock.cpu().tolist())
        line = csv_line(tm, tn, tk, s, dt, e0.elapsed_time(e1) / TIMED, 1e3 * cyc / ns if ns else None)
        emit(line, line)


# ---------------------------------------------------------------- per-point binaries
def run_binaries(points, emit, jobs: int):
    build = HERE / "build"
    build.mkdir(exist_ok=True)
    subprocess.run(["make", "-s", "-C", str(PKG_DIR)], check=True, capture_output=True)

    def binary(p):
        return build / ("bench_%d_%d_%d_s%d_d%d" % p)

    def make(p):
        if binary(p).exists():
            return p, True
        tm, tn, tk, s, dt = p
        r = subprocess.run(["make", "-s", "-C", str(HERE), f"TILE_M={tm}", f"TILE_N={tn}", f"TILE_K={tk}",
                            f"STAGES={s}", f"DTYPE_ID={dt}", f"OUT={binary(p)}"], capture_output=True, text=True)
        (build / (binary(p).name + ".log")).write_text(r.stdout + r.stderr)
        return p, r.returncode == 0

    print(f"building {len(points)} binaries ({jobs} at a time)", file=sys.stderr)
    with cf.ThreadPoolExecutor(jobs) as ex:
        built = dict(ex.map(make, points))
    for p in points:
        if not built[p]:
            emit(f"# BUILD_FAILED: {cfg_text(p)}", "build failed")
            continue
        r = subprocess.run([str(binary(p))], capture_output=True, text=True, timeout=600)
        if r.returncode == 1 and "Cannot implement" in r.stderr:
            emit(f"# BUILD_FAILED: {cfg_text(p)}", r.stderr.strip()[:120])
        elif r.returncode != 0 or not r.stdout.strip():
            emit(f"# FAILED: {cfg_text(p)}", (r.stderr or "no output").strip()[:120])
        else:
            line = r.stdout.strip().splitlines()[-1]
            emit(line, line)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--scope", choices=["focus", "full"], default=os.environ.get("SWEEP", "focus"))
    ap.add_argument("--out", default=os.environ.get("OUTFILE", str(HERE / "results.csv")))
    ap.add_argument("--binaries", action="store_true", help="build and run one harness binary per point")
    ap.add_argument("--jobs", type=int, default=int(os.environ.get("MAX_JOBS", os.cpu_count() or 4)))
    args = ap.parse_args()
    points = sweep_points(args.scope)
    out = open(args.out, "w")
    out.write(HEADER + ("" if args.binaries else EXTRA_COLUMNS) + "\n")
    gpu = "unknown GPU"
    try:
        gpu = subprocess.run(["nvidia-smi", "--query-gpu=name,driver_version", "--format=csv,noheader", "-i", "0"],
                             capture_output=True, text=True).stdout.strip() or gpu
    except OSError:
        pass
    out.write(f"# sweep.py --scope {args.scope}{' --binaries' if args.binaries else ''}: {gpu}, "
              f"{datetime.datetime.now(datetime.timezone.utc):%Y-%m-%dT%H:%MZ}\n")
    count = [0]

    def emit(row, note):
        count[0] += 1
        out.write(row + "\n")
        out.flush()
        print(f"[{count[0]}/{len(points)}] {note}", file=sys.stderr)

    if args.binaries:
        run_binaries(points, emit, args.jobs)
    else:
        run_in_process(points, emit)
    out.close()
    print(f"done: {args.out}", file=sys.stderr)


if __name__ == "__main__":
    main()
