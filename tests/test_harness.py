"""The drop-in harness and sweep: same knobs, CSV schema and failure rows as
the reference's cutlass_gemm_mainloop/{cutlass_gemm_bench.cu, sweep.sh}."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "microbench-blackwell_b200" / "harness"
HEADER = "M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS"   # cutlass_gemm_mainloop/sweep.sh:21


def _sweep():
    import importlib.util
    spec = importlib.util.spec_from_file_location("sweep_for_tests", HARNESS / "sweep.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_sweep_writes_the_reference_header_stages_and_failure_rows():
    sw = _sweep()
    assert sw.HEADER == HEADER
    assert sw.STAGE_LIST == (0, 2, 3, 4, 5, 6, 7, 8)                    # sweep.sh:23
    assert sw.K_EXPERIMENT == 131072 and (sw.WARMUP, sw.TIMED) == (1, 20)  # cutlass_gemm_bench.cu:52-55
    text = (HARNESS / "sweep.py").read_text()
    assert '"# FAILED: {cfg_text(p)}"' in text and '"# BUILD_FAILED: {cfg_text(p)}"' in text
    line = sw.csv_line(128, 256, 64, 4, 0, 1.0)
    assert line.split(",")[:8] == ["128", "256", "131072", "128", "256", "64", "4", "BF16"]
    assert abs(float(line.split(",")[9]) - 2 * 128 * 256 * 131072 / 1e-3 / 1e12) < 1e-3


def test_full_sweep_covers_every_reference_point():
    """The reference's lists (sweep.sh:28-65) at every stage count, in the full scope."""
    sw = _sweep()
    pts = set(sw.sweep_points("full"))
    tile_n = (16, 32, 64, 128, 192, 256)
    for dt, ks in ((0, (16, 32, 64, 128, 256)), (1, (32, 64, 128, 256, 512))):
        for tm in (64, 128):
            for tn in tile_n:
                for tk in ks:
                    for s in (0, 2, 3, 4, 5, 6, 7, 8):
                        assert (tm, tn, tk, s, dt) in pts


def test_harness_builds_with_reference_knobs(tmp_path):
    out = tmp_path / "gemm_bench_test"
    subprocess.run(["make", "-s", "-C", str(HARNESS), "TILE_M=128", "TILE_N=256", "TILE_K=64", "STAGES=4",
                    "DTYPE_ID=0", f"OUT={out}"], check=True)
    assert out.exists()
    # NVFP4 and CTA-pair knobs compile too
    for extra in (["DTYPE_ID=2", "TILE_K=256"], ["TILE_M=256", "TILE_N=512"]):
        o2 = tmp_path / ("b_" + "_".join(extra))
        subprocess.run(["make", "-s", "-C", str(HARNESS), f"OUT={o2}", *extra], check=True)
        assert o2.exists()


def run_bin(path, *args):
    return subprocess.run([str(path), *args], capture_output=True, text=True, timeout=300)


@pytest.mark.gpu
def test_reference_experiment_line(cuda):
    """No argv: one CTA, M=TILE_M, N=TILE_N, K=131072, one 10-column CSV line (cutlass_gemm_bench.cu:253-257)."""
    r = run_bin(HARNESS / "bin" / "gemm_bench_128_256_64_s4_d0")
    assert r.returncode == 0, r.stderr
    fields = r.stdout.strip().split(",")
    assert len(fields) == 10
    assert fields[:8] == ["128", "256", "131072", "128", "256", "64", "4", "BF16"]
    assert float(fields[9]) > 1.0


@pytest.mark.gpu
def test_cannot_implement_exits_1(cuda, tmp_path):
    out = tmp_path / "gemm_bench_s5"
    subprocess.run(["make", "-s", "-C", str(HARNESS), "TILE_N=256", "TILE_K=64", "STAGES=5", f"OUT={out}"], check=True)
    r = run_bin(out)
    assert r.returncode == 1 and "Cannot implement" in r.stderr and r.stdout == ""


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,args", [
    ((128, 256, 64, 4, 0), ["--m", "1024", "--n", "768", "--k", "2048", "--check"]),
    ((128, 256, 128, 0, 1), ["--m", "768", "--n", "1024", "--k", "4096", "--check"]),
    ((256, 512, 64, 0, 0), ["--m", "1024", "--n", "1536", "--k", "1024", "--check"]),
])
def test_full_problem_self_check(cuda, cfg, args):
    r = run_bin(HARNESS / "bin" / ("gemm_bench_%d_%d_%d_s%d_d%d" % cfg), *args)
    assert r.returncode == 0, r.stderr
    f = r.stdout.strip().split(",")
    assert len(f) == 14 and 0.0 <= float(f[13]) <= 2e-3
