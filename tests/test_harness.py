"""The drop-in harness and sweep: same knobs, CSV schema and failure rows as
the reference's cutlass_gemm_mainloop/{cutlass_gemm_bench.cu, sweep.sh}."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "microbench-blackwell_b200" / "harness"
HEADER = "M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS"   # cutlass_gemm_mainloop/sweep.sh:21


def test_sweep_writes_the_reference_header_and_failure_rows():
    text = (HARNESS / "sweep.sh").read_text()
    assert f'echo "{HEADER}" > "$OUTFILE"' in text
    assert '"# FAILED: $cfg"' in text and '"# BUILD_FAILED: $cfg"' in text
    assert "STAGE_LIST=(0 2 3 4 5 6 7 8)" in text             # sweep.sh:23


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
