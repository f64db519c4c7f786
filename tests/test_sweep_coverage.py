"""Every tile of the reference sweep is implementable and was measured.

The reference's tile lists (cutlass_gemm_mainloop/sweep.sh:28-65): TILE_M in {64, 128},
TILE_N in {16, 32, 64, 128, 192, 256}, TILE_K in {16..256} for BF16 and {32..512} for
FP8_E4M3, each at STAGES in {0, 2..8} (sweep.sh:23).  The experiment is one CTA with
M = TILE_M, N = TILE_N, K = 131072 (cutlass_gemm_bench.cu:52-55)."""
import csv
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
RESULTS = ROOT / "microbench-blackwell_b200" / "harness" / "results_b200.csv"

TILE_N = (16, 32, 64, 128, 192, 256)
REF_TILES = ([(0, tm, tn, tk) for tm in (64, 128) for tn in TILE_N for tk in (16, 32, 64, 128, 256)] +
             [(1, tm, tn, tk) for tm in (64, 128) for tn in TILE_N for tk in (32, 64, 128, 256, 512)])
K_REF = 131072


def _experiment_args(pkg, dtype, tm, tn, tk, stages=0):
    return pkg.make_args(dtype=dtype, m=tm, n=tn, k=K_REF, a=0x10000, b=0x20000, d=0x30000,
                         tile_m=tm, tile_n=tn, tile_k=tk, stages=stages, max_ctas=1)


@pytest.mark.parametrize("dtype,tm,tn,tk", REF_TILES)
def test_reference_tile_is_implementable(pkg, dtype, tm, tn, tk):
    rc, info = pkg.query(_experiment_args(pkg, dtype, tm, tn, tk))
    assert rc == pkg.OK, info.reason
    assert (info.tile_m, info.tile_n, info.tile_k) == (tm, tn, tk)
    assert info.grid_ctas == 1 and info.num_tiles == 1


def test_stage_counts_follow_shared_memory(pkg):
    """STAGES beyond the shared-memory budget fail like the reference's BUILD_FAILED rows
    (bf16 128x256x64 holds 4 stages of 48 KiB; results.csv:462-465)."""
    rc, info = pkg.query(_experiment_args(pkg, 0, 128, 256, 64, stages=4))
    assert rc == pkg.OK and info.max_stages == 4
    rc, info = pkg.query(_experiment_args(pkg, 0, 128, 256, 64, stages=5))
    assert rc == pkg.ERR_CANNOT_IMPLEMENT and b"stages" in info.reason


def test_committed_sweep_csv_has_the_reference_schema():
    """The committed sweep (regenerated with sweep.py; its first comment line names the
    GPU and the date) parses as the reference's results.csv: header, experiment shape
    M = TILE_M, N = TILE_N, K = 131072 on every row, and only comment rows otherwise."""
    with RESULTS.open() as f:
        header = next(csv.reader(f))
        assert header[:10] == "M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS".split(",")
        rows = 0
        for line in f:
            if line.startswith("#"):
                continue
            r = line.strip().split(",")
            assert len(r) == len(header) and r[7] in ("BF16", "FP8_E4M3", "NVFP4")
            assert int(r[2]) == K_REF and int(r[0]) == int(r[3]) and int(r[1]) == int(r[4])
            rows += 1
    assert rows > 0
