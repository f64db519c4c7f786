"""The sweep's SOL table (harness/sol_table.py), data-frame step on CPU: the
reference's 1300 MHz formula (cutlass_gemm_mainloop/plot_results.py:22-27,42-43)
extended to NVFP4 and CTA pairs, the measured-rate SOL at each point's own clock,
and the ratio to the reference's published results."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "microbench-blackwell_b200" / "harness"

CSV = """M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS,sm_mhz
# sweep.py --scope focus: test
128,256,131072,128,256,64,4,BF16,0.7,15.0,1965.0
128,256,131072,128,256,64,3,BF16,0.9,11.0,1965.0
# BUILD_FAILED: 128,256,64,5,0
256,256,131072,256,256,64,0,BF16,0.7,30.0,1900.0
128,256,131072,128,256,256,0,NVFP4,0.2,60.0,1800.0
"""
PUBLISHED = """M,N,K,TILE_M,TILE_N,TILE_K,STAGES,dtype,time_ms,TFLOPS
128,256,131072,128,256,64,4,BF16,0.8,10.4596
"""


@pytest.fixture(scope="module")
def sol():
    pytest.importorskip("pandas")
    spec = importlib.util.spec_from_file_location("sol_table_for_tests", HARNESS / "sol_table.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_sol_columns(sol, tmp_path):
    (tmp_path / "r.csv").write_text(CSV)
    (tmp_path / "p.csv").write_text(PUBLISHED)
    df = sol.with_sol(sol.read_results(tmp_path / "r.csv"), {"BF16": 8100.0, "FP8_E4M3": 16200.0, "NVFP4": 32400.0},
                      sol.read_results(tmp_path / "p.csv"))
    assert len(df) == 4                                         # comment rows skipped
    r = df[(df.STAGES == 4) & (df.dtype == "BF16")].iloc[0]
    assert r.pct_sol_1300 == pytest.approx(100 * 15.0 / (8192 * 1300e6 / 1e12))
    assert r.pct_sol_measured == pytest.approx(100 * 15.0 / (8100 * 1965e6 / 1e12))
    assert r.vs_published == pytest.approx(15.0 / 10.4596)
    pair = df[df.TILE_M == 256].iloc[0]
    assert pair.sms == 2 and pair.pct_sol_1300 == pytest.approx(100 * 30.0 / (2 * 8192 * 1300e6 / 1e12))
    nv = df[df.dtype == "NVFP4"].iloc[0]
    assert nv.pct_sol_measured == pytest.approx(100 * 60.0 / (32400 * 1800e6 / 1e12))
    best = sol.best_per_tile(df)
    assert list(best[best.tile_label == "128x256x64"].STAGES) == [4]
    assert "pct_sol_measured" in sol.markdown(best, "test")


def test_committed_sweep_reads(sol):
    df = sol.with_sol(sol.read_results(HARNESS / "results_b200.csv"), dict(sol.NOMINAL_FLOP_PER_CLK_SM))
    assert len(df) > 0 and df["pct_sol_1300"].notna().all()
