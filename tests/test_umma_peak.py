"""The tcgen05 peak probe (the SOL denominator; replaces umma_throughput/).
The reference measured 8152.85 / 16344.5 / 32721 FLOP/clk/SM for bf16 / e4m3 /
4-bit at 1SM M128 N256 (umma_throughput/tput_results_max.csv:13,49,121); the
probe must land near those (theoretical 8192 / 16384 / 32768)."""
import pytest

pytestmark = pytest.mark.gpu

THEORY = {0: 8192, 1: 16384, 2: 32768}


@pytest.mark.parametrize("dtype", [0, 1, 2])
@pytest.mark.parametrize("cta_group", [1, 2])
def test_single_sm_peak_near_theory(pkg, cuda, dtype, cta_group):
    r = pkg.umma_peak(dtype, cta_group=cta_group, num_ctas=cta_group, depth=256, iters=20)
    assert 0.9 * THEORY[dtype] <= r["flop_per_clk_per_sm"] <= 1.01 * THEORY[dtype], r
    assert 500 < r["sm_mhz"] < 2200, r


def test_whole_gpu_mode(pkg, cuda):
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    r = pkg.umma_peak(0, cta_group=2, num_ctas=sms - sms % 2, depth=256, iters=20)
    assert r["tflops"] > 1000 and r["flop_per_clk_per_sm"] > 0.9 * THEORY[0], r
