"""Pin the CPU oracle against the golden fixtures (tests/golden/, made by
make_golden.py from independent restatements: Python-int splitmix64, libm
Box-Muller, PyTorch dtype casts, a numpy NVFP4 quantiser, numpy fp64 GEMM)."""
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"


def test_rng_bits_and_uniform_exact(orc):
    g = np.load(GOLD / "rng.npz")
    L = orc.lib()
    for i in range(0, len(g["bits"]), 7):
        s, st, ix = int(g["seed"][i]), int(g["stream"][i]), int(g["idx"][i])
        assert L.orc_bits(s, st, ix) == int(g["bits"][i])
        assert np.float32(L.orc_uniform(s, st, ix)) == g["uniform"][i]


def test_normal_matches_libm_box_muller(orc):
    """The oracle's own ln/cos series must reproduce libm Box-Muller in float32."""
    g = np.load(GOLD / "rng.npz")
    L = orc.lib()
    got = np.array([L.orc_normal(int(s), int(st), int(ix))
                    for s, st, ix in zip(g["seed"], g["stream"], g["idx"])], dtype=np.float32)
    exact = np.mean(got == g["normal"])
    assert exact > 0.999, exact                      # bit-exact on (nearly) every draw
    np.testing.assert_allclose(got, g["normal"], rtol=2e-7, atol=1e-7)


def test_uniform_and_normal_moments(orc):
    u = orc.generate(256, 256, orc.BF16, orc.UNIFORM, 1.0, 0, 0)
    uf = orc.bf16_bits_to_f32(u)
    assert -1.0 <= uf.min() and uf.max() <= 1.0 and abs(uf.mean()) < 0.01
    n = orc.generate(256, 256, orc.FP8_E4M3, orc.NORMAL, 1.0, 0, 1)
    nf = orc.dequant(n, orc.FP8_E4M3)
    assert abs(nf.mean()) < 0.02 and abs(nf.std() - 1.0) < 0.03


def test_bf16_and_e4m3_match_torch_casts(orc):
    q = np.load(GOLD / "quant.npz")
    L = orc.lib()
    b = np.array([L.orc_f32_to_bf16(float(v)) for v in q["x"]], dtype=np.uint16)
    e = np.array([L.orc_f32_to_e4m3(float(v)) for v in q["x"]], dtype=np.uint8)
    np.testing.assert_array_equal(b, q["bf16"])
    np.testing.assert_array_equal(e, q["e4m3"])


def test_e4m3_saturates_and_decodes(orc):
    L = orc.lib()
    assert L.orc_f32_to_e4m3(1e6) == 0x7E and L.orc_f32_to_e4m3(-500.0) == 0xFE
    assert L.orc_e4m3_to_f32(0x7E) == 448.0 and L.orc_e4m3_to_f32(0x01) == 2.0 ** -9
    for code in range(0, 0x7F):
        v = L.orc_e4m3_to_f32(code)
        assert L.orc_f32_to_e4m3(v) == code


@pytest.mark.parametrize("x,code", [(0.25, 0), (0.26, 1), (0.75, 2), (1.25, 2), (1.3, 3), (1.75, 4),
                                    (2.5, 4), (2.6, 5), (3.5, 6), (5.0, 6), (5.1, 7), (100.0, 7),
                                    (-0.75, 10), (-6.0, 15)])
def test_e2m1_round_to_nearest_even(orc, x, code):
    assert orc.lib().orc_f32_to_e2m1(x) == code


def test_ue4m3_round_up_never_below(orc):
    L = orc.lib()
    for t in np.geomspace(1e-7, 500, 2000).astype(np.float32):
        q = L.orc_ue4m3_round_up(float(t))
        v = L.orc_e4m3_to_f32(q)
        if t < 448:
            assert v >= t and (q == 1 or L.orc_e4m3_to_f32(q - 1) < t)


def test_nvfp4_matches_numpy_restatement(orc):
    g = np.load(GOLD / "nvfp4.npz")
    vals = g["values"]
    R, K = vals.shape
    packed = np.empty((R, K // 2), dtype=np.uint8)
    scales = np.zeros(orc.sf_bytes(R, K), dtype=np.uint8)
    L = orc.lib()
    # Quantise the golden values block by block with the oracle's primitives.
    for r in range(R):
        for cb in range(K // 16):
            blk = vals[r, cb * 16:(cb + 1) * 16]
            amax = np.float32(np.abs(blk).max())
            sq = L.orc_ue4m3_round_up(float(np.float32(amax / np.float32(6.0))))
            scales[L.orc_sf_offset(r, cb, K)] = sq
            s = np.float32(L.orc_e4m3_to_f32(sq))
            codes = [L.orc_f32_to_e2m1(float(np.float32(v / s))) if sq else 0 for v in blk]
            for j in range(0, 16, 2):
                packed[r, (cb * 16 + j) // 2] = codes[j] | (codes[j + 1] << 4)
    np.testing.assert_array_equal(scales, g["scales"])
    np.testing.assert_array_equal(packed, g["packed"])


def test_nvfp4_generator_consistent_with_dequant(orc):
    packed, scales = orc.generate_nvfp4(128, 256, 1.0, 0, 0)
    deq = orc.dequant_nvfp4(packed, scales, 256)
    ref = np.array([[orc.lib().orc_normal(0, 0, r * 256 + c) for c in range(256)] for r in range(128)],
                   dtype=np.float32)
    # per-block relative error of NVFP4 is bounded by half an e2m1 step at the block max
    err = np.abs(deq - ref).reshape(128, 16, 16).max(axis=2)
    amax = np.abs(ref).reshape(128, 16, 16).max(axis=2)
    assert np.all(err <= amax / 6.0 * 1.0 * 1.125 + 1e-6)


@pytest.mark.parametrize("name", ["bf16_64x48x96", "e4m3_32x40x128", "bf16_1x1x1000"])
def test_gemm_f64_matches_numpy(orc, name):
    g = np.load(GOLD / "gemm.npz")
    A, B, D = g[name + "_A"], g[name + "_B"], g[name + "_D"]
    got = orc.gemm_f64(A, B)
    np.testing.assert_allclose(got, D, rtol=1e-12, atol=1e-12)
    # sampled selection matches the full result
    rows = np.array([0, A.shape[0] - 1]); cols = np.array([B.shape[0] - 1, 0])
    np.testing.assert_allclose(orc.gemm_f64(A, B, rows=rows, cols=cols), D[np.ix_(rows, cols)], rtol=1e-12)


def test_cpu_baseline_gemm_within_tolerance(orc):
    g = np.load(GOLD / "gemm.npz")
    A, B, D = g["bf16_64x48x96_A"], g["bf16_64x48x96_B"], g["bf16_64x48x96_D"]
    out = orc.gemm_omp_f32(A, B)            # bf16 column-major
    err = orc.rel_frobenius(out, A.shape[0], D)
    assert err < 2e-3, err


def test_rel_frobenius_detects_a_planted_error(orc):
    """A mistake planted in the oracle-side data must be caught by the metric."""
    g = np.load(GOLD / "gemm.npz")
    A, B, D = g["bf16_64x48x96_A"], g["bf16_64x48x96_B"], g["bf16_64x48x96_D"]
    out = orc.gemm_omp_f32(A, B)
    bad = out.copy()
    bad[:64] = orc.lib().orc_f32_to_bf16(0.0)      # zero one output column
    assert orc.rel_frobenius(bad, 64, D) > 2e-2
