"""GPU parity tests: the sm_100a kernels through the C ABI against the CPU
oracle (fp64 GEMM over the same dequantised inputs).  Tolerance: relative
Frobenius error <= 2e-3 for bf16 / fp8 inputs and <= 1e-2 for NVFP4, D
compared after its bf16 rounding.  Layout KATs (identity, single non-zero)
are bit-exact."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {0: 2e-3, 1: 2e-3, 2: 1e-2}


def raw_u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def host_operands(orc, pkg, ops):
    if ops.dtype == pkg.BF16:
        return orc.dequant(raw_u16(ops.a), orc.BF16), orc.dequant(raw_u16(ops.b), orc.BF16)
    if ops.dtype == pkg.FP8_E4M3:
        return orc.dequant(ops.a.cpu().numpy(), orc.FP8_E4M3), orc.dequant(ops.b.cpu().numpy(), orc.FP8_E4M3)
    return (orc.dequant_nvfp4(ops.a.cpu().numpy(), ops.sfa.cpu().numpy(), ops.k),
            orc.dequant_nvfp4(ops.b.cpu().numpy(), ops.sfb.cpu().numpy(), ops.k))


def rel_err(orc, pkg, ops, rows=None, cols=None, alpha=1.0):
    A, B = host_operands(orc, pkg, ops)
    ref = orc.gemm_f64(A, B, alpha=alpha, rows=rows, cols=cols)
    return orc.rel_frobenius(raw_u16(ops.d).reshape(-1), ops.m, ref, rows=rows, cols=cols)


def make(pkg, dtype, m, n, k, dev, seed=0, n0=0):
    if dtype == pkg.BF16:
        return pkg.make_operands(dtype, m, n, k, seed=seed, device=dev, n0=n0)
    return pkg.make_operands(dtype, m, n, k, seed=seed, device=dev, n0=n0,
                             a_dist=pkg.NORMAL, a_scale=0.25, b_dist=pkg.NORMAL, b_scale=0.25)


# --------------------------------------------------------------------------- generator
@pytest.mark.parametrize("dtype,dist,scale,stream", [(0, 0, 1.0, 0), (1, 1, 0.25, 1), (0, 1, 1.0, 3), (1, 1, 0.02, 1)])
def test_device_generator_matches_oracle_bit_exact(pkg, orc, cuda, dtype, dist, scale, stream):
    rows, cols, row0 = 96, 320, 1000
    t = torch.empty((rows, cols), dtype=torch.bfloat16 if dtype == 0 else torch.uint8, device=cuda)
    pkg.generate(t.data_ptr(), dtype, dist, scale, 7, stream, row0, rows, cols)
    torch.cuda.synchronize()
    dev = raw_u16(t) if dtype == 0 else t.cpu().numpy()
    host = orc.generate(rows, cols, dtype, dist, scale, 7, stream, row0=row0)
    np.testing.assert_array_equal(dev, host)


def test_device_nvfp4_quantiser_matches_oracle_bit_exact(pkg, orc, cuda):
    rows, cols, row0 = 256, 512, 128
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=cuda)
    scales = torch.zeros(pkg.sf_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    pkg.generate_nvfp4(packed.data_ptr(), scales.data_ptr(), 1.0, 0, 1, row0, rows, cols)
    torch.cuda.synchronize()
    hp, hs = orc.generate_nvfp4(rows, cols, 1.0, 0, 1, row0=row0)
    np.testing.assert_array_equal(packed.cpu().numpy(), hp)
    np.testing.assert_array_equal(scales.cpu().numpy(), hs)


# --------------------------------------------------------------------------- bf16 1-SM
def test_config1_bf16_256_full_check(pkg, orc, cuda):
    """bf16 256^3, uniform[-1,1) seed 0, full fp64 check."""
    ops = make(pkg, pkg.BF16, 256, 256, 256, cuda)
    pkg.gemm(ops, tile_n=256, tile_k=64)
    err = rel_err(orc, pkg, ops)
    assert err <= TOL[0], err


def test_identity_b_reproduces_a_exactly(pkg, orc, cuda):
    """D = A . I^T = A: pins the swizzled smem layout and descriptors of both operands."""
    m = n = k = 256
    ops = make(pkg, pkg.BF16, m, n, k, cuda)
    ops.b.zero_()
    ops.b.copy_(torch.eye(n, k, dtype=torch.bfloat16, device=cuda))
    pkg.gemm(ops, tile_n=256, tile_k=64)
    np.testing.assert_array_equal(raw_u16(ops.d.t().contiguous()), raw_u16(ops.a[:, :n]))


@pytest.mark.parametrize("i,kk", [(0, 0), (5, 17), (127, 63), (128, 64), (200, 191), (255, 255)])
def test_single_nonzero_in_a_selects_one_column_of_b(pkg, orc, cuda, i, kk):
    m = n = k = 256
    ops = make(pkg, pkg.BF16, m, n, k, cuda)
    ops.a.zero_()
    ops.a[i, kk] = 1.0
    pkg.gemm(ops, tile_n=128, tile_k=64, stages=2)
    D = ops.d.t().float().cpu()                       # (m, n)
    expect = torch.zeros(m, n)
    expect[i, :] = ops.b[:, kk].float().cpu()
    assert torch.equal(D, expect)


@pytest.mark.parametrize("m,n,k,tile_n,tile_k", [(200, 300, 320, 256, 64), (128, 16, 64, 16, 64),
                                                 (384, 272, 192, 128, 128), (1000, 520, 1000, 64, 64)])
def test_tails_and_partial_tiles(pkg, orc, cuda, m, n, k, tile_n, tile_k):
    if k % 8:
        pytest.skip("k must keep 16-byte rows")
    ops = make(pkg, pkg.BF16, m, n, k, cuda)
    pkg.gemm(ops, tile_n=tile_n, tile_k=tile_k)
    err = rel_err(orc, pkg, ops)
    assert err <= TOL[0], err


def test_alpha_scales_the_result(pkg, orc, cuda):
    ops = make(pkg, pkg.BF16, 256, 256, 512, cuda)
    pkg.gemm(ops, alpha=0.5)
    assert rel_err(orc, pkg, ops, alpha=0.5) <= TOL[0]


def test_tile_and_stage_choices_agree_bitwise(pkg, orc, cuda):
    """Every (tile_n, tile_k, stages) point accumulates in the same K order, so
    all of them must produce identical bits (and match the oracle)."""
    ops = make(pkg, pkg.BF16, 1024, 1024, 1024, cuda)
    pkg.gemm(ops, tile_n=256, tile_k=64, stages=4)
    ref = ops.d.clone()
    assert rel_err(orc, pkg, ops) <= TOL[0]
    for tn, tk, s in [(128, 64, 2), (192, 64, 3), (64, 128, 4), (32, 64, 6), (16, 64, 8), (256, 128, 2), (256, 64, 1)]:
        ops.d.fill_(0)
        pkg.gemm(ops, tile_n=tn, tile_k=tk, stages=s)
        assert torch.equal(ops.d, ref), (tn, tk, s)


@pytest.mark.parametrize("dtype,tile_k", [(0, 16), (0, 32), (1, 32), (1, 64)])
@pytest.mark.parametrize("cta_group,tile_n", [(1, 256), (1, 64), (1, 16), (2, 256), (2, 512)])
def test_narrow_tile_k_swizzle_modes(pkg, orc, cuda, dtype, tile_k, cta_group, tile_n):
    """TILE_K below one 128-byte row (32- and 64-byte swizzle, the reference
    sweep's bf16 TILE_K 16/32 and fp8 32/64) against the oracle, and bit-identical
    to the 128-byte-row kernel: the MMAs walk K in the same 32-byte steps."""
    m, n, k = 512, 1024, 328 if dtype == 0 else 336       # K tail inside the last stage
    ops = make(pkg, dtype, m, n, k, cuda)
    pkg.gemm(ops, cta_group=cta_group, tile_n=tile_n, tile_k=tile_k)
    assert rel_err(orc, pkg, ops) <= TOL[dtype]
    narrow = ops.d.clone()
    ops.d.fill_(0)
    pkg.gemm(ops, cta_group=1, tile_n=256, tile_k=64 if dtype == 0 else 128)
    assert torch.equal(ops.d, narrow)


def test_tile_m_64_identity_kat(pkg, orc, cuda):
    """M = 64 accumulator layout: with A = I, D = B^T exactly (each product
    is one bf16 value times 1), so every row and column must land in place."""
    m, n, k = 192, 256, 192
    ops = make(pkg, pkg.BF16, m, n, k, cuda)
    ops.a.copy_(torch.eye(m, k, dtype=torch.bfloat16, device=cuda))
    pkg.gemm(ops, tile_m=64, tile_n=128, tile_k=64)
    assert torch.equal(ops.d, ops.b[:, :m].contiguous())   # D^T storage (n, m) = B[:, :m]


@pytest.mark.parametrize("dtype,tile_k", [(0, 64), (0, 16), (1, 128), (1, 32)])
@pytest.mark.parametrize("m,n,k,tile_n", [(200, 300, 320, 256), (448, 512, 512, 128), (64, 16, 1024, 16)])
def test_tile_m_64_matches_oracle_and_128_bitwise(pkg, orc, cuda, dtype, tile_k, m, n, k, tile_n):
    """TILE_M = 64 (partial M and N tiles included) against the oracle, and
    bit-identical to the TILE_M = 128 kernel."""
    ops = make(pkg, dtype, m, n, k, cuda)
    pkg.gemm(ops, tile_m=64, tile_n=tile_n, tile_k=tile_k)
    assert rel_err(orc, pkg, ops) <= TOL[dtype]
    d64 = ops.d.clone()
    ops.d.fill_(0)
    pkg.gemm(ops, tile_n=256, tile_k=64 if dtype == 0 else 128)
    assert torch.equal(ops.d, d64)


def test_config2_bf16_8192_sampled(pkg, orc, cuda):
    """BASELINE config 2 (bf16 8192^3, 128x256x64, 4 stages), sampled fp64 check:
    a random 128 x 128 block plus two full rows and two full columns."""
    m = n = k = 8192
    ops = make(pkg, pkg.BF16, m, n, k, cuda)
    pkg.gemm(ops, tile_n=256, tile_k=64, stages=4)
    rng = np.random.default_rng(0)
    rows = np.concatenate([rng.choice(m, 128, replace=False), [0, m - 1]])
    cols = np.concatenate([rng.choice(n, 128, replace=False), [0, n - 1]])
    A = orc.dequant(raw_u16(ops.a[torch.as_tensor(rows)]), orc.BF16)
    B = orc.dequant(raw_u16(ops.b), orc.BF16)
    ref = orc.gemm_f64(A, B, rows=None, cols=cols)          # (len(rows), len(cols))
    D = raw_u16(ops.d).reshape(n, m)                          # D^T storage
    got = orc.bf16_bits_to_f32(D[np.ix_(cols, rows)].T)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err <= TOL[0], err
    # two full rows of D
    fr = orc.gemm_f64(A[-2:], B)
    got_rows = orc.bf16_bits_to_f32(D[:, rows[-2:]].T)
    assert np.linalg.norm(got_rows - fr) / np.linalg.norm(fr) <= TOL[0]


def test_single_cta_reference_mode(pkg, orc, cuda):
    """The reference's experiment shape (one CTA, M=TILE_M, N=TILE_N, long K)."""
    ops = make(pkg, pkg.BF16, 128, 256, 16384, cuda)
    pkg.gemm(ops, tile_n=256, tile_k=64, stages=4, max_ctas=1)
    assert rel_err(orc, pkg, ops) <= TOL[0]


# --------------------------------------------------------------------------- fp8 1-SM
@pytest.mark.parametrize("m,n,k,tile_n", [(512, 768, 1024, 256), (256, 192, 384, 192), (384, 128, 256, 128)])
def test_fp8_e4m3_1sm(pkg, orc, cuda, m, n, k, tile_n):
    ops = make(pkg, pkg.FP8_E4M3, m, n, k, cuda)
    pkg.gemm(ops, tile_n=tile_n, tile_k=128)
    err = rel_err(orc, pkg, ops)
    assert err <= TOL[1], err


# --------------------------------------------------------------------------- failure detection
def test_injected_stall_times_out_and_context_survives(pkg, orc, cuda):
    """A wait that nothing satisfies must end with GEMM_ERR_TIMEOUT (not a hang),
    and the context must stay usable for the next GEMM."""
    ops = make(pkg, pkg.BF16, 256, 256, 256, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    pkg.gemm_into(ops, status=status, timeout_ms=100, flags=pkg.FLAG_INJECT_STALL)
    rc, detail = pkg.read_status(status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == pkg.ERR_TIMEOUT
    assert detail & 0xFF == 3 and ((detail >> 8) & 0xF) in (2, 3)    # MMA or epilogue gave up
    pkg.gemm(ops)
    assert rel_err(orc, pkg, ops) <= TOL[0]


# --------------------------------------------------------------------------- 2-SM (cta_group::2)
@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("m,n,k,tile_n", [(512, 512, 512, 256), (384, 320, 256, 128), (256, 192, 1024, 192),
                                          (1280, 640, 768, 64), (512, 1024, 512, 512), (384, 640, 256, 512)])
def test_pair_mode_matches_oracle_and_single_sm_bitwise(pkg, orc, cuda, dtype, m, n, k, tile_n):
    """cta_group::2 (256 x N per CTA pair, B split across the pair) against the oracle, and
    bit-identical to the 1-SM kernel (same K accumulation order)."""
    tk = 64 if dtype == 0 else 128
    ops = make(pkg, dtype, m, n, k, cuda)
    pkg.gemm(ops, cta_group=2, tile_n=tile_n, tile_k=tk)
    err = rel_err(orc, pkg, ops)
    assert err <= TOL[dtype], err
    pair = ops.d.clone()
    ops.d.fill_(0)
    pkg.gemm(ops, cta_group=1, tile_n=min(tile_n, 256), tile_k=tk)
    assert torch.equal(ops.d, pair)


def test_pair_mode_identity_kat(pkg, orc, cuda):
    m = n = k = 512
    ops = make(pkg, pkg.BF16, m, n, k, cuda)
    ops.b.copy_(torch.eye(n, k, dtype=torch.bfloat16, device=cuda))
    pkg.gemm(ops, cta_group=2, tile_n=256, tile_k=64)
    np.testing.assert_array_equal(raw_u16(ops.d.t().contiguous()), raw_u16(ops.a[:, :n]))


def test_pair_mode_injected_stall(pkg, orc, cuda):
    ops = make(pkg, pkg.BF16, 512, 512, 256, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    pkg.gemm_into(ops, status=status, timeout_ms=100, flags=pkg.FLAG_INJECT_STALL, cta_group=2)
    rc, detail = pkg.read_status(status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == pkg.ERR_TIMEOUT
    pkg.gemm(ops, cta_group=2)
    assert rel_err(orc, pkg, ops) <= TOL[0]


def test_config3_fp8_16384_pair_sampled(pkg, orc, cuda):
    """e4m3 16384^3, N(0,1)/4 inputs, cta_group::2 256x256x128; sampled check."""
    m = n = k = 16384
    ops = make(pkg, pkg.FP8_E4M3, m, n, k, cuda)
    pkg.gemm(ops, cta_group=2, tile_n=256, tile_k=128)
    rng = np.random.default_rng(1)
    rows = np.sort(rng.choice(m, 96, replace=False))
    cols = np.sort(rng.choice(n, 96, replace=False))
    A = orc.dequant(ops.a[torch.as_tensor(rows)].cpu().numpy(), orc.FP8_E4M3)
    B = orc.dequant(ops.b[torch.as_tensor(cols)].cpu().numpy(), orc.FP8_E4M3)
    ref = orc.gemm_f64(A, B)
    D = raw_u16(ops.d).reshape(n, m)
    got = orc.bf16_bits_to_f32(D[np.ix_(cols, rows)].T)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err <= TOL[1], err


# --------------------------------------------------------------------------- NVFP4 (1-SM)
E2M1_ONE = 0x2          # e2m1 code of 1.0
UE4M3_ONE = 0x38        # e4m3 code of 1.0


def nvfp4_identity(torch_dev, n, k):
    """Packed e2m1 identity rows (B[n][k] = 1 if n == k) with all scales 1.0."""
    packed = torch.zeros((n, k // 2), dtype=torch.uint8)
    for i in range(min(n, k)):
        packed[i, i // 2] = E2M1_ONE << (4 * (i % 2))
    return packed.to(torch_dev)


@pytest.mark.parametrize("tile_n", [128, 256])
def test_nvfp4_identity_b_reproduces_a_with_its_block_scales(pkg, orc, cuda, tile_n):
    """D = A . I^T reproduces A's dequantised values (e2m1 x its per-16 ue4m3 scale), exactly:
    pins the packed-fp4 smem descriptors and the SFA scale layout in TMEM."""
    m, n, k = 256, 256, 512
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=2, device=cuda)
    ops.b.copy_(nvfp4_identity(cuda, n, k))
    ops.sfb.fill_(UE4M3_ONE)
    pkg.gemm(ops, tile_n=tile_n, tile_k=256)
    A = orc.dequant_nvfp4(ops.a.cpu().numpy(), ops.sfa.cpu().numpy(), k)
    D = orc.bf16_bits_to_f32(raw_u16(ops.d.t().contiguous()))
    np.testing.assert_array_equal(D, A[:, :n])


def test_nvfp4_identity_a_reproduces_b_with_its_block_scales(pkg, orc, cuda):
    """The mirror case pins the SFB layout (256 B rows = two 128-row scale atoms)."""
    m, n, k = 256, 256, 512
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=3, device=cuda)
    ops.a.copy_(nvfp4_identity(cuda, m, k))
    ops.sfa.fill_(UE4M3_ONE)
    pkg.gemm(ops, tile_n=256, tile_k=256)
    B = orc.dequant_nvfp4(ops.b.cpu().numpy(), ops.sfb.cpu().numpy(), k)
    D = orc.bf16_bits_to_f32(raw_u16(ops.d.t().contiguous()))
    np.testing.assert_array_equal(D, B[:, :m].T)


@pytest.mark.parametrize("m,n,k,tile_n,stages", [(256, 256, 1024, 256, 0), (384, 512, 2048, 128, 0),
                                                 (128, 256, 256, 256, 2), (512, 768, 4096, 256, 3)])
def test_nvfp4_matches_oracle(pkg, orc, cuda, m, n, k, tile_n, stages):
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=0, device=cuda)
    pkg.gemm(ops, tile_n=tile_n, tile_k=256, stages=stages)
    err = rel_err(orc, pkg, ops)
    assert err <= TOL[2], err


# --------------------------------------------------------------------------- NVFP4 (CTA pair)
@pytest.mark.parametrize("tile_n", [128, 256])
def test_nvfp4_pair_identity_b_pins_sfa_on_both_ctas(pkg, orc, cuda, tile_n):
    """cta_group::2 block-scaled MMA: D = A . I^T reproduces A exactly, so the
    scale factors of A reach the TMEM of both CTAs of the pair in place."""
    m, n, k = 512, 256, 512
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=4, device=cuda)
    ops.b.copy_(nvfp4_identity(cuda, n, k))
    ops.sfb.fill_(UE4M3_ONE)
    pkg.gemm(ops, cta_group=2, tile_n=tile_n, tile_k=256)
    A = orc.dequant_nvfp4(ops.a.cpu().numpy(), ops.sfa.cpu().numpy(), k)
    D = orc.bf16_bits_to_f32(raw_u16(ops.d.t().contiguous()))
    np.testing.assert_array_equal(D, A[:, :n])


@pytest.mark.parametrize("tile_n", [128, 256])
def test_nvfp4_pair_identity_a_pins_sfb(pkg, orc, cuda, tile_n):
    """The mirror case: every CTA of the pair stages the whole tile's B scales."""
    m, n, k = 256, 512, 512
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=5, device=cuda)
    ops.a.copy_(nvfp4_identity(cuda, m, k))
    ops.sfa.fill_(UE4M3_ONE)
    pkg.gemm(ops, cta_group=2, tile_n=tile_n, tile_k=256)
    B = orc.dequant_nvfp4(ops.b.cpu().numpy(), ops.sfb.cpu().numpy(), k)
    D = orc.bf16_bits_to_f32(raw_u16(ops.d.t().contiguous()))
    np.testing.assert_array_equal(D, B[:, :m].T)


@pytest.mark.parametrize("m,n,k,tile_n,tile_k,stages", [(512, 512, 2048, 256, 256, 0), (256, 384, 1024, 128, 256, 0),
                                                        (768, 1024, 4096, 256, 512, 0), (512, 256, 1024, 256, 256, 2)])
def test_nvfp4_pair_matches_oracle_and_single_sm_bitwise(pkg, orc, cuda, m, n, k, tile_n, tile_k, stages):
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=1, device=cuda)
    pkg.gemm(ops, cta_group=2, tile_n=tile_n, tile_k=tile_k, stages=stages)
    assert rel_err(orc, pkg, ops) <= TOL[2]
    pair = ops.d.clone()
    ops.d.fill_(0)
    pkg.gemm(ops, cta_group=1, tile_n=tile_n, tile_k=tile_k)
    assert torch.equal(ops.d, pair)


def test_config4_nvfp4_mlp_sampled(pkg, orc, cuda):
    """NVFP4 M=8192, N=28672, K=8192; sampled fp64 check."""
    m, n, k = 8192, 28672, 8192
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=0, device=cuda)
    pkg.gemm(ops, tile_n=256, tile_k=256)
    rng = np.random.default_rng(4)
    rows = np.sort(rng.choice(m // 128, 1, replace=False))[0] * 128 + np.arange(128)   # one 128-row scale block
    cols = np.sort(rng.choice(n, 96, replace=False))
    A = orc.dequant_nvfp4(ops.a[rows[0]:rows[0] + 128].cpu().numpy(),
                          ops.sfa[(rows[0] // 128) * (k // 64) * 512:(rows[0] // 128 + 1) * (k // 64) * 512].cpu().numpy(), k)
    Bfull_packed = ops.b.cpu().numpy(); Bsf = ops.sfb.cpu().numpy()
    B = orc.dequant_nvfp4(Bfull_packed, Bsf, k)[cols]
    ref = orc.gemm_f64(A, B)
    D = raw_u16(ops.d).reshape(n, m)
    got = orc.bf16_bits_to_f32(D[np.ix_(cols, rows)].T)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err <= TOL[2], err
