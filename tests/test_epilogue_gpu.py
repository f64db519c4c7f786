"""The epilogue as CUTLASS's LinearCombination defines it (the reference's
cutlass_gemm_bench.cu:117-118 fusion, :196-204 arguments):

    D = alpha * scale_a * scale_b * (A . B^T) + beta * C      (fp32, rounded once to bf16)

with D (and C) column-major, as in the reference (LayoutD, :105), or row-major.

* The staged epilogue (TMA stores from shared memory) and the direct one
  (stores from registers) are bit-identical for every tile shape.
* Row-major D holds exactly the bits of column-major D, transposed.
* Per-tensor scales fold into alpha: bit-identical to alpha = scale_a * scale_b.
* beta * C against the fp64 oracle (C in both layouts, and C aliasing D), within
  the relative Frobenius tolerance of north_star."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = {0: 2e-3, 1: 2e-3, 2: 1e-2}


def operands(pkg, dtype, m, n, k, dev, seed=0):
    kw = {} if dtype != pkg.FP8_E4M3 else dict(a_dist=pkg.NORMAL, a_scale=0.25, b_dist=pkg.NORMAL, b_scale=0.25)
    return pkg.make_operands(dtype, m, n, k, seed=seed, device=dev, **kw)


def run(pkg, ops, d, *, ldd=None, flags=0, status=None, **kw):
    args = pkg.make_args(dtype=ops.dtype, m=ops.m, n=ops.n, k=ops.k, a=ops.a.data_ptr(), b=ops.b.data_ptr(),
                         d=d.data_ptr(), ldd=ldd, sfa=None if ops.sfa is None else ops.sfa.data_ptr(),
                         sfb=None if ops.sfb is None else ops.sfb.data_ptr(), flags=flags,
                         status=None if status is None else status.data_ptr(), **kw)
    pkg.launch(args, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return args


def host_ab(orc, pkg, ops):
    def u16(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    if ops.dtype == pkg.BF16:
        return orc.dequant(u16(ops.a), orc.BF16), orc.dequant(u16(ops.b), orc.BF16)
    if ops.dtype == pkg.FP8_E4M3:
        return orc.dequant(ops.a.cpu().numpy(), orc.FP8_E4M3), orc.dequant(ops.b.cpu().numpy(), orc.FP8_E4M3)
    return (orc.dequant_nvfp4(ops.a.cpu().numpy(), ops.sfa.cpu().numpy(), ops.k),
            orc.dequant_nvfp4(ops.b.cpu().numpy(), ops.sfb.cpu().numpy(), ops.k))


SHAPES = [
    # dtype, m, n, k, knobs
    (0, 512, 1024, 256, dict(cta_group=2, tile_n=512, tile_k=64)),           # single accumulator, 2 groups
    (0, 520, 1000, 192, dict(cta_group=2, tile_n=512, tile_k=64)),           # partial tiles
    (0, 384, 768, 320, dict(cta_group=1, tile_n=256, tile_k=64, stages=4)),
    (0, 200, 300, 128, dict(cta_group=1, tile_n=192, tile_k=64)),
    (0, 192, 256, 192, dict(cta_group=1, tile_m=64, tile_n=128, tile_k=64)),  # M = 64 lane layout
    (0, 256, 80, 128, dict(cta_group=1, tile_n=16, tile_k=64)),              # 16-column chunks
    (0, 512, 640, 256, dict(cta_group=2, tile_n=128, tile_k=64)),
    (1, 512, 1536, 512, dict(cta_group=2, tile_n=512, tile_k=128)),
    (1, 256, 512, 384, dict(cta_group=1, tile_n=256, tile_k=128)),
    (2, 256, 512, 1024, dict(cta_group=1, tile_n=256, tile_k=256)),          # NVFP4: one staging buffer
    (2, 512, 512, 1024, dict(cta_group=2, tile_n=256, tile_k=256)),
]


@pytest.mark.parametrize("case", range(len(SHAPES)))
def test_staged_and_direct_epilogues_agree_bitwise(pkg, orc, cuda, case):
    dt, m, n, k, knobs = SHAPES[case]
    ops = operands(pkg, dt, m, n, k, cuda)
    rc, info = pkg.query(pkg.make_args(dtype=dt, m=m, n=n, k=k, a=ops.a.data_ptr(), b=ops.b.data_ptr(),
                                       d=ops.d.data_ptr(), sfa=None if ops.sfa is None else ops.sfa.data_ptr(),
                                       sfb=None if ops.sfb is None else ops.sfb.data_ptr(), **knobs))
    assert rc == pkg.OK and info.epilogue_staging_buffers > 0
    staged = torch.full_like(ops.d, float("nan"))
    direct = torch.full_like(ops.d, float("nan"))
    run(pkg, ops, staged, **knobs)
    run(pkg, ops, direct, flags=pkg.FLAG_DIRECT_EPILOGUE, **knobs)
    assert not torch.isnan(staged).any()
    assert torch.equal(staged, direct)
    A, B = host_ab(orc, pkg, ops)
    ref = orc.gemm_f64(A, B)
    err = orc.rel_frobenius(staged.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1), m, ref)
    assert err <= TOL[dt], err


@pytest.mark.parametrize("case", [0, 1, 2, 4, 5, 7, 9])
@pytest.mark.parametrize("direct", [False, True])
def test_row_major_d_is_the_transpose_bitwise(pkg, cuda, case, direct):
    dt, m, n, k, knobs = SHAPES[case]
    ops = operands(pkg, dt, m, n, k, cuda)
    col = torch.empty((n, m), dtype=torch.bfloat16, device=cuda)
    ldd = (n + 7) // 8 * 8 + 8                                  # padded rows: the padding must stay untouched
    row = torch.full((m, ldd), float("nan"), dtype=torch.bfloat16, device=cuda)
    run(pkg, ops, col, **knobs)
    run(pkg, ops, row, ldd=ldd, d_layout=pkg.ROW_MAJOR, flags=pkg.FLAG_DIRECT_EPILOGUE if direct else 0, **knobs)
    assert torch.equal(row[:, :n], col.t())
    assert torch.isnan(row[:, n:]).all()


@pytest.mark.parametrize("case", [0, 3, 7, 9])
def test_per_tensor_scales_fold_into_alpha(pkg, cuda, case):
    dt, m, n, k, knobs = SHAPES[case]
    ops = operands(pkg, dt, m, n, k, cuda)
    folded = torch.empty_like(ops.d)
    scaled = torch.empty_like(ops.d)
    run(pkg, ops, folded, alpha=0.75 * 0.5 * 4.0, **knobs)
    run(pkg, ops, scaled, alpha=0.75, scale_a=0.5, scale_b=4.0, **knobs)
    assert torch.equal(folded, scaled)


@pytest.mark.parametrize("case", [0, 1, 3, 4, 7, 9])
@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("direct", [False, True])
def test_beta_c_matches_oracle(pkg, orc, cuda, case, layout, direct):
    dt, m, n, k, knobs = SHAPES[case]
    ops = operands(pkg, dt, m, n, k, cuda)
    alpha, beta = 0.5, -1.25
    ld = m if layout == 0 else (n + 7) // 8 * 8                 # leading dimension of C and D (multiple of 8)
    shape = (n, ld) if layout == 0 else (m, ld)                 # storage of C and D
    gen = torch.Generator(device="cpu").manual_seed(case)
    c = (torch.rand(shape, generator=gen) * 2 - 1).to(torch.bfloat16).to(cuda)
    d = torch.full(shape, float("nan"), dtype=torch.bfloat16, device=cuda)
    run(pkg, ops, d, ldd=ld, alpha=alpha, beta=beta, c=c.data_ptr(), ldc=ld, d_layout=layout,
        flags=pkg.FLAG_DIRECT_EPILOGUE if direct else 0, **knobs)
    A, B = host_ab(orc, pkg, ops)
    ref = orc.gemm_f64(A, B, alpha=alpha)                        # (m, n)
    c64 = c.float().cpu().numpy().astype(np.float64)
    c64 = c64[:, :m].T if layout == 0 else c64[:, :n]
    ref = ref + beta * c64
    got = d.float().cpu().numpy().astype(np.float64)
    got = got[:, :m].T if layout == 0 else got[:, :n]
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err <= TOL[dt], err


def test_beta_c_in_place(pkg, orc, cuda):
    """C may be D itself: D <- alpha * A.B^T + beta * D."""
    dt, m, n, k, knobs = SHAPES[2]
    ops = operands(pkg, dt, m, n, k, cuda)
    d = (torch.rand((n, m), device=cuda) * 2 - 1).to(torch.bfloat16)
    c_copy = d.clone()
    out_sep = torch.empty_like(d)
    run(pkg, ops, out_sep, alpha=1.0, beta=0.5, c=c_copy.data_ptr(), **knobs)
    run(pkg, ops, d, alpha=1.0, beta=0.5, c=d.data_ptr(), **knobs)
    assert torch.equal(d, out_sep)


def test_row_major_gather_is_rejected(pkg, cuda):
    ops = operands(pkg, 0, 256, 256, 256, cuda)
    args = pkg.make_args(dtype=0, m=256, n=256, k=256, a=ops.a.data_ptr(), b=ops.b.data_ptr(),
                         d=ops.d.data_ptr(), d_layout=pkg.ROW_MAJOR)
    extra = torch.empty_like(ops.d)
    with pytest.raises(pkg.GemmError):
        pkg.launch_gather(args, [extra.data_ptr()], torch.cuda.current_stream().cuda_stream)
