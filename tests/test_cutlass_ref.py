"""Agreement with the reference's own kernel family: the CUTLASS SM100 GEMM run
by oracle/_ref/libcutlass_ref.so on the same seeded device inputs.

Kernels (oracle/cutlass_ref.cu): id 0/1 are the reference's 1SM schedule at its
best bf16 / e4m3 tiles (cutlass_gemm_bench.cu:101-156, results.csv:461,938);
id 4 the 1SM Nvf4 block-scaled schedule for NVFP4, which reads the same scale
buffers.  Every configuration of ours (1-SM and CTA pair) is checked against them.  Tolerance (north_star): relative Frobenius error 2e-3 for bf16 and
e4m3, 1e-2 for NVFP4, between the two bf16 results.  The last cases run the
bench's exact knob sets at each BASELINE configuration's full shape."""
import ctypes as C
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libcutlass_ref.so"
TOL = {0: 2e-3, 1: 2e-3, 2: 1e-2}


@pytest.fixture(scope="module")
def cutlass(cuda):
    if not LIB.exists():
        pytest.skip("oracle/_ref/libcutlass_ref.so not built (oracle/ref_build.sh)")
    L = C.CDLL(str(LIB))
    L.cutlass_ref_run.restype = C.c_int
    L.cutlass_ref_run.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
    return L


def rel(a, b):
    a = a.float(); b = b.float()
    return (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item()


def run_cutlass(L, kid, ops):
    ref = torch.empty_like(ops.d)
    rc = L.cutlass_ref_run(kid, ops.a.data_ptr(), ops.b.data_ptr(),
                           None if ops.sfa is None else ops.sfa.data_ptr(),
                           None if ops.sfb is None else ops.sfb.data_ptr(),
                           ref.data_ptr(), ops.m, ops.n, ops.k, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, f"cutlass_ref_run({kid}) = {rc}"
    return ref


def operands(pkg, dtype, m, n, k, dev, b_scale=None):
    if dtype == pkg.BF16:
        return pkg.make_operands(dtype, m, n, k, seed=3, device=dev)
    if dtype == pkg.FP8_E4M3:
        return pkg.make_operands(dtype, m, n, k, seed=3, device=dev, a_dist=pkg.NORMAL, a_scale=0.25,
                                 b_dist=pkg.NORMAL, b_scale=0.25 if b_scale is None else b_scale)
    return pkg.make_operands(dtype, m, n, k, seed=3, device=dev)


@pytest.mark.parametrize("kid,dtype,m,n,k,knobs", [
    (0, 0, 2048, 2048, 2048, dict(cta_group=1, tile_n=256, tile_k=64, stages=4)),
    (0, 0, 2048, 2048, 2048, dict(cta_group=2, tile_n=512, tile_k=64)),
    (0, 0, 2048, 2048, 2048, dict(cta_group=2, tile_n=256, tile_k=64, raster_group=4)),
    (1, 1, 2048, 1536, 4096, dict(cta_group=1, tile_n=256, tile_k=128)),
    (1, 1, 2048, 1536, 4096, dict(cta_group=2, tile_n=256, tile_k=128)),
    (1, 1, 2048, 1536, 4096, dict(cta_group=2, tile_n=512, tile_k=128)),
    (4, 2, 1024, 1536, 2048, dict(cta_group=1, tile_n=256, tile_k=256)),
    (4, 2, 1024, 1536, 2048, dict(cta_group=2, tile_n=256, tile_k=256)),
])
def test_matches_cutlass_on_same_inputs(pkg, orc, cutlass, cuda, kid, dtype, m, n, k, knobs):
    ops = operands(pkg, dtype, m, n, k, cuda)
    pkg.gemm(ops, **knobs)
    ref = run_cutlass(cutlass, kid, ops)
    assert rel(ops.d, ref) <= TOL[dtype]


def test_nvfp4_cutlass_reads_the_same_scale_layout(pkg, orc, cutlass, cuda):
    """With B = identity (scales 1.0) both kernels reproduce A's dequantised values
    exactly, so CUTLASS's K-major 128x4 scale atom and ours are the same bytes."""
    import numpy as np
    m, n, k = 256, 256, 512
    ops = pkg.make_operands(pkg.NVFP4, m, n, k, seed=2, device=cuda)
    packed = torch.zeros((n, k // 2), dtype=torch.uint8)
    for i in range(n):
        packed[i, i // 2] = 0x2 << (4 * (i % 2))        # e2m1 1.0 on the diagonal
    ops.b.copy_(packed.to(cuda))
    ops.sfb.fill_(0x38)                                   # ue4m3 1.0
    ref = run_cutlass(cutlass, 4, ops)
    A = orc.dequant_nvfp4(ops.a.cpu().numpy(), ops.sfa.cpu().numpy(), k)
    got = orc.bf16_bits_to_f32(ref.t().contiguous().view(torch.int16).cpu().numpy().view(np.uint16))
    np.testing.assert_array_equal(got, A[:, :n])


# The bench's configurations at full size, each against the CUTLASS kernel of its dtype.
FULL = [
    ("bf16_8192", 0), ("bf16_8192_1sm", 0), ("e4m3_16384_2sm", 1), ("e4m3_8192", 1), ("nvfp4_mlp", 4),
    ("e4m3_nsplit", 1),
]


@pytest.mark.parametrize("name,kid", FULL)
def test_bench_configurations_match_cutlass_full_size(pkg, orc, cutlass, cuda, name, kid):
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_for_cutlass", Path(__file__).resolve().parent.parent / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    wl = bench.WORKLOADS[name]
    dt = {"bf16": pkg.BF16, "e4m3": pkg.FP8_E4M3, "nvfp4": pkg.NVFP4}[wl["dtype"]]
    dist = {"uniform": pkg.UNIFORM, "normal": pkg.NORMAL}
    ops = pkg.make_operands(dt, wl["m"], wl["n"], wl["k"], seed=0, device=cuda,
                            a_dist=dist[wl["a"][0]], a_scale=wl["a"][1], b_dist=dist[wl["b"][0]], b_scale=wl["b"][1])
    pkg.gemm(ops, **wl["knobs"])
    ref = run_cutlass(cutlass, kid, ops)
    assert rel(ops.d, ref) <= TOL[dt]
