"""Agreement with the reference's own kernel family: the CUTLASS SM100 GEMM
(1SM, the reference's best tiles) run by oracle/_ref/libcutlass_ref.so on the
same seeded device inputs.  Tolerance: relative Frobenius 2e-3 between the two
bf16 results (and each against the fp64 oracle)."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libcutlass_ref.so"


@pytest.fixture(scope="module")
def cutlass(cuda):
    if not LIB.exists():
        pytest.skip("oracle/_ref/libcutlass_ref.so not built (needs the reference tree at build time)")
    L = C.CDLL(str(LIB))
    L.cutlass_ref_gemm.restype = C.c_int
    L.cutlass_ref_gemm.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                   C.c_int, C.c_void_p]
    return L


def rel(a, b):
    a = a.float(); b = b.float()
    return (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item()


@pytest.mark.parametrize("dtype,m,n,k,knobs", [
    (0, 2048, 2048, 2048, dict(cta_group=1, tile_n=256, tile_k=64, stages=4)),
    (0, 2048, 2048, 2048, dict(cta_group=2, tile_n=512, tile_k=64)),
    (1, 2048, 1536, 4096, dict(cta_group=1, tile_n=256, tile_k=128)),
    (1, 2048, 1536, 4096, dict(cta_group=2, tile_n=256, tile_k=128)),
])
def test_matches_cutlass_on_same_inputs(pkg, orc, cutlass, cuda, dtype, m, n, k, knobs):
    kw = {} if dtype == 0 else dict(a_dist=pkg.NORMAL, a_scale=0.25, b_dist=pkg.NORMAL, b_scale=0.25)
    ops = pkg.make_operands(dtype, m, n, k, seed=3, device=cuda, **kw)
    pkg.gemm(ops, **knobs)
    ref = torch.empty_like(ops.d)
    rc = cutlass.cutlass_ref_gemm(dtype, ops.a.data_ptr(), ops.b.data_ptr(), ref.data_ptr(), m, n, k, 0,
                                  torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    assert rel(ops.d, ref) <= 2e-3
