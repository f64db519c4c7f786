"""GEMM fused with the all-gather of D (gemm_sm100a_launch_gather).

The N-split multi-GPU configuration (each GPU owns a column slab of B and D)
gathers the full D on every GPU.  The fused entry point makes each GPU's
epilogue store its D block into the other GPUs' full D as well, so the gather
overlaps the GEMM.  Checks are bitwise against the plain launch (same kernel,
same accumulation order)."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _args(pkg, ops, d_ptr, **knobs):
    return pkg.make_args(dtype=ops.dtype, m=ops.m, n=ops.n, k=ops.k, a=ops.a.data_ptr(), b=ops.b.data_ptr(),
                         d=d_ptr, lda=ops.k, ldb=ops.k, ldd=ops.m,
                         sfa=None if ops.sfa is None else ops.sfa.data_ptr(),
                         sfb=None if ops.sfb is None else ops.sfb.data_ptr(), **knobs)


@pytest.mark.parametrize("n", [1536, 1500])                                      # whole tiles, and an N tail
@pytest.mark.parametrize("knobs", [dict(cta_group=2, tile_n=512, tile_k=64),    # one accumulator: staged epilogue
                                   dict(cta_group=1, tile_n=256, tile_k=64),    # double-buffered epilogue
                                   dict(cta_group=1, tile_n=16, tile_k=64),     # 16-column chunks
                                   dict(cta_group=1, tile_m=64, tile_n=256, tile_k=64)])  # M = 64 lane layout
def test_extra_destinations_on_one_gpu_match_d(pkg, cuda, knobs, n):
    m, k = 512, 1024
    ops = pkg.make_operands(pkg.BF16, m, n, k, seed=3, device=cuda)
    extra = [torch.full_like(ops.d, 7) for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream
    pkg.launch_gather(_args(pkg, ops, ops.d.data_ptr(), **knobs), [e.data_ptr() for e in extra], st)
    torch.cuda.synchronize()
    plain = torch.empty_like(ops.d)
    pkg.launch(_args(pkg, ops, plain.data_ptr(), **knobs), st)
    torch.cuda.synchronize()
    assert torch.equal(ops.d, plain)
    for e in extra:
        assert torch.equal(e, plain)


def test_bad_destinations_are_rejected_before_launch(pkg, cuda):
    ops = pkg.make_operands(pkg.BF16, 256, 256, 256, seed=0, device=cuda)
    args = _args(pkg, ops, ops.d.data_ptr())
    st = torch.cuda.current_stream().cuda_stream
    L = pkg.lib()
    host = np.zeros(256 * 256, dtype=np.uint16)
    # Exact-size allocations (torch's caching allocator would hand out slices of larger segments).
    from cuda.bindings import runtime as rt
    err, short = rt.cudaMalloc(256 * 256)             # half of the 256 x 256 bf16 block
    assert err == rt.cudaError_t.cudaSuccess
    err, exact = rt.cudaMalloc(256 * 256 * 2)         # exactly one block
    assert err == rt.cudaError_t.cudaSuccess
    for peers, n in [([host.ctypes.data], 1),                     # host memory
                     ([ops.d.data_ptr() + 2], 1),                 # not 16-byte aligned
                     ([ops.d.data_ptr()] * 8, 8),                 # more than 7 destinations
                     ([int(short)], 1),                           # allocation shorter than the block
                     ([int(exact) + 64 * 256 * 2], 1)]:           # block runs past the end of its allocation
        arr = (C.c_void_p * len(peers))(*peers)
        assert L.gemm_sm100a_launch_gather(C.byref(args), arr, n, C.c_void_p(st)) == pkg.ERR_BAD_ARGS
    # the exact allocation itself is accepted
    arr = (C.c_void_p * 1)(int(exact))
    assert L.gemm_sm100a_launch_gather(C.byref(args), arr, 1, C.c_void_p(st)) == pkg.OK
    torch.cuda.synchronize()
    rt.cudaFree(short)
    rt.cudaFree(exact)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("dtype,knobs", [(0, dict(cta_group=2, tile_n=512, tile_k=64)),
                                         (1, dict(cta_group=2, tile_n=512, tile_k=128))])
def test_nsplit_gather_across_two_gpus(pkg, dtype, knobs):
    """Each GPU computes its column slab and writes it into both GPUs' full D."""
    G, m, n_total, k = 2, 1024, 2048, 1024
    n_local = n_total // G
    devs = [torch.device("cuda", i) for i in range(G)]
    ops, full, streams = [], [], []
    for i, dev in enumerate(devs):
        with torch.cuda.device(dev):
            kw = {} if dtype == 0 else dict(a_dist=pkg.NORMAL, a_scale=0.25, b_dist=pkg.NORMAL, b_scale=0.25)
            ops.append(pkg.make_operands(dtype, m, n_local, k, seed=5, n0=i * n_local, device=dev, **kw))
            full.append(torch.zeros((n_total, m), dtype=torch.bfloat16, device=dev))
            streams.append(torch.cuda.current_stream(dev).cuda_stream)
    for i in range(G):
        with torch.cuda.device(devs[i]):
            mine = full[i][i * n_local:(i + 1) * n_local]
            peers = [full[j][i * n_local:(i + 1) * n_local].data_ptr() for j in range(G) if j != i]
            pkg.launch_gather(_args(pkg, ops[i], mine.data_ptr(), **knobs), peers, streams[i])
    for dev in devs:
        torch.cuda.synchronize(dev)
    for i in range(G):
        with torch.cuda.device(devs[i]):
            pkg.launch(_args(pkg, ops[i], ops[i].d.data_ptr(), **knobs), streams[i])
            torch.cuda.synchronize(devs[i])
    slabs = torch.cat([o.d.cpu() for o in ops])
    for f in full:
        assert torch.equal(f.cpu(), slabs)
