"""gemm_sm100a_launch inside a CUDA graph: a launch captured on a stream and
replayed gives the bits of the same launch made directly (1-SM, CTA pair,
NVFP4), and replays of a graph of several launches keep giving them.  The
launcher allocates nothing and does not query a capturing stream's device,
so the capture stays valid; the first launch of each kernel on a device
(which raises its shared-memory limit) is made before capturing."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,m,n,k,knobs", [
    (0, 256, 256, 256, dict(tile_n=256, tile_k=64, stages=4)),
    (0, 1024, 1024, 512, dict(cta_group=2, tile_n=256, tile_k=64, raster_group=4)),
    (1, 512, 768, 1024, dict(cta_group=2, tile_n=256, tile_k=128)),
    (2, 512, 512, 1024, dict(cta_group=2, tile_n=256, tile_k=256)),
])
def test_captured_launch_replays_the_direct_result(pkg, cuda, dtype, m, n, k, knobs):
    kw = {} if dtype != pkg.FP8_E4M3 else dict(a_dist=pkg.NORMAL, a_scale=0.25, b_dist=pkg.NORMAL, b_scale=0.25)
    ops = pkg.make_operands(dtype, m, n, k, seed=9, device=cuda, **kw)
    direct = torch.empty_like(ops.d)
    replayed = torch.full_like(ops.d, float("nan"))
    common = dict(dtype=dtype, m=m, n=n, k=k, a=ops.a.data_ptr(), b=ops.b.data_ptr(),
                  sfa=None if ops.sfa is None else ops.sfa.data_ptr(),
                  sfb=None if ops.sfb is None else ops.sfb.data_ptr(), **knobs)
    a_direct = pkg.make_args(d=direct.data_ptr(), **common)
    a_graph = pkg.make_args(d=replayed.data_ptr(), **common)
    L = pkg.lib()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        assert L.gemm_sm100a_launch(C.byref(a_direct), C.c_void_p(stream.cuda_stream)) == pkg.OK
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(3):
            assert L.gemm_sm100a_launch(C.byref(a_graph), C.c_void_p(stream.cuda_stream)) == pkg.OK
    assert torch.isnan(replayed).all()                       # capturing launched nothing
    for _ in range(2):
        replayed.fill_(float("nan"))
        with torch.cuda.stream(stream):
            graph.replay()
        stream.synchronize()
        assert torch.equal(replayed, direct)
    del graph
