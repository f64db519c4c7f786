"""N-split host logic with world_size 2 on CPU (gloo): partition, max-over-ranks
timing and the all-gather of column-major D slices reproduce the full GEMM."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_pkg


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, m, n, k, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        load_pkg()
        import microbench_blackwell_b200.nsplit as ns
        slab = ns.partition(n, world, rank, align=8)
        g = torch.Generator().manual_seed(0)
        A = torch.randn(m, k, generator=g)                     # replicated: same seed on every rank
        Bfull = torch.randn(n, k, generator=g)
        B = Bfull[slab.n0:slab.n0 + slab.n_local]
        d_local = (B @ A.t()).contiguous()                     # (n_local, m) = column-major m x n_local
        full = ns.gather_columns(d_local, n)
        ref = Bfull @ A.t()
        ok = torch.allclose(full, ref, rtol=1e-5, atol=1e-5)
        slow = ns.max_over_ranks(float(rank + 1))
        q.put((rank, ok, slow, slab.n0, slab.n_local))
    finally:
        dist.destroy_process_group()


def test_nsplit_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 48, 64, 32, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(ok for _, ok, _, _, _ in res)
    assert [s for _, _, s, _, _ in res] == [2.0, 2.0]          # max over ranks
    assert [(n0, nl) for _, _, _, n0, nl in res] == [(0, 32), (32, 32)]


def test_partition_rejects_uneven_split():
    load_pkg()
    import microbench_blackwell_b200.nsplit as ns
    with pytest.raises(ValueError):
        ns.partition(100, 3, 0)
    with pytest.raises(ValueError):
        ns.partition(64, 2, 2)
    s = ns.partition(57344, 8, 7, align=256)
    assert (s.n0, s.n_local) == (50176, 7168)
