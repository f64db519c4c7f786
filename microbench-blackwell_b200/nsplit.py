"""N-split of one GEMM across ranks (one process per GPU).

D = A . B^T is partitioned along N: rank g owns B rows / D columns
[g*N/G, (g+1)*N/G).  A is replicated (each rank regenerates it from the seed,
so A never crosses the interconnect); because D is column-major (M
contiguous), each rank's D slice is one contiguous block and the optional
gather of the full D is a single all-gather with no re-layout.  There is no
collective on the GEMM's data path.

The reference is single-GPU (cutlass_gemm_mainloop/cutlass_gemm_bench.cu:188-190,
sm_count = 1); this module is the multi-GPU layer the benchmark plan adds.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Slab:
    rank: int
    world: int
    n_total: int
    n0: int          # first global column of this rank
    n_local: int     # columns owned


def partition(n_total: int, world: int, rank: int, align: int = 1) -> Slab:
    """Even column split; `align` keeps every slab a multiple of `align` columns
    (e.g. the tile width or 128 for NVFP4 scale atoms)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    if n_total % (world * align) != 0:
        raise ValueError(f"N={n_total} does not split into {world} slabs of a multiple of {align}")
    n_local = n_total // world
    return Slab(rank, world, n_total, rank * n_local, n_local)


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (the slowest rank's time); identity without a process group."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_columns(d_local, n_total: int):
    """All-gather the column-major D slices (each a (n_local, M) tensor whose
    rows are D's columns) into the full (n_total, M) D on every rank."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size()
    n_local, m = d_local.shape
    if n_local * world != n_total:
        raise ValueError("slab sizes do not add up to N")
    full = torch.empty((n_total, m), dtype=d_local.dtype, device=d_local.device)
    dist.all_gather_into_tensor(full, d_local.contiguous())
    return full


def fused_gather_timing(pkg, g, ops, slab, full_ref, stream, dev, local_rank, reps: int = 3) -> dict:
    """Time the fused GEMM + all-gather (gemm_sm100a_launch_gather) of this rank's slab.

    Every rank allocates its full column-major D (cudaMalloc, exact size) and shares it
    with the others by CUDA IPC; each launch then writes this rank's D block into its own
    full D and, over NVLink, into the same block of every peer's full D.  Returns the
    max-over-ranks time of the fastest of `reps` launches and whether the gathered D
    equals `full_ref` (the NCCL all-gather result) bit for bit.  Every rank takes the same
    collective steps, and the IPC mappings are closed and the buffer freed before return."""
    import ctypes as C
    import torch
    import torch.distributed as dist
    from cuda.bindings import runtime as rt

    def ok(err):
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"CUDA runtime error {err}")

    world, rank = dist.get_world_size(), dist.get_rank()
    m = ops.m
    nbytes = slab.n_total * m * 2
    err, base = rt.cudaMalloc(nbytes)
    ok(err)
    opened = []
    try:
        err, handle = rt.cudaIpcGetMemHandle(base)
        ok(err)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle.reserved))
        peers = {}
        for j in range(world):
            if j == rank:
                continue
            h = rt.cudaIpcMemHandle_t()
            h.reserved = handles[j]
            err, ptr = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
            ok(err)
            opened.append(ptr)
            peers[j] = int(ptr)
        off = slab.n0 * m * 2                                   # this rank's column block
        args = pkg.GemmArgs.from_buffer_copy(g)
        args.d, args.ldd = int(base) + off, m
        peer_ptrs = [peers[j] + off for j in sorted(peers)]
        st = stream.cuda_stream
        pkg.launch_gather(args, peer_ptrs, st)                 # warm-up
        stream.synchronize()
        times = []
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(reps):
            dist.barrier(device_ids=[local_rank])
            e0.record(stream)
            pkg.launch_gather(args, peer_ptrs, st)
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        dist.barrier(device_ids=[local_rank])                  # every peer's stores have landed
        got = torch.empty_like(full_ref)
        ok(rt.cudaMemcpy(got.data_ptr(), base, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)[0])
        same = bool(torch.equal(got, full_ref))
        ms = max_over_ranks(min(times), device=dev)
        sent = (world - 1) * slab.n_local * m * 2
        return {"ms": ms, "bytes_sent_per_rank": sent, "GBps_per_rank": sent / (ms * 1e-3) / 1e9,
                "matches_nccl_allgather": same,
                "path": "gemm_sm100a_launch_gather: staged epilogue blocks stored into every peer's full D "
                        "(CUDA IPC mappings, NVLink), no loads from peers"}
    finally:
        dist.barrier(device_ids=[local_rank])
        for ptr in opened:
            rt.cudaIpcCloseMemHandle(ptr)
        dist.barrier(device_ids=[local_rank])
        rt.cudaFree(base)
