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
