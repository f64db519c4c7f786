"""Torch-facing helpers over the C ABI: operand allocation, seeded generation
and a one-call GEMM.  Torch tensors only carry device memory and streams; all
arithmetic runs in libgemm_sm100a.so kernels.

Operand layouts follow the reference (cutlass_gemm_mainloop/cutlass_gemm_bench.cu:103-105):
A is M x K row-major, B is N x K (K contiguous), D is M x N column-major bf16,
stored here as a (N, M) row-major tensor.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import (BF16, FP8_E4M3, NVFP4, NORMAL, UNIFORM, GemmError, generate, generate_nvfp4,
               launch, make_args, read_status, sf_bytes)


@dataclass
class Operands:
    dtype: int
    m: int
    n: int
    k: int
    a: torch.Tensor                 # bf16 (m, k) | uint8 (m, k) e4m3 | uint8 (m, k/2) packed e2m1
    b: torch.Tensor                 # same, (n, ...)
    d: torch.Tensor                 # bf16 (n, m): column-major m x n
    sfa: torch.Tensor | None = None # uint8 interleaved ue4m3 scales (NVFP4)
    sfb: torch.Tensor | None = None
    n0: int = 0                     # global column offset of this B/D slice (N-split)


def _storage_dtype(dtype: int):
    return torch.bfloat16 if dtype == BF16 else torch.uint8


def _cols(dtype: int, k: int) -> int:
    return k // 2 if dtype == NVFP4 else k


def make_operands(dtype: int, m: int, n: int, k: int, *, seed: int = 0,
                  a_dist: int = UNIFORM, a_scale: float = 1.0,
                  b_dist: int = UNIFORM, b_scale: float = 1.0,
                  n0: int = 0, device: str | torch.device = "cuda", stream: int | None = None) -> Operands:
    """Allocate and generate seeded operands on `device`.

    A uses generator stream 0, B stream 1 (rows n0 .. n0+n of the global B, so
    an N-split shard regenerates exactly its slice).  NVFP4 inputs are normal
    draws quantised per 16-element block (the distribution arguments select
    the scale only).
    """
    dev = torch.device(device)
    st = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    sdt = _storage_dtype(dtype)
    a = torch.empty((m, _cols(dtype, k)), dtype=sdt, device=dev)
    b = torch.empty((n, _cols(dtype, k)), dtype=sdt, device=dev)
    d = torch.empty((n, m), dtype=torch.bfloat16, device=dev)
    sfa = sfb = None
    if dtype == NVFP4:
        if m % 128 or n % 128 or n0 % 128 or k % 64:
            raise ValueError("NVFP4 operands need m, n, n0 multiples of 128 and k a multiple of 64")
        sfa = torch.zeros(sf_bytes(m, k), dtype=torch.uint8, device=dev)
        sfb = torch.zeros(sf_bytes(n, k), dtype=torch.uint8, device=dev)
        generate_nvfp4(a.data_ptr(), sfa.data_ptr(), a_scale, seed, 0, 0, m, k, st)
        generate_nvfp4(b.data_ptr(), sfb.data_ptr(), b_scale, seed, 1, n0, n, k, st)
    else:
        generate(a.data_ptr(), dtype, a_dist, a_scale, seed, 0, 0, m, k, k, st)
        generate(b.data_ptr(), dtype, b_dist, b_scale, seed, 1, n0, n, k, k, st)
    return Operands(dtype, m, n, k, a, b, d, sfa, sfb, n0)


def gemm_into(ops: Operands, *, alpha: float = 1.0, status: torch.Tensor | None = None,
              stream: int | None = None, **knobs) -> None:
    """Enqueue D = alpha * A . B^T into ops.d (one launch of the library kernel)."""
    st = torch.cuda.current_stream(ops.a.device).cuda_stream if stream is None else stream
    args = make_args(dtype=ops.dtype, m=ops.m, n=ops.n, k=ops.k,
                     a=ops.a.data_ptr(), b=ops.b.data_ptr(), d=ops.d.data_ptr(),
                     lda=ops.k, ldb=ops.k, ldd=ops.m,
                     sfa=None if ops.sfa is None else ops.sfa.data_ptr(),
                     sfb=None if ops.sfb is None else ops.sfb.data_ptr(),
                     alpha=alpha, status=None if status is None else status.data_ptr(), **knobs)
    launch(args, st)


def gemm(ops: Operands, *, alpha: float = 1.0, check_status: bool = True, **knobs) -> torch.Tensor:
    """Run one GEMM synchronously and return D as an (m, n) view (column-major storage)."""
    status = torch.zeros(1, dtype=torch.int32, device=ops.a.device)
    gemm_into(ops, alpha=alpha, status=status, **knobs)
    rc, detail = read_status(status.data_ptr(), torch.cuda.current_stream(ops.a.device).cuda_stream)
    if check_status and rc != 0:
        raise GemmError(rc, f"device status 0x{detail & 0xFFFFFFFF:08x}")
    return ops.d.t()


def flops(m: int, n: int, k: int) -> float:
    """2*M*N*K, the reference's FLOP count (cutlass_gemm_bench.cu:249)."""
    return 2.0 * m * n * k
