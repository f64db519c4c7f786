"""ctypes wrapper over oracle/liboracle.so -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg (and
its ``--impl reference`` arm) import this module, and only as the checker or
the reported CPU baseline.  The GPU product path never imports it.

The C sources (oracle.c, cpu_gemm.c) restate the reference's arithmetic
(cutlass_mainloop/cutlass_gemm_bench.cu:101-156,249: D = alpha * A . B^T,
fp32 accumulate, bf16 column-major D) and the benchmark's seeded inputs; see
the header of oracle.c for the full list and the parity status.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

BF16, FP8_E4M3, NVFP4 = 0, 1, 2
UNIFORM, NORMAL = 0, 1


def build(force: bool = False) -> Path:
    """Compile liboracle.so with oracle/Makefile (gcc + OpenMP)."""
    if force or not _LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = C.CDLL(str(_LIB_PATH))
        u64, i64, f32, f64, vp = C.c_uint64, C.c_int64, C.c_float, C.c_double, C.c_void_p
        L.orc_bits.restype = u64; L.orc_bits.argtypes = [u64, u64, u64]
        L.orc_uniform.restype = f32; L.orc_uniform.argtypes = [u64, u64, u64]
        L.orc_normal.restype = f32; L.orc_normal.argtypes = [u64, u64, u64]
        L.orc_f32_to_bf16.restype = C.c_uint16; L.orc_f32_to_bf16.argtypes = [f32]
        L.orc_bf16_to_f32.restype = f32; L.orc_bf16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_e4m3.restype = C.c_uint8; L.orc_f32_to_e4m3.argtypes = [f32]
        L.orc_e4m3_to_f32.restype = f32; L.orc_e4m3_to_f32.argtypes = [C.c_uint8]
        L.orc_f32_to_e2m1.restype = C.c_uint8; L.orc_f32_to_e2m1.argtypes = [f32]
        L.orc_e2m1_to_f32.restype = f32; L.orc_e2m1_to_f32.argtypes = [C.c_uint8]
        L.orc_ue4m3_round_up.restype = C.c_uint8; L.orc_ue4m3_round_up.argtypes = [f32]
        L.orc_generate.restype = None
        L.orc_generate.argtypes = [vp, C.c_int, C.c_int, f32, u64, u64, i64, i64, i64, i64]
        L.orc_sf_offset.restype = i64; L.orc_sf_offset.argtypes = [i64, i64, i64]
        L.orc_generate_nvfp4.restype = None
        L.orc_generate_nvfp4.argtypes = [vp, vp, f32, u64, u64, i64, i64, i64]
        L.orc_dequant.restype = None
        L.orc_dequant.argtypes = [vp, C.c_int, i64, i64, i64, vp]
        L.orc_dequant_nvfp4.restype = None
        L.orc_dequant_nvfp4.argtypes = [vp, vp, i64, i64, vp]
        L.orc_gemm_f64.restype = None
        L.orc_gemm_f64.argtypes = [vp, vp, i64, i64, i64, vp, i64, vp, i64, f64, vp]
        L.orc_rel_frobenius.restype = f64
        L.orc_rel_frobenius.argtypes = [vp, i64, vp, i64, vp, i64, vp]
        L.orc_gemm_omp_f32.restype = None
        L.orc_gemm_omp_f32.argtypes = [vp, vp, i64, i64, i64, f32, vp, i64]
        L.orc_num_threads.restype = C.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"] or a.flags["F_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- generation
def generate(rows: int, cols: int, dtype: int, dist: int, scale: float, seed: int, stream: int,
             row0: int = 0) -> np.ndarray:
    """Seeded matrix, raw storage: uint16 (bf16 bits) or uint8 (e4m3 bits), row-major."""
    out = np.empty((rows, cols), dtype=np.uint16 if dtype == BF16 else np.uint8)
    lib().orc_generate(_p(out), dtype, dist, scale, seed, stream, row0, rows, cols, cols)
    return out


def sf_bytes(rows: int, cols: int) -> int:
    """Bytes of the interleaved NVFP4 scale buffer for rows x cols (rows padded to 128)."""
    return ((rows + 127) // 128) * (cols // 64) * 512


def generate_nvfp4(rows: int, cols: int, scale: float, seed: int, stream: int, row0: int = 0):
    """(packed e2m1 uint8 [rows, cols/2], ue4m3 scales uint8 [sf_bytes]) for normal(0,1)*scale."""
    assert rows % 128 == 0 and cols % 64 == 0 and row0 % 128 == 0
    packed = np.empty((rows, cols // 2), dtype=np.uint8)
    scales = np.zeros(sf_bytes(rows, cols), dtype=np.uint8)
    lib().orc_generate_nvfp4(_p(packed), _p(scales), scale, seed, stream, row0, rows, cols)
    return packed, scales


# ---------------------------------------------------------------- dequantise
def dequant(raw: np.ndarray, dtype: int) -> np.ndarray:
    rows, cols = raw.shape
    raw = np.ascontiguousarray(raw)
    out = np.empty((rows, cols), dtype=np.float32)
    lib().orc_dequant(_p(raw), dtype, rows, cols, cols, _p(out))
    return out


def dequant_nvfp4(packed: np.ndarray, scales: np.ndarray, cols: int) -> np.ndarray:
    rows = packed.shape[0]
    out = np.empty((rows, cols), dtype=np.float32)
    lib().orc_dequant_nvfp4(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales)),
                            rows, cols, _p(out))
    return out


# ---------------------------------------------------------------- GEMM
def gemm_f64(A: np.ndarray, B: np.ndarray, alpha: float = 1.0, rows=None, cols=None) -> np.ndarray:
    """fp64 reference over fp32 dequantised A [M,K], B [N,K]; returns the
    selected block of D (len(rows) x len(cols), as a C-ordered float64 array)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N = B.shape[0]
    ri = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    ci = None if cols is None else np.ascontiguousarray(cols, dtype=np.int64)
    nr = M if ri is None else len(ri)
    nc = N if ci is None else len(ci)
    out = np.empty((nc, nr), dtype=np.float64)  # column-major selection
    lib().orc_gemm_f64(_p(A), _p(B), M, N, K,
                       None if ri is None else _p(ri), nr,
                       None if ci is None else _p(ci), nc, alpha, _p(out))
    return np.ascontiguousarray(out.T)


def rel_frobenius(D_bf16_colmajor: np.ndarray, M: int, Dref: np.ndarray, rows=None, cols=None) -> float:
    """||D - Dref||_F / ||Dref||_F; D is the raw uint16 column-major buffer (ldd = M)."""
    D = np.ascontiguousarray(D_bf16_colmajor).reshape(-1)
    ri = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    ci = None if cols is None else np.ascontiguousarray(cols, dtype=np.int64)
    nr, nc = Dref.shape
    ref_cm = np.ascontiguousarray(Dref.T)
    return lib().orc_rel_frobenius(_p(D), M, None if ri is None else _p(ri), nr,
                                   None if ci is None else _p(ci), nc, _p(ref_cm))


def gemm_omp_f32(A: np.ndarray, B: np.ndarray, alpha: float = 1.0, D: np.ndarray | None = None,
                 ldd: int | None = None) -> np.ndarray:
    """CPU baseline: OpenMP fp32-accumulate GEMM, bf16 column-major output (raw uint16)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N = B.shape[0]
    if ldd is None:
        ldd = M
    if D is None:
        D = np.empty(ldd * N, dtype=np.uint16)
    lib().orc_gemm_omp_f32(_p(A), _p(B), M, N, K, alpha, _p(D), ldd)
    return D


def num_threads() -> int:
    return int(lib().orc_num_threads())


def bf16_bits_to_f32(x: np.ndarray) -> np.ndarray:
    return (x.astype(np.uint32) << 16).view(np.float32)
