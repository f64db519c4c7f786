"""Python binding of libgemm_sm100a.so, the B200 (sm_100a) dense GEMM mainloop.

The library replaces the CUTLASS SM100 GEMM driven by the reference benchmark
cutlass_gemm_mainloop/cutlass_gemm_bench.cu (GEMM types :101-156; the
Gemm::can_implement / initialize / run sequence :206-239).  This module is the
ctypes view of the C ABI in include/gemm_sm100a.h: every call goes through
``gemm_sm100a_launch``; PyTorch only provides device memory and streams.

There is no fallback: if the shared library is missing or fails to load,
``lib()`` raises, and every entry point raises ``GemmError`` on a non-zero
return code (the reference's ``can_implement`` / ``initialize`` failures exit
with status 1, cutlass_gemm_bench.cu:211-224).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libgemm_sm100a.so"

# Element types; values equal the reference's DTYPE_ID (cutlass_gemm_bench.cu:57-66) + NVFP4.
BF16, FP8_E4M3, NVFP4 = 0, 1, 2
DTYPE_NAMES = {BF16: "BF16", FP8_E4M3: "FP8_E4M3", NVFP4: "NVFP4"}
DTYPE_BITS = {BF16: 16, FP8_E4M3: 8, NVFP4: 4}

OK, ERR_CANNOT_IMPLEMENT, ERR_LAUNCH, ERR_TIMEOUT, ERR_BAD_ARGS = 0, -1, -2, -3, -4
FLAG_INJECT_STALL, FLAG_DIRECT_EPILOGUE = 1, 2
COL_MAJOR, ROW_MAJOR = 0, 1

UNIFORM, NORMAL = 0, 1


class GemmArgs(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32), ("dtype", C.c_int32),
        ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
        ("a", C.c_void_p), ("lda", C.c_int64),
        ("b", C.c_void_p), ("ldb", C.c_int64),
        ("d", C.c_void_p), ("ldd", C.c_int64),
        ("sfa", C.c_void_p), ("sfb", C.c_void_p),
        ("alpha", C.c_float),
        ("tile_m", C.c_int32), ("tile_n", C.c_int32), ("tile_k", C.c_int32), ("stages", C.c_int32),
        ("cta_group", C.c_int32), ("cluster_m", C.c_int32), ("max_ctas", C.c_int32),
        ("raster_group", C.c_int32),
        ("status", C.c_void_p), ("timeout_ms", C.c_uint32), ("flags", C.c_uint32),
        ("l2_prefetch", C.c_int32),
        ("clock_out", C.c_void_p),
        ("beta", C.c_float), ("c", C.c_void_p), ("ldc", C.c_int64), ("d_layout", C.c_int32),
        ("scale_a", C.c_float), ("scale_b", C.c_float),
    ]


class GemmInfo(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("tile_m", C.c_int32), ("tile_n", C.c_int32), ("tile_k", C.c_int32), ("stages", C.c_int32),
        ("cta_group", C.c_int32), ("cluster_m", C.c_int32), ("max_stages", C.c_int32),
        ("smem_bytes_per_stage", C.c_int64), ("smem_bytes", C.c_int64),
        ("tmem_columns", C.c_int32), ("grid_ctas", C.c_int32), ("num_tiles", C.c_int64),
        ("num_sms", C.c_int32), ("can_implement", C.c_int32), ("reason", C.c_char * 128),
        ("epilogue_staging_buffers", C.c_int32),
    ]


# Every symbol include/gemm_sm100a.h declares.
EXPORTED = (
    "gemm_sm100a_query", "gemm_sm100a_launch", "gemm_sm100a_launch_gather", "gemm_sm100a_read_status",
    "gemm_sm100a_strerror", "gemm_sm100a_version",
    "gemm_sm100a_generate", "gemm_sm100a_generate_nvfp4", "gemm_sm100a_umma_peak",
    "gemm_sm100a_tma_read_probe",
)


class GemmError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {strerror(code)} ({code})")


_lib = None


def lib():
    """Load libgemm_sm100a.so (raises if it was not built: no fallback path exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR}` "
                               "(or __graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(str(LIB_PATH))
        vp, i32, i64, u64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float
        L.gemm_sm100a_query.restype = C.c_int
        L.gemm_sm100a_query.argtypes = [C.POINTER(GemmArgs), C.POINTER(GemmInfo)]
        L.gemm_sm100a_launch.restype = C.c_int
        L.gemm_sm100a_launch.argtypes = [C.POINTER(GemmArgs), vp]
        L.gemm_sm100a_launch_gather.restype = C.c_int
        L.gemm_sm100a_launch_gather.argtypes = [C.POINTER(GemmArgs), C.POINTER(vp), C.c_int32, vp]
        L.gemm_sm100a_read_status.restype = C.c_int
        L.gemm_sm100a_read_status.argtypes = [vp, vp, C.POINTER(i32)]
        L.gemm_sm100a_strerror.restype = C.c_char_p
        L.gemm_sm100a_strerror.argtypes = [C.c_int]
        L.gemm_sm100a_version.restype = C.c_int
        L.gemm_sm100a_version.argtypes = []
        L.gemm_sm100a_generate.restype = C.c_int
        L.gemm_sm100a_generate.argtypes = [vp, i32, i32, f32, u64, u64, i64, i64, i64, i64, vp]
        L.gemm_sm100a_generate_nvfp4.restype = C.c_int
        L.gemm_sm100a_generate_nvfp4.argtypes = [vp, vp, f32, u64, u64, i64, i64, i64, vp]
        L.gemm_sm100a_umma_peak.restype = C.c_int
        L.gemm_sm100a_umma_peak.argtypes = [i32, i32, i32, i32, i32, vp, vp]
        L.gemm_sm100a_tma_read_probe.restype = C.c_int
        L.gemm_sm100a_tma_read_probe.argtypes = [vp, i64, i32, i32, i32, i32, vp, vp]
        _lib = L
    return _lib


def strerror(code: int) -> str:
    try:
        return lib().gemm_sm100a_strerror(code).decode()
    except RuntimeError:
        return f"error {code}"


def make_args(*, dtype: int, m: int, n: int, k: int, a: int, b: int, d: int,
              lda: int | None = None, ldb: int | None = None, ldd: int | None = None,
              sfa: int | None = None, sfb: int | None = None, alpha: float = 1.0,
              tile_m: int = 0, tile_n: int = 0, tile_k: int = 0, stages: int = 0,
              cta_group: int = 0, cluster_m: int = 0, max_ctas: int = 0, raster_group: int = 0,
              status: int | None = None, timeout_ms: int = 0, flags: int = 0,
              l2_prefetch: int = 0, clock_out: int | None = None, beta: float = 0.0,
              c: int | None = None, ldc: int | None = None, d_layout: int = 0,
              scale_a: float = 1.0, scale_b: float = 1.0) -> GemmArgs:
    """GemmArgs from raw device addresses (ints).  Leading dimensions default to packed
    (ldd and ldc follow d_layout: m for column-major, n for row-major)."""
    g = GemmArgs()
    g.struct_size = C.sizeof(GemmArgs)
    g.dtype = dtype
    g.m, g.n, g.k = m, n, k
    g.a, g.lda = a, (k if lda is None else lda)
    g.b, g.ldb = b, (k if ldb is None else ldb)
    packed_ld = m if d_layout == COL_MAJOR else n
    g.d, g.ldd = d, (packed_ld if ldd is None else ldd)
    g.sfa, g.sfb = sfa, sfb
    g.alpha = alpha
    g.tile_m, g.tile_n, g.tile_k, g.stages = tile_m, tile_n, tile_k, stages
    g.cta_group, g.cluster_m, g.max_ctas, g.raster_group = cta_group, cluster_m, max_ctas, raster_group
    g.status = status
    g.timeout_ms, g.flags = timeout_ms, flags
    g.l2_prefetch = l2_prefetch
    g.clock_out = clock_out
    g.beta, g.c, g.ldc = beta, c, (packed_ld if ldc is None else ldc)
    g.d_layout, g.scale_a, g.scale_b = d_layout, scale_a, scale_b
    return g


def query(args: GemmArgs) -> tuple[int, GemmInfo]:
    info = GemmInfo()
    rc = lib().gemm_sm100a_query(C.byref(args), C.byref(info))
    return rc, info


def launch(args: GemmArgs, stream: int = 0) -> None:
    """Enqueue one GEMM (one kernel launch) on `stream` (a cudaStream_t as int)."""
    rc = lib().gemm_sm100a_launch(C.byref(args), C.c_void_p(stream))
    if rc != OK:
        _, info = query(args)
        raise GemmError(rc, f"gemm_sm100a_launch ({info.reason.decode()})")


def launch_gather(args: GemmArgs, peer_d: list[int], stream: int = 0) -> None:
    """One GEMM whose epilogue also writes its D block into each buffer of
    `peer_d` (device addresses, at most 7; e.g. the same block of the full D on
    the other GPUs of an N-split), fusing the all-gather into the launch."""
    arr = (C.c_void_p * max(1, len(peer_d)))(*peer_d)
    rc = lib().gemm_sm100a_launch_gather(C.byref(args), arr, len(peer_d), C.c_void_p(stream))
    if rc != OK:
        _, info = query(args)
        raise GemmError(rc, f"gemm_sm100a_launch_gather ({info.reason.decode() or 'peer pointers'})")


def read_status(status_ptr: int, stream: int = 0) -> tuple[int, int]:
    detail = C.c_int32(0)
    rc = lib().gemm_sm100a_read_status(C.c_void_p(status_ptr), C.c_void_p(stream), C.byref(detail))
    return rc, detail.value


def generate(out_ptr: int, dtype: int, dist: int, scale: float, seed: int, stream_id: int,
             row0: int, rows: int, cols: int, ld: int | None = None, cuda_stream: int = 0) -> None:
    rc = lib().gemm_sm100a_generate(C.c_void_p(out_ptr), dtype, dist, scale, seed, stream_id,
                                    row0, rows, cols, cols if ld is None else ld, C.c_void_p(cuda_stream))
    if rc != OK:
        raise GemmError(rc, "gemm_sm100a_generate")


def generate_nvfp4(packed_ptr: int, scales_ptr: int, scale: float, seed: int, stream_id: int,
                   row0: int, rows: int, cols: int, cuda_stream: int = 0) -> None:
    rc = lib().gemm_sm100a_generate_nvfp4(C.c_void_p(packed_ptr), C.c_void_p(scales_ptr), scale, seed,
                                          stream_id, row0, rows, cols, C.c_void_p(cuda_stream))
    if rc != OK:
        raise GemmError(rc, "gemm_sm100a_generate_nvfp4")


K_ELEMS_PER_MMA = {BF16: 16, FP8_E4M3: 32, NVFP4: 64}


def umma_peak(dtype: int, cta_group: int = 1, num_ctas: int = 1, depth: int = 256, iters: int = 200,
              device=None) -> dict:
    """Run the tcgen05 peak probe and summarise it.

    flop_per_clk_per_sm: median over issuing CTAs of FLOPs / clock64 cycles, per SM
    (a CTA pair counts as two SMs); sm_mhz: median cycles / ns; tflops: total FLOPs of
    all issuing CTAs / the longest CTA time (the whole-GPU dense peak when num_ctas
    covers every SM)."""
    import statistics
    import torch
    dev = torch.device("cuda" if device is None else device)
    res = torch.zeros(3 * num_ctas, dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    rc = lib().gemm_sm100a_umma_peak(dtype, cta_group, num_ctas, depth, iters, C.c_void_p(res.data_ptr()),
                                     C.c_void_p(st))
    if rc != OK:
        raise GemmError(rc, "gemm_sm100a_umma_peak")
    torch.cuda.synchronize(dev)
    r = res.view(num_ctas, 3).cpu().tolist()
    leaders = [x for x in r if x[0] > 0]
    if any(x[2] for x in r):
        raise GemmError(ERR_TIMEOUT, "umma_peak wait")
    flop_per_mma = 2.0 * 128 * cta_group * 256 * K_ELEMS_PER_MMA[dtype]
    total = flop_per_mma * depth * iters
    fpc = [total / x[0] / cta_group for x in leaders]
    mhz = [x[0] / x[1] * 1e3 for x in leaders]
    return {"dtype": DTYPE_NAMES[dtype], "cta_group": cta_group, "num_ctas": num_ctas, "depth": depth,
            "iters": iters, "flop_per_clk_per_sm": statistics.median(fpc), "sm_mhz": statistics.median(mhz),
            "tflops": total * len(leaders) / (max(x[1] for x in leaders) * 1e-9) / 1e12}


L2_FLUSH_BYTES = 256 << 20     # twice the B200's 126 MB L2


def tma_read_probe(buf, box_rows: int, stages: int, ctas_per_sm: int = 1, box_width: int = 128,
                   flush=None, device=None) -> dict:
    """Run the TMA-2D read probe over the device tensor `buf` once (L2 flushed first by
    writing `flush`, a device buffer larger than L2) and summarise it: bytes / event time,
    per-CTA cycles, tiles and cycles per TMA load -- the columns of the reference's
    tma2d_throughput results (tma2d_tput_results.csv)."""
    import statistics
    import torch
    dev = buf.device if device is None else torch.device(device)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    grid = sms * ctas_per_sm
    res = torch.zeros(5 * grid, dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream(dev)
    if flush is not None:
        flush.fill_(0xA5)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nbytes = buf.numel() * buf.element_size()
    e0.record(st)
    rc = lib().gemm_sm100a_tma_read_probe(C.c_void_p(buf.data_ptr()), nbytes, box_width, box_rows, stages,
                                          ctas_per_sm, C.c_void_p(res.data_ptr()), C.c_void_p(st.cuda_stream))
    e1.record(st)
    if rc != OK:
        raise GemmError(rc, "gemm_sm100a_tma_read_probe")
    e1.synchronize()
    r = res.view(grid, 5).cpu().tolist()
    if any(x[4] for x in r):
        raise GemmError(ERR_TIMEOUT, "tma_read_probe wait")
    tile_bytes = 4 * box_width * box_rows
    tiles = sum(x[2] for x in r)
    ms = e0.elapsed_time(e1)
    busy = [x for x in r if x[2] > 0]
    cyc = statistics.mean(x[0] for x in busy)
    return {"ctas_per_sm": ctas_per_sm, "stages": stages, "box_width": box_width, "box_rows": box_rows,
            "bytes_in_flight_per_sm": ctas_per_sm * stages * tile_bytes, "bytes": tiles * tile_bytes,
            "ms": ms, "GBps": tiles * tile_bytes / (ms * 1e-3) / 1e9, "sm_cycles_avg": cyc,
            "tma_ops_avg": statistics.mean(x[2] for x in busy), "cycles_per_tma": statistics.mean(x[0] / x[2] for x in busy),
            # from the CTAs' own counters (no launch overhead): bytes per SM clock, and the
            # aggregate rate over the median CTA duration
            "bytes_per_clk_per_cta": statistics.median(x[2] * tile_bytes / x[0] for x in busy),
            "sm_mhz": statistics.median(x[0] / x[1] * 1e3 for x in busy if x[1] > 0),
            "GBps_in_kernel": tiles * tile_bytes / statistics.median(x[1] for x in busy),
            "checksums": [x[3] for x in r], "tiles_per_cta": [x[2] for x in r]}


def sf_bytes(rows: int, cols: int) -> int:
    """Size of an interleaved NVFP4 scale buffer (rows padded to 128, one byte per 16 columns)."""
    return ((rows + 127) // 128) * (cols // 64) * 512


from .torch_api import Operands, make_operands, gemm, gemm_into, flops  # noqa: E402,F401
