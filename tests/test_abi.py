"""CPU tests of the C ABI (no kernel launches): the library loads, exports
every symbol include/gemm_sm100a.h declares, and resolves / rejects knobs the
way the reference's can_implement does (cutlass_gemm_bench.cu:211-218)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_functions():
    text = (ROOT / "include" / "gemm_sm100a.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(gemm_sm100a_\w+)\s*\(", text, re.M)))


def test_header_lists_the_exported_api(pkg):
    assert set(header_functions()) == set(pkg.EXPORTED)


def test_library_exports_every_declared_symbol(pkg):
    L = C.CDLL(str(pkg.LIB_PATH))
    for name in header_functions():
        assert hasattr(L, name), name


def test_version_and_strerror(pkg):
    assert pkg.lib().gemm_sm100a_version() >= 100
    assert "cannot implement" in pkg.strerror(pkg.ERR_CANNOT_IMPLEMENT)
    assert "timed out" in pkg.strerror(pkg.ERR_TIMEOUT)


def _args(pkg, **kw):
    base = dict(dtype=pkg.BF16, m=8192, n=8192, k=8192, a=0x1000, b=0x2000, d=0x3000)
    base.update(kw)
    return pkg.make_args(**base)


def test_struct_size_guard(pkg):
    a = _args(pkg)
    rc, _ = pkg.query(a)
    assert rc == pkg.OK
    a.struct_size = 8
    rc, info = pkg.query(a)
    assert rc == pkg.ERR_BAD_ARGS and b"struct_size" in info.reason


def test_reference_defaults_and_smem_per_stage(pkg):
    rc, info = pkg.query(_args(pkg, tile_n=256, tile_k=64))
    assert rc == pkg.OK and info.can_implement
    assert info.tile_m == 128 and info.tile_n == 256 and info.tile_k == 64
    assert info.smem_bytes_per_stage == (128 + 256) * 64 * 2          # 48 KiB, as in the reference
    assert info.max_stages == 4 and info.stages == 4                  # auto = as many as fit
    assert info.tmem_columns == 512
    assert info.num_tiles == 64 * 32


@pytest.mark.parametrize("stages,ok", [(2, True), (3, True), (4, True), (5, False), (8, False)])
def test_stage_limit_mirrors_reference_build_failures(pkg, stages, ok):
    """128x256x64 bf16: the reference's S=5..8 rows are BUILD_FAILED (results.csv:462-465)."""
    rc, info = pkg.query(_args(pkg, tile_n=256, tile_k=64, stages=stages))
    assert (rc == pkg.OK) == ok
    if not ok:
        assert b"shared memory" in info.reason


def test_fp8_tile_defaults(pkg):
    rc, info = pkg.query(_args(pkg, dtype=pkg.FP8_E4M3, tile_n=256, tile_k=128))
    assert rc == pkg.OK and info.smem_bytes_per_stage == (128 + 256) * 128 and info.max_stages == 4


def test_pair_mode_resolution(pkg):
    rc, info = pkg.query(_args(pkg, dtype=pkg.FP8_E4M3, m=16384, n=16384, k=16384,
                               cta_group=2, tile_n=256, tile_k=128))
    assert rc == pkg.OK
    assert info.tile_m == 256 and info.cta_group == 2
    assert info.smem_bytes_per_stage == (128 + 128) * 128     # each CTA holds half of B
    assert info.grid_ctas % 2 == 0
    assert info.num_tiles == 64 * 64


@pytest.mark.parametrize("kw,frag", [
    (dict(tile_n=48), b"tile_n"),
    (dict(tile_k=48), b"tile_k"),
    (dict(tile_k=96), b"tile_k"),
    (dict(cta_group=3), b"cta_group"),
    (dict(lda=8191), b"lda"),
    (dict(k=4, lda=8192, ldb=8192), b"k must"),
    (dict(a=0x1001), b"aligned"),
    (dict(ldd=100, m=101), b"ldd"),
])
def test_cannot_implement_reasons(pkg, kw, frag):
    rc, info = pkg.query(_args(pkg, **kw))
    assert rc in (pkg.ERR_CANNOT_IMPLEMENT, pkg.ERR_BAD_ARGS)
    assert frag in info.reason, info.reason


@pytest.mark.parametrize("dtype,tile_k,row_bytes", [("bf16", 16, 32), ("bf16", 32, 64),
                                                    ("fp8", 32, 32), ("fp8", 64, 64)])
def test_narrow_tile_k_uses_narrow_swizzle(pkg, dtype, tile_k, row_bytes):
    """TILE_K below one 128-byte row (the reference sweeps bf16 16/32 and fp8
    32/64) is one 64- or 32-byte swizzle atom per stage."""
    dt = pkg.BF16 if dtype == "bf16" else pkg.FP8_E4M3
    rc, info = pkg.query(_args(pkg, dtype=dt, tile_n=256, tile_k=tile_k))
    assert rc == pkg.OK, info.reason
    assert info.tile_k == tile_k
    assert info.smem_bytes_per_stage == (128 + 256) * row_bytes


@pytest.mark.parametrize("dtype,tile_k", [("bf16", 64), ("fp8", 128), ("bf16", 16)])
def test_tile_m_64_is_a_1sm_tile(pkg, dtype, tile_k):
    """TILE_M = 64 (the reference sweeps 64 and 128) is an M = 64 MMA on one SM."""
    dt = pkg.BF16 if dtype == "bf16" else pkg.FP8_E4M3
    rc, info = pkg.query(_args(pkg, dtype=dt, tile_m=64, tile_n=128, tile_k=tile_k))
    assert rc == pkg.OK, info.reason
    assert info.tile_m == 64 and info.cta_group == 1
    row_bytes = min(128, tile_k * (2 if dtype == "bf16" else 1))
    assert info.smem_bytes_per_stage == (64 + 128) * row_bytes * max(1, tile_k * (2 if dtype == "bf16" else 1) // 128)
    assert info.num_tiles == (8192 // 64) * (8192 // 128)
    rc, info = pkg.query(_args(pkg, dtype=dt, tile_m=64, cta_group=2, tile_n=256, tile_k=tile_k))
    assert rc == pkg.ERR_CANNOT_IMPLEMENT and b"tile_m" in info.reason


def test_nvfp4_pair_query(pkg):
    """NVFP4 cta_group::2: 256 x tile_n tiles; each CTA stages its 128 rows of
    A scales and the whole tile's B scales; one accumulator at tile_n 256."""
    args = _args(pkg, dtype=pkg.NVFP4, cta_group=2, tile_n=256, tile_k=256, sfa=0x40000, sfb=0x50000)
    rc, info = pkg.query(args)
    assert rc == pkg.OK, info.reason
    assert info.tile_m == 256 and info.cta_group == 2
    # per CTA: A 128 rows + B 128 rows of 128 B, SFA 4 atoms, SFB 4 atoms x 2 row blocks
    assert info.smem_bytes_per_stage == (128 + 128) * 128 + 4 * 512 * (1 + 2)
    rc, info = pkg.query(_args(pkg, dtype=pkg.NVFP4, cta_group=2, tile_n=256, tile_k=256, m=8192 - 128,
                               sfa=0x40000, sfb=0x50000))
    assert rc == pkg.ERR_CANNOT_IMPLEMENT and b"m %" in info.reason


def test_null_pointers_are_bad_args(pkg):
    rc, _ = pkg.query(_args(pkg, a=None))
    assert rc == pkg.ERR_BAD_ARGS
    rc, _ = pkg.query(_args(pkg, dtype=pkg.NVFP4, k=8192))
    assert rc == pkg.ERR_BAD_ARGS          # NVFP4 without scale factors


def test_single_cta_reference_mode(pkg):
    """max_ctas=1 reproduces the reference's 1-CTA grid (cutlass_gemm_bench.cu:190)."""
    rc, info = pkg.query(_args(pkg, m=128, n=256, k=131072, tile_n=256, max_ctas=1))
    assert rc == pkg.OK and info.grid_ctas == 1 and info.num_tiles == 1


def test_launch_rejects_before_touching_the_gpu(pkg):
    with pytest.raises(pkg.GemmError) as e:
        pkg.launch(_args(pkg, stages=7, tile_n=256))
    assert e.value.code == pkg.ERR_CANNOT_IMPLEMENT


def test_gather_rejects_bad_destination_lists_before_any_cuda_call(pkg):
    """gemm_sm100a_launch_gather: at most 7 extra destinations, and a list when any."""
    import ctypes as C
    L = pkg.lib()
    args = _args(pkg)
    arr = (C.c_void_p * 8)(*([0x10000] * 8))
    assert L.gemm_sm100a_launch_gather(C.byref(args), arr, 8, None) == pkg.ERR_BAD_ARGS
    assert L.gemm_sm100a_launch_gather(C.byref(args), None, 1, None) == pkg.ERR_BAD_ARGS
    assert L.gemm_sm100a_launch_gather(C.byref(args), arr, -1, None) == pkg.ERR_BAD_ARGS


def test_epilogue_staging_buffers(pkg):
    """The TMA-store epilogue stages D in shared memory when it fits next to the
    ring (the stage count, and so can_implement, never depends on it)."""
    cases = [(dict(tile_n=256, tile_k=64, stages=4), 2),                       # bf16 128x256x64 S4
             (dict(tile_n=512, tile_k=64, cta_group=2), 1),                    # pair 256x512, four groups
             (dict(tile_n=128, tile_k=64), 0),                                 # 7 stages fill shared memory
             (dict(tile_n=256, tile_k=64, stages=4, flags=pkg.FLAG_DIRECT_EPILOGUE), 0)]
    for knobs, bufs in cases:
        rc, info = pkg.query(_args(pkg, **knobs))
        assert rc == pkg.OK and info.epilogue_staging_buffers == bufs, (knobs, info.epilogue_staging_buffers)
        assert info.smem_bytes <= 232448
    rc, info = pkg.query(_args(pkg, tile_n=128, tile_k=64))
    assert info.stages == 7                                                     # as the reference's auto count
    rc, info = pkg.query(_args(pkg, dtype=pkg.NVFP4, sfa=0x4000, sfb=0x5000, tile_n=256, tile_k=256))
    assert rc == pkg.OK and info.stages == 4 and info.epilogue_staging_buffers == 1


def test_epilogue_argument_checks(pkg):
    rc, info = pkg.query(_args(pkg, beta=1.0))                                  # beta without C
    assert rc == pkg.ERR_BAD_ARGS and b"needs C" in info.reason
    rc, _ = pkg.query(_args(pkg, beta=1.0, c=0x6000))
    assert rc == pkg.OK
    rc, info = pkg.query(_args(pkg, beta=1.0, c=0x6008))                        # misaligned C
    assert rc == pkg.ERR_CANNOT_IMPLEMENT
    rc, info = pkg.query(_args(pkg, d_layout=2))
    assert rc == pkg.ERR_CANNOT_IMPLEMENT and b"d_layout" in info.reason
    rc, _ = pkg.query(_args(pkg, m=8192, n=1000, d_layout=pkg.ROW_MAJOR))       # ldd = n = 1000
    assert rc == pkg.OK
    rc, info = pkg.query(_args(pkg, m=1000, n=8192, d_layout=pkg.ROW_MAJOR, ldd=1000))   # ldd < n
    assert rc == pkg.ERR_CANNOT_IMPLEMENT
