// tma_probe.cu -- TMA-2D HBM read-throughput probe for B200 (sm_100a).
//
// Replaces the reference's tma2d_throughput/tma2d_tput.cu (kernel :42-126,
// launch :131-219): CTAs of one warp stream a large 2-D tensor of 32-bit
// words through a STAGES-deep shared-memory ring with cp.async.bulk.tensor.2d
// loads of (box_rows x box_width) boxes, refilling each slot as soon as its
// load has landed.  It measures the memory roof that bounds small and skinny
// GEMMs, where the tensor-core roof does not apply.
//
// Differences from the reference, by design: the shape is a runtime argument
// (no recompilation per point), every mbarrier wait is bounded (status word on
// expiry, then a bounded drain of loads in flight), and each CTA records its
// cycles, nanoseconds, tiles and an XOR checksum of the first 128 bytes of
// every tile, so the host can check that the data actually landed and compute
// bandwidth from CUDA events instead of profiler counters.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "gemm_sm100a.h"
#define GEMM_TMA_CACHE_HINT 0   // plain loads, no L2 policy (as the reference's probe)
#include "sm100_ptx.cuh"
#include "device_guard.cuh"

using namespace sm100;

namespace {

constexpr int kProbeSmem = 232448;         // pinned at the 227 KiB maximum, as the reference does (:200-205)
constexpr int kProbeMaxStages = 64;

struct ProbeParams {
  int64_t tiles_total;      // box_rows-row tiles in the tensor
  int32_t box_rows;
  int32_t stages;
  uint32_t tile_bytes;
  uint64_t timeout_ns;
  unsigned long long* results;   // per CTA: cycles, ns, tiles, checksum, status
};

__global__ void __launch_bounds__(32, 1)
tma_read_probe_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ ProbeParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + (uint32_t)p.stages * p.tile_bytes;
  const uint32_t lane = threadIdx.x & 31u;
  if (lane == 0) {
    prefetch_tmap(&tm);
    for (int s = 0; s < p.stages; ++s) mbar_init(bars + 8u * s, 1);
    fence_mbar_init();
  }
  __syncwarp();
  const uint32_t issue = elect_one() ? 1u : 0u;
  const unsigned long long c0 = clock64(), t0 = globaltimer_ns();

  // This CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int64_t first = blockIdx.x, stride = gridDim.x;
  const int64_t n = first < p.tiles_total ? (p.tiles_total - first + stride - 1) / stride : 0;
  auto issue_tile = [&](int64_t i) {
    const uint32_t slot = (uint32_t)(i % p.stages);
    const uint32_t bar = bars + 8u * slot;
    mbar_arrive_expect_tx(bar, p.tile_bytes, issue);
    const int32_t y = (int32_t)((first + i * stride) * p.box_rows);
    tma_load_2d(base + slot * p.tile_bytes, &tm, bar, 0, y, 0ull, issue);
  };
  for (int64_t i = 0; i < n && i < p.stages; ++i) issue_tile(i);

  uint32_t checksum = 0, status = 0;
  int64_t done = 0;
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t slot = (uint32_t)(i % p.stages);
    const uint32_t bar = bars + 8u * slot;
    const uint32_t parity = (uint32_t)((i / p.stages) & 1);
    bool ok = mbar_test_wait(bar, parity);
    if (!ok) {
      const uint64_t w0 = globaltimer_ns();
      while (!(ok = mbar_try_wait_hint(bar, parity, 100000u))) {
        if (globaltimer_ns() - w0 > p.timeout_ns) break;
      }
    }
    if (!__all_sync(0xffffffffu, ok)) { status = 3u; break; }
    checksum ^= ld_shared_volatile_u32(base + slot * p.tile_bytes + 4u * lane);
    fence_proxy_async_shared();      // the reads above come before the next load into this slot
    __syncwarp();
    ++done;
    if (i + p.stages < n) issue_tile(i + p.stages);
  }
  if (status) {
    // Let every load still in flight land (bounded) before the CTA exits.
    for (int64_t i = done; i < n && i < done + p.stages; ++i) {
      const uint32_t slot = (uint32_t)(i % p.stages);
      const uint64_t w0 = globaltimer_ns();
      while (!mbar_try_wait(bars + 8u * slot, (uint32_t)((i / p.stages) & 1)))
        if (globaltimer_ns() - w0 > 100000000ull) break;
    }
  }
  for (int off = 16; off > 0; off >>= 1) checksum ^= __shfl_xor_sync(0xffffffffu, checksum, off);
  if (lane == 0) {
    unsigned long long* r = p.results + 5ull * blockIdx.x;
    r[0] = clock64() - c0;
    r[1] = globaltimer_ns() - t0;
    r[2] = (unsigned long long)done;
    r[3] = checksum;
    r[4] = status;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_probe_encode = nullptr;
std::once_flag g_probe_encode_once;

}  // namespace

extern "C" int gemm_sm100a_tma_read_probe(const void* buf, int64_t bytes, int32_t box_width, int32_t box_rows,
                                          int32_t stages, int32_t ctas_per_sm, unsigned long long* results,
                                          void* stream) {
  if (!buf || !results || bytes <= 0) return GEMM_ERR_BAD_ARGS;
  if (box_width < 4 || box_width > 256 || box_width % 4 || box_rows < 1 || box_rows > 256) return GEMM_ERR_BAD_ARGS;
  if (stages < 1 || stages > kProbeMaxStages || ctas_per_sm < 1 || ctas_per_sm > 32) return GEMM_ERR_BAD_ARGS;
  if (reinterpret_cast<uintptr_t>(buf) & 15) return GEMM_ERR_BAD_ARGS;
  const uint32_t tile_bytes = (uint32_t)box_width * (uint32_t)box_rows * 4u;
  if (tile_bytes < 128) return GEMM_ERR_BAD_ARGS;   // the checksum reads each tile's first 128 bytes
  if ((int64_t)stages * tile_bytes + 1024 + 8 * kProbeMaxStages > kProbeSmem) return GEMM_ERR_CANNOT_IMPLEMENT;
  const int64_t rows = bytes / (4 * (int64_t)box_width);
  const int64_t tiles = rows / box_rows;
  if (tiles < 1 || rows > INT32_MAX) return GEMM_ERR_CANNOT_IMPLEMENT;

  StreamDeviceGuard guard(reinterpret_cast<cudaStream_t>(stream));
  if (!guard.ok) return GEMM_ERR_LAUNCH;
  std::call_once(g_probe_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_probe_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_probe_encode) return GEMM_ERR_LAUNCH;
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)box_width, (cuuint64_t)(tiles * box_rows)};
  cuuint64_t strides[1] = {(cuuint64_t)box_width * 4u};
  cuuint32_t box[2] = {(cuuint32_t)box_width, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  if (g_probe_encode(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(buf), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return GEMM_ERR_CANNOT_IMPLEMENT;

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  ProbeParams p;
  memset(&p, 0, sizeof(p));
  p.tiles_total = tiles;
  p.box_rows = box_rows;
  p.stages = stages;
  p.tile_bytes = tile_bytes;
  p.timeout_ns = 2000000000ull;
  p.results = results;
  if (cudaFuncSetAttribute(tma_read_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem) !=
      cudaSuccess) {
    cudaGetLastError();
    return GEMM_ERR_LAUNCH;
  }
  tma_read_probe_kernel<<<sms * ctas_per_sm, 32, kProbeSmem, reinterpret_cast<cudaStream_t>(stream)>>>(tm, p);
  if (cudaGetLastError() != cudaSuccess) return GEMM_ERR_LAUNCH;
  return GEMM_OK;
}
