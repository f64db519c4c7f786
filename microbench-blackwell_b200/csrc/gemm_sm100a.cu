// gemm_sm100a.cu -- persistent warp-specialised dense GEMM for B200 (sm_100a).
//
// Replaces the CUTLASS SM100 GEMM instantiated by the reference benchmark
// (cutlass_gemm_mainloop/cutlass_gemm_bench.cu:101-156: CollectiveBuilder with
// KernelTmaWarpSpecialized1SmSm100 mainloop + NoSmemWarpSpecialized1Sm
// epilogue) with a hand-written kernel of the same math
//     D(bf16, column-major) = alpha * A(row-major) . B(N x K)^T, fp32 accumulate
// for bf16, fp8 e4m3 and NVFP4 (e2m1 + ue4m3 per-16 scales) operands, in
// 1-SM (cta_group::1, 128 x BN) and 2-SM (cta_group::2, 256 x BN per CTA pair)
// forms.
//
// One CTA per SM (persistent over output tiles), 192 threads (320 when the
// tile fills TMEM):
//   warp 0      TMA producer: 128B-swizzled A/B k-atoms into a STAGES-deep
//               shared-memory ring, guarded by full/empty mbarriers (a TILE_K
//               narrower than 128 bytes is one 64B- or 32B-swizzled atom).
//   warp 1      TMEM allocator + tcgen05.mma issuer; commits free ring slots
//               and hands finished accumulators to the epilogue.
//   warps 2..   epilogue (4, or 8): tcgen05.ld of the fp32 accumulator (one
//               TMEM lane quadrant each), alpha scale, bf16 round, column-major
//               stores.
// Warps 0 and 1 run their loops converged, so addresses and descriptors are
// warp-uniform; TMA, mbarrier and tcgen05 issue is predicated on one elected
// lane (in CTA-pair kernels that lane issues inside a branch instead); the
// loops are instantiated per stage shape (atoms x MMA K steps).  The accumulator is double-buffered in TMEM (2 x BN columns) when it
// fits, so the epilogue of tile i overlaps the mainloop of tile i+1; a single
// accumulator is drained into registers and released before D is written.
//
// Every mbarrier wait is bounded (globaltimer budget): on expiry the kernel
// records a status word, tells the other roles to stop, drains its own
// in-flight copies / MMAs with a bounded wait, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "gemm_sm100a.h"
#include "sm100_ptx.cuh"
#include "device_guard.cuh"

using namespace sm100;

// Tuning switches (compile time).
#ifndef GEMM_L2_PROMOTION
#define GEMM_L2_PROMOTION CU_TENSOR_MAP_L2_PROMOTION_L2_256B
#endif
#ifndef GEMM_TMA_CACHE_HINT
#define GEMM_TMA_CACHE_HINT 1   // 1: loads carry an L2 evict_normal policy; 0: no hint
#endif
#ifndef GEMM_TRACE
#define GEMM_TRACE 0            // 1: log CTA 0's pipeline events (trace builds only)
#endif
#ifndef GEMM_WIDE_EPI_WARPS
#define GEMM_WIDE_EPI_WARPS 16  // epilogue warps of a 512-column tile (8 or 16)
#endif
#ifndef GEMM_WIDE_EARLY_RELEASE
#define GEMM_WIDE_EARLY_RELEASE 0  // 1: a 512-column accumulator is drained into registers and released
                                   //    before D is written; 0: written chunk by chunk, released after the last read
#endif

#if GEMM_TRACE
// Pipeline event log of CTA 0 (trace builds only).  Each role writes its own
// region with plain stores (no atomics on the critical path); entry =
// clock64 << 16 | role << 12 | kind << 8 | stage.
constexpr unsigned kTraceRegion = 1u << 14;
__device__ unsigned long long g_trace_log[4 * kTraceRegion];
#define TRACE_EVENT(role, kind, stage)                                                     \
  do {                                                                                     \
    if (blockIdx.x == 0 && (threadIdx.x & 31u) == 0 && trace_i < kTraceRegion)            \
      g_trace_log[(role) * kTraceRegion + trace_i++] =                                     \
          ((unsigned long long)clock64() << 16) | ((role) << 12) | ((kind) << 8) | ((stage) & 0xFF); \
  } while (0)
#else
#define TRACE_EVENT(role, kind, stage) do { } while (0)
#endif

namespace {

template <int V>
struct IntC { static constexpr int value = V; };

// Threads per CTA: producer warp + MMA warp + EPI_WARPS epilogue warps.
// Epilogue warps: 4 (one per TMEM lane quadrant), or GEMM_WIDE_EPI_WARPS for a
// 512-column tile (one accumulator filling TMEM): 16 warps read it in four
// column groups, which shortens the time the MMA warp waits for it.
__host__ __device__ constexpr int epi_warps_for(int bn) { return bn > 256 ? GEMM_WIDE_EPI_WARPS : 4; }
__host__ __device__ constexpr int threads_for(int bn) { return 64 + 32 * epi_warps_for(bn); }
constexpr int kSmemLimit = 232448;      // 227 KiB of opt-in dynamic shared memory per CTA
constexpr int kBarrierBytes = 1024;     // barrier block + bookkeeping words
constexpr int kMaxStages = 32;
constexpr int kMaxGatherPeers = 7;   // peer D destinations of the fused gather (8 GPUs per box)
constexpr int kDefaultL2Prefetch = 0;         // k-blocks of L2 prefetch ahead of the ring (0 = off)
constexpr int kMinSmemPerCta = 120 * 1024;  // > half of the SM's 228 KiB: at most one CTA per SM
#ifndef GEMM_ACC_OVERLAP
#define GEMM_ACC_OVERLAP 64     // overlapped accumulator positions for 256-wide NVFP4 tiles (columns; 0 = off)
#endif
constexpr int kAccOverlap = GEMM_ACC_OVERLAP;

enum Role : uint32_t { ROLE_PRODUCER = 1, ROLE_MMA = 2, ROLE_EPILOGUE = 3, ROLE_DRAIN = 4 };

struct KernelParams {
  int32_t m, n, k;
  int32_t num_m_units, num_n_units, num_units;
  int32_t num_k_blocks;
  int32_t atoms;          // 128-byte K atoms per stage
  int32_t stages;
  int32_t raster_group;
  int32_t tmem_cols;
  uint32_t stage_bytes;   // per CTA: A + B (+ scale factors)
  uint32_t a_atom_bytes, b_atom_bytes;
  uint32_t row_bytes;     // bytes of one operand row in a K atom: 128, 64 or 32 (the swizzle width)
  int32_t cta_rows;       // A rows (accumulator rows) per CTA: 128, or 64 for a 1-SM TILE_M = 64
  uint32_t sf_stage_bytes;  // NVFP4: SFA + SFB bytes per stage per CTA
  uint32_t idesc;
  float alpha;
  __nv_bfloat16* d;
  int64_t ldd;
  int32_t* status;
  uint64_t timeout_ns;
  uint32_t flags;
  const uint8_t* sfa;
  const uint8_t* sfb;
  int32_t sf_kblocks;     // K / 64 (NVFP4 scale atoms along K)
  int32_t sf_slots;       // NVFP4: TMEM scale-factor slots (stage s uses slot s % sf_slots)
  // Fused gather: the epilogue also writes every D element to these buffers
  // (other GPUs' D, reached over NVLink), at the same row/column offsets and ldd.
  int32_t n_d_peer;
  __nv_bfloat16* d_peer[kMaxGatherPeers];
  int32_t l2_prefetch;    // k-blocks the L2 prefetch cursor runs ahead of the loads (0 = off)
  unsigned long long* clock_out;   // optional: [cycles, ns] summed over the launch's CTAs
  int32_t num_acc;        // accumulator buffers in TMEM (2 = epilogue overlaps the next tile)
  int32_t acc_overlap;    // > 0: one accumulator barrier, two positions (0 and BN - acc_overlap)
                          // alternating per tile; the epilogue frees the shared columns first
  float beta;             // D = alpha * acc + beta * C (C read only when beta != 0)
  const __nv_bfloat16* c; // C, same layout as D, leading dimension ldc
  int64_t ldc;
  int32_t d_row_major;    // 0: D (and C) column-major (M contiguous), 1: row-major (N contiguous)
  int32_t stg_bufs;       // staging buffers per epilogue group (0 = direct stores from registers)
  uint32_t stg_offset;    // shared-memory offset of the staging area from the aligned base
  uint32_t stg_bytes;     // bytes of one staging buffer (BM rows x CW columns of bf16)
};

// Elements of each dtype in one 128-byte swizzle atom row.
__host__ __device__ constexpr int atom_elems(int dt) { return dt == 0 ? 64 : (dt == 1 ? 128 : 256); }

// tcgen05 instruction descriptor.
//  dense (kind::f16 / kind::f8f6f4): [4,6) D format (1 = F32), [7,10) A format,
//    [10,13) B format (BF16 = 1 for kind::f16, E4M3 = 0 for kind::f8f6f4),
//    [15] / [16] A / B major (0 = K), [17,23) N >> 3, [24,29) M >> 4.
//  block-scaled (kind::mxf4nvf4): [4,6) B scale id, [7,10) A format (E2M1 = 1),
//    [10,12) B format, [17,23) N >> 3, [23] scale type (0 = UE4M3),
//    [24,29) M >> 4, [29,31) A scale id, [31] K = 64.
__host__ __device__ constexpr uint32_t make_idesc(int dt, int mma_m, int mma_n) {
  uint32_t d = 0;
  if (dt == 2) {
    d |= 1u << 7;
    d |= 1u << 10;
    d |= (uint32_t)(mma_n >> 3) << 17;
    d |= (uint32_t)(mma_m >> 4) << 24;
  } else {
    const uint32_t fmt = dt == 0 ? 1u : 0u;
    d |= 1u << 4;
    d |= fmt << 7;
    d |= fmt << 10;
    d |= (uint32_t)(mma_n >> 3) << 17;
    d |= (uint32_t)(mma_m >> 4) << 24;
  }
  return d;
}

struct SharedCtl {
  uint32_t abort_addr;     // local abort flag (shared::cta address)
  uint32_t abort_peer;     // the pair peer's abort flag (shared::cluster), 0 if none
  uint64_t timeout_ns;
  int32_t* status;
};

__device__ __noinline__ void raise_abort(const SharedCtl& c, uint32_t role, uint32_t idx) {
  if (c.status) {
    const int32_t code = (int32_t)(0x3u | (role << 8) | ((idx & 0xFFu) << 12) | ((blockIdx.x & 0x7FFu) << 20));
    atomicCAS(c.status, 0, code);
  }
  st_shared_u32(c.abort_addr, 1u);
  if (c.abort_peer) st_shared_cluster_u32(c.abort_peer, 1u);
}

// Bounded wait for phase `parity` of mbarrier `bar`; false when aborted.
// The probes are plain try_wait (no suspend-time hint: resuming a suspended
// thread added latency to every pipeline round trip); the abort flag is
// checked after every probe and the timer every 8 probes.
template <bool kCluster>
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const SharedCtl& c,
                                         uint32_t role, uint32_t idx) {
  if (kCluster ? mbar_test_wait_cluster(bar, parity) : mbar_test_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t probe = 1;; ++probe) {
    if (kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity))
      return true;
    if (ld_shared_volatile_u32(c.abort_addr)) return false;
    if ((probe & 7u) == 1u) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > c.timeout_ns) {
        raise_abort(c, role, idx);
        return false;
      }
    }
  }
}

// Wait with a short fixed budget during abort drains; never raises.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t budget_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > budget_ns) break;
  }
}

// Output-tile rasterisation.  raster_group G > 0: groups of G M-tiles, M
// fastest inside a group (tiles sharing B run together); G < 0: groups of |G|
// N-tiles, N fastest (tiles sharing A run together).
__device__ __forceinline__ void unit_coords(int u, const KernelParams& p, int& um, int& un) {
  if (p.raster_group > 0) {
    const int G = p.raster_group;
    const int per_group = G * p.num_n_units;
    const int g = u / per_group;
    const int first_m = g * G;
    const int rows = min(p.num_m_units - first_m, G);
    const int r = u - g * per_group;
    um = first_m + r % rows;
    un = r / rows;
  } else {
    const int G = -p.raster_group;
    const int per_group = G * p.num_m_units;
    const int g = u / per_group;
    const int first_n = g * G;
    const int cols = min(p.num_n_units - first_n, G);
    const int r = u - g * per_group;
    un = first_n + r % cols;
    um = r / cols;
  }
}

// ----------------------------------------------------------------------------
// The kernel.  DT: 0 bf16, 1 e4m3, 2 NVFP4.  CG: 1 or 2 (CTA pair).  BN: MMA N
// (the pair's full N for CG = 2; each CTA of the pair loads BN / 2 rows of B).
// ----------------------------------------------------------------------------
template <int DT, int CG, int BN>
__global__ void __launch_bounds__(threads_for(BN), 1)
gemm_sm100a_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_sfa,   // NVFP4 pair kernel only
                   const __grid_constant__ CUtensorMap tmap_sfb,   // NVFP4 pair kernel only
                   const __grid_constant__ CUtensorMap tmap_d,     // D, for the staged epilogue's TMA stores
                   const __grid_constant__ KernelParams p) {
  // A rows per CTA.  128 fills the 128 TMEM lanes; a 1-SM TILE_M = 64 tile
  // (M = 64 MMA) puts row r of the accumulator in lane 32*(r/16) + r%16, i.e.
  // the first 16 lanes of each 32-lane quadrant.
  const int BM = CG == 2 ? 128 : p.cta_rows;
  constexpr int MMA_N = BN > 256 ? 256 : BN;  // N of one tcgen05.mma
  constexpr int N_SUB = BN / MMA_N;       // MMAs per K step (N halves of a 512-wide pair tile)
  constexpr int B_BOX = MMA_N / CG;       // B rows per CTA per N half (one TMA box)
  constexpr int EPI_WARPS = epi_warps_for(BN);
  const int MMA_M = BM * CG;
  constexpr int KIND = DT == 0 ? 0 : 1;
  constexpr int SF_COLS_A = 4;            // TMEM columns of SFA per 64-element K step (NVFP4)
  constexpr int SF_COLS_B = ((BN + 127) / 128) * 4;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw_base);

  const uint32_t ring = base;
  const uint32_t bars = base + (uint32_t)p.stages * p.stage_bytes;
  const uint32_t full_bar = bars;                         // [stages]
  const uint32_t empty_bar = bars + 8u * kMaxStages;      // [stages]
  const uint32_t tfull_bar = bars + 16u * kMaxStages;     // [2]
  const uint32_t tempty_bar = tfull_bar + 16u;            // [2]
  const uint32_t drain_bar = tempty_bar + 16u;
  const uint32_t tmem_slot = drain_bar + 8u;
  const uint32_t abort_flag = tmem_slot + 4u;
  uint32_t* const tmem_slot_ptr = reinterpret_cast<uint32_t*>(base_ptr + (tmem_slot - base));

  const uint32_t warp = __shfl_sync(0xffffffffu, threadIdx.x >> 5, 0);   // warp-uniform
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t cta_rank = CG == 2 ? cluster_ctarank() : 0u;
  const bool leader = cta_rank == 0;
  const int pair = (int)(blockIdx.x / CG);
  const int num_pairs = (int)(gridDim.x / CG);

  const unsigned long long clk0 = clock64(), ns0 = globaltimer_ns();
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    if constexpr (DT == 2 && CG == 2) {
      prefetch_tmap(&tmap_sfa);
      prefetch_tmap(&tmap_sfb);
    }
    if (p.stg_bufs > 0) prefetch_tmap(&tmap_d);
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full_bar + 8u * s, 1);
      mbar_init(empty_bar + 8u * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar + 8u * a, 1);
      mbar_init(tempty_bar + 8u * a, EPI_WARPS * CG);   // one arrive per epilogue warp of the pair
    }
    mbar_init(drain_bar, 1);
    st_shared_u32(abort_flag, 0u);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc<CG>(tmem_slot, (uint32_t)p.tmem_cols);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  if constexpr (CG == 2) { cluster_arrive(); cluster_wait(); } else { __syncthreads(); }
  tc_fence_after();
  const uint32_t tmem_base = __shfl_sync(0xffffffffu, *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr), 0);

  SharedCtl ctl;
  ctl.abort_addr = abort_flag;
  ctl.abort_peer = CG == 2 ? mapa_shared(abort_flag, cta_rank ^ 1u) : 0u;
  ctl.timeout_ns = p.timeout_ns;
  ctl.status = p.status;

  // Shape of one pipeline stage as compile-time constants: NA K atoms per
  // stage, KS MMAs (32-byte K steps) per atom row of KS * 32 bytes.  The
  // producer and MMA loops are instantiated per shape and dispatched once,
  // so no runtime loop or branch on the tile shape sits in the k-block loop.
  auto with_stage_shape = [&](auto&& body) {
    switch (p.atoms * 8 + (int)(p.row_bytes / 32u)) {
      case 1 * 8 + 4: body(IntC<1>{}, IntC<4>{}); break;
      case 2 * 8 + 4: body(IntC<2>{}, IntC<4>{}); break;
      case 4 * 8 + 4: body(IntC<4>{}, IntC<4>{}); break;
      case 1 * 8 + 2: body(IntC<1>{}, IntC<2>{}); break;
      case 1 * 8 + 1: body(IntC<1>{}, IntC<1>{}); break;
      default: break;   // the host admits no other shape
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop so every address below is warp-uniform;
    // the loads are predicated on one elected lane (no branch around them).
    if (!(p.flags & GEMM_FLAG_INJECT_STALL)) with_stage_shape([&](auto na_c, auto ks_c) {
      constexpr int NA = decltype(na_c)::value;
      constexpr uint32_t RB = (uint32_t)decltype(ks_c)::value * 32u;   // bytes per atom row
      constexpr int ELEMS = (int)RB / (DT == 0 ? 2 : 1);                 // tensor-map elements per atom row
      const uint32_t issue = elect_one() ? 1u : 0u;
      const uint64_t policy = policy_evict_normal();
      unsigned trace_i = 0;
      (void)trace_i;
      const uint32_t leader_full = CG == 2 ? mapa_shared(full_bar, 0) : full_bar;
      const uint32_t tx_bytes = p.stage_bytes * CG;
      const uint32_t st_bytes = p.stage_bytes, a_bytes = p.a_atom_bytes, b_bytes = p.b_atom_bytes;
      const int n_kb = p.num_k_blocks, n_stages = p.stages;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      // L2 prefetch cursor: runs p.l2_prefetch k-blocks ahead of the load
      // cursor over the same (unit, k-block) sequence.
      int pf_u = pair, pf_kb = 0, pf_m0 = 0, pf_n0 = 0;
      auto pf_coords = [&]() {
        int um, un;
        unit_coords(pf_u, p, um, un);
        pf_m0 = um * MMA_M + (int32_t)cta_rank * BM;
        pf_n0 = un * BN + (int32_t)cta_rank * B_BOX;
      };
      auto pf_step = [&]() {
        if (pf_u >= p.num_units) return;
#pragma unroll
        for (int ka = 0; ka < NA; ++ka) {
          const int32_t x = (pf_kb * NA + ka) * ELEMS;
          tma_prefetch_l2_2d(&tmap_a, x, pf_m0, issue);
#pragma unroll
          for (int h = 0; h < N_SUB; ++h) tma_prefetch_l2_2d(&tmap_b, x, pf_n0 + h * MMA_N, issue);
        }
        if (++pf_kb == n_kb) {
          pf_kb = 0;
          pf_u += num_pairs;
          if (pf_u < p.num_units) pf_coords();
        }
      };
      if (p.l2_prefetch > 0 && pf_u < p.num_units) {
        pf_coords();
        for (int i = 0; i < p.l2_prefetch; ++i) pf_step();
      }
      for (int u = pair; u < p.num_units && ok; u += num_pairs) {
        int um, un;
        unit_coords(u, p, um, un);
        const int32_t m0 = um * MMA_M + (int32_t)cta_rank * BM;
        const int32_t n0 = un * BN + (int32_t)cta_rank * B_BOX;
        for (int kb = 0; kb < n_kb; ++kb) {
          // Fast path: the slot is already free, take it with no warp vote (a
          // per-stage vote made this loop the bottleneck of small single-CTA
          // tiles).  Only a real wait votes, over the lanes that took it.
          if (!mbar_test_wait(empty_bar + 8u * stage, phase ^ 1u)) {
            const bool w = wait_bar<false>(empty_bar + 8u * stage, phase ^ 1u, ctl, ROLE_PRODUCER, stage);
            if (!__all_sync(__activemask(), w)) { ok = false; break; }
          }
          TRACE_EVENT(1u, 1u, stage);
          if (p.l2_prefetch > 0) pf_step();
          const uint32_t sbase = ring + (uint32_t)stage * st_bytes;
          const uint32_t fb = full_bar + 8u * stage;
          const uint32_t target = CG == 2 ? leader_full + 8u * stage : fb;
          // In pair mode one thread issues the stage's expect_tx and loads inside
          // a branch (cheaper there than a whole-warp predicated issue); 1-SM
          // kernels issue from the converged warp, predicated on the elected lane.
          if (CG == 1 || issue) {
          mbar_arrive_expect_tx(fb, tx_bytes, leader ? issue : 0u);
#pragma unroll
          for (int ka = 0; ka < NA; ++ka) {
            const int32_t x = (kb * NA + ka) * ELEMS;
            const uint32_t a_dst = sbase + (uint32_t)ka * a_bytes;
            const uint32_t b_dst = sbase + (uint32_t)NA * a_bytes + (uint32_t)ka * b_bytes;
#pragma unroll
            for (int h = 0; h < N_SUB; ++h) {
              if constexpr (CG == 2) {
                if (h == 0) tma_load_2d_pair(a_dst, &tmap_a, target, x, m0, policy, issue);
                tma_load_2d_pair(b_dst + (uint32_t)(h * B_BOX) * RB, &tmap_b, target, x, n0 + h * MMA_N, policy, issue);
              } else {
                if (h == 0) tma_load_2d(a_dst, &tmap_a, target, x, m0, policy, issue);
                tma_load_2d(b_dst + (uint32_t)(h * B_BOX) * RB, &tmap_b, target, x, n0 + h * MMA_N, policy, issue);
              }
            }
          }
          if constexpr (DT == 2) {
            // Scale factors: one 512-byte atom (128 rows x 4 scales) per 64 K
            // elements; a stage covers NA*4 of them for this CTA's 128 rows of
            // A, and for each of the tile's BN/128 row blocks of B (the whole
            // tile N, also in a CTA pair, whose MMA reads every B scale from
            // each CTA's own TMEM).
            const uint32_t sf_base = sbase + (uint32_t)NA * (a_bytes + b_bytes);
            const int kq0 = kb * NA * 4;
            constexpr int NSF = NA * 4;
            if constexpr (CG == 2) {
              // 3-D maps (512-byte atom, K atom, row block): the loads signal
              // the leader's barrier like the pair's A/B loads.
              tma_load_3d_pair(sf_base, &tmap_sfa, target, 0, kq0, m0 / 128, policy, issue);
              tma_load_3d_pair(sf_base + (uint32_t)NSF * 512u, &tmap_sfb, target, 0, kq0, un * (BN / 128), policy,
                               issue);
            } else {
              const uint8_t* sfa_src = p.sfa + ((int64_t)(m0 / 128) * p.sf_kblocks + kq0) * 512;
              bulk_load(sf_base, sfa_src, (uint32_t)NSF * 512u, target, policy, issue);
#pragma unroll
              for (int bb = 0; bb < BN / 128; ++bb) {
                const uint8_t* sfb_src = p.sfb + ((int64_t)(n0 / 128 + bb) * p.sf_kblocks + kq0) * 512;
                bulk_load(sf_base + (uint32_t)NSF * 512u * (1 + bb), sfb_src, (uint32_t)NSF * 512u, target, policy, issue);
              }
            }
          }
          }
          TRACE_EVENT(1u, 2u, stage);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == n_stages) { stage = 0; phase ^= 1u; }
        }
        ok = __all_sync(0xffffffffu, ok);   // one uniform abort decision per tile
      }
      if (!ok && (CG == 1 || leader)) {
        // Let every load already issued land before the CTA may exit.  In a
        // pair the leader's full barrier of a stage completes only when both
        // CTAs' loads of that stage have landed, so the leader's drain also
        // covers its peer's loads; the teardown cluster barrier then keeps the
        // peer resident until the drain is over.
        for (int s = 0; s < n_stages; ++s)
          if (issued_mask & (1u << s)) drain_wait(full_bar + 8u * s, (issued_parity >> s) & 1u, 100000000ull);
      } else if (!ok) {
        // Pair peer: its loads complete on the leader's barriers, which it
        // cannot wait on; give them a short fixed window before the teardown barrier.
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {}
      }
    });
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Converged warp: descriptors and addresses are warp-uniform; each
    // stage's tcgen05 ops are issued by one lane, elected once, so its
    // commits track all of its MMAs.
    if (leader) with_stage_shape([&](auto na_c, auto ks_c) {
      constexpr int NA = decltype(na_c)::value;
      constexpr int KS = decltype(ks_c)::value;
      constexpr uint32_t RB = (uint32_t)KS * 32u;
      const uint32_t issue = elect_one() ? 1u : 0u;
      unsigned trace_i = 0;
      (void)trace_i;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int pos = 0;            // accumulator position of the next tile when positions overlap
      bool ok = true;
      bool issued = false;
      // Loop-invariant parameters in registers.
      const int n_units = p.num_units, n_kb = p.num_k_blocks, n_stages = p.stages;
      const uint32_t st_bytes = p.stage_bytes, a_bytes = p.a_atom_bytes, b_bytes = p.b_atom_bytes;
      const uint32_t idesc = p.idesc;
      const int n_acc = p.num_acc;
      // NVFP4: each stage's scales go to the next of p.sf_slots TMEM slots, so
      // the copy for stage s+1 never overwrites scales the MMAs of stage s are
      // still reading (with one shared slot each copy waits for those MMAs;
      // the ring measured ~3 % faster).
      const int n_sf_slots = DT == 2 ? p.sf_slots : 1;
      int sf_slot = 0;
      (void)n_sf_slots;
      (void)sf_slot;
      for (int u = pair; u < n_units && ok; u += num_pairs) {
        const bool wt = wait_bar<CG == 2>(tempty_bar + 8u * acc, acc_phase ^ 1u, ctl, ROLE_MMA, 0x80u | acc);
        if (!__all_sync(0xffffffffu, wt)) { ok = false; break; }
        TRACE_EVENT(2u, 3u, acc);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(p.acc_overlap ? pos * (BN - p.acc_overlap) : acc * BN);
        if (p.acc_overlap) pos ^= 1;
        bool ready = false;   // next stage's data already seen (probed after the previous commit)
        for (int kb = 0; kb < n_kb; ++kb) {
          // No warp vote per stage (it cost the MMA-bound small tiles 4-9 %):
          // every lane probes the same barrier in the same instruction, and the
          // tcgen05 ops below are single-thread, so a lane that left early
          // blocks nothing.  The vote after the k-block loop makes the abort
          // decision uniform before the next warp-collective step.
          const bool w = ready || wait_bar<CG == 2>(full_bar + 8u * stage, phase, ctl, ROLE_MMA, stage);
          if (!w) { ok = false; break; }
          TRACE_EVENT(2u, 1u, stage);
          tc_fence_after();
          const uint32_t sbase = ring + (uint32_t)stage * st_bytes;
          const uint32_t bbase = sbase + (uint32_t)NA * a_bytes;
          // Pair mode: the stage's tcgen05 ops are issued by one thread inside a
          // branch -- a predicated issue by the whole warp made every two-CTA
          // tcgen05.cp and tcgen05.mma cost ~70 cycles.  1-SM kernels keep the
          // converged, predicated issue, whose operands stay warp-uniform (small
          // tiles issue a stage every few dozen cycles).
          if (CG == 1 || issue) {
          if constexpr (DT == 2) {
            // Copy this stage's scale factors into TMEM (columns after the
            // accumulators), then issue the block-scaled MMAs.
            const uint32_t sf_base = bbase + (uint32_t)NA * b_bytes;
            constexpr int NSF = NA * 4;
            constexpr uint32_t SF_STAGE_COLS = (uint32_t)NSF * (SF_COLS_A + SF_COLS_B);
            const uint32_t sf0 = p.acc_overlap ? (uint32_t)(2 * BN - p.acc_overlap) : (uint32_t)(n_acc * BN);
            const uint32_t sfa_t = tmem_base + sf0 + (uint32_t)sf_slot * SF_STAGE_COLS;
            const uint32_t sfb_t = sfa_t + (uint32_t)NSF * SF_COLS_A;
            if (++sf_slot == n_sf_slots) sf_slot = 0;
#pragma unroll
            for (int q = 0; q < NSF; ++q) {
              tmem_cp_32x128b_warpx4<CG>(sfa_t + (uint32_t)q * SF_COLS_A, plain_desc(sf_base + (uint32_t)q * 512u), issue);
#pragma unroll
              for (int bb = 0; bb < SF_COLS_B / 4; ++bb)
                tmem_cp_32x128b_warpx4<CG>(sfb_t + (uint32_t)q * SF_COLS_B + 4u * bb,
                                           plain_desc(sf_base + (uint32_t)NSF * 512u * (1 + bb) + (uint32_t)q * 512u), issue);
            }
#pragma unroll
            for (int ka = 0; ka < NA; ++ka) {
              const uint64_t ad = swz_kmajor_desc(sbase + (uint32_t)ka * a_bytes, RB);
              const uint64_t bd = swz_kmajor_desc(bbase + (uint32_t)ka * b_bytes, RB);
#pragma unroll
              for (int kk = 0; kk < KS; ++kk) {
                const int q = ka * KS + kk;
                mma_nvf4<CG>(d_tmem, ad + 2u * kk, bd + 2u * kk, idesc,
                             sfa_t + (uint32_t)q * SF_COLS_A, sfb_t + (uint32_t)q * SF_COLS_B,
                             (kb | ka | kk) != 0, issue);
              }
            }
          } else {
#pragma unroll
            for (int ka = 0; ka < NA; ++ka) {
              const uint64_t ad = swz_kmajor_desc(sbase + (uint32_t)ka * a_bytes, RB);
              const uint64_t bd = swz_kmajor_desc(bbase + (uint32_t)ka * b_bytes, RB);
#pragma unroll
              for (int kk = 0; kk < KS; ++kk)
#pragma unroll
                for (int h = 0; h < N_SUB; ++h)
                  mma_ss<CG, KIND>(d_tmem + (uint32_t)(h * MMA_N), ad + 2u * kk,
                                   bd + (uint64_t)(((uint32_t)(h * B_BOX) * RB) >> 4) + 2u * kk, idesc,
                                   (kb | ka | kk) != 0, issue);
            }
          }
          if constexpr (CG == 2) mma_commit_pair(empty_bar + 8u * stage, 0x3, issue);
          else mma_commit(empty_bar + 8u * stage, issue);
          }
          TRACE_EVENT(2u, 2u, stage);
          issued = true;
          if (++stage == n_stages) { stage = 0; phase ^= 1u; }
          // Probe the next stage now so the barrier round trip overlaps the
          // MMAs just issued instead of opening the next iteration.
          ready = CG == 2 ? mbar_test_wait_cluster(full_bar + 8u * stage, phase)
                          : mbar_test_wait(full_bar + 8u * stage, phase);
        }
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        if constexpr (CG == 2) mma_commit_pair(tfull_bar + 8u * acc, 0x3, issue);
        else mma_commit(tfull_bar + 8u * acc, issue);
        TRACE_EVENT(2u, 4u, acc);
        if (++acc == n_acc) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok && issued) {
        // Wait (bounded) until every MMA already issued has finished with TMEM.
        if constexpr (CG == 2) mma_commit_pair(drain_bar, 0x1, issue);
        else mma_commit(drain_bar, issue);
        drain_wait(drain_bar, 0, 100000000ull);
      }
    });
  } else {
    // ------------------------------------------------------------ epilogue
    // Warps 2..: a group of 4 warps (one per TMEM lane quadrant, 128 lanes)
    // owns COLS accumulator columns of the tile and emits them in chunks of
    // CW columns: tcgen05.ld -> alpha * acc (+ beta * C) -> bf16 pairs, then
    // either staged through shared memory and written by one TMA store per
    // chunk (every D column of the chunk is one contiguous BM-row run, whole
    // cache lines), or stored directly from registers when the staging
    // buffers do not fit next to the ring.
    const uint32_t q = warp & 3u;                   // TMEM lane quadrant of this warp
    constexpr int GROUPS = EPI_WARPS / 4;
    constexpr int COLS = BN / GROUPS;               // accumulator columns per group
    constexpr int CW = COLS % 32 == 0 ? 32 : 16;    // columns per chunk (one tcgen05.ld)
    const int grp = (int)((warp - 2u) / 4u);
    const int c_begin = grp * COLS;
    const uint32_t gtid = ((warp - 2u) & 3u) * 32u + lane;   // thread index within the group
    const bool issuer = gtid == 0;
    const uint32_t bar_id = 1u + (uint32_t)grp;     // named barrier of this group
    const int q_rows = BM / 4;                      // accumulator rows in this warp's quadrant
    const int r_loc = q_rows * (int)q + (int)lane;  // row within the CTA's BM rows (lane < q_rows)
    const float alpha = p.alpha, beta = p.beta;
    const bool row_major = p.d_row_major != 0;
    const int nbuf = p.stg_bufs;
    const uint32_t stg_grp = base + p.stg_offset + (uint32_t)(grp * nbuf) * p.stg_bytes;
    uint32_t chunk_no = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int pos = 0;                                    // accumulator position (overlapped positions)
    const uint32_t leader_tempty = CG == 2 ? mapa_shared(tempty_bar, 0) : tempty_bar;
    unsigned trace_i = 0;
    (void)trace_i;
    for (int u = pair; u < p.num_units; u += num_pairs) {
      int um, un;
      unit_coords(u, p, um, un);
      // Warp-uniform decision: tcgen05.ld below is warp-collective, so every
      // lane must agree to proceed even if one lane saw an abort.  Once one
      // warp of a group has seen the phase complete, every warp of the group
      // does (the first probe tests the barrier before the abort flag), so
      // the group's named barriers below never wait for a warp that left.
      const bool ok = wait_bar<false>(tfull_bar + 8u * acc, acc_phase, ctl, ROLE_EPILOGUE, acc);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (warp == 2) TRACE_EVENT(3u, 1u, acc);
      tc_fence_after();
      const int64_t m0 = (int64_t)um * MMA_M + (int64_t)cta_rank * BM;
      const int64_t row = m0 + r_loc;
      const int64_t n0 = (int64_t)un * BN;
      const bool row_ok = (int)lane < q_rows && row < p.m;
      const int ov = p.acc_overlap;
      const int cur_pos = pos;                         // accumulator position of this tile
      if (ov) pos ^= 1;
      const uint32_t t_row = tmem_base + ((32u * q) << 16) + (uint32_t)(ov ? cur_pos * (BN - ov) : acc * BN);

      auto release_acc = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 2) mbar_arrive_cluster(leader_tempty + 8u * acc); else mbar_arrive(tempty_bar + 8u * acc);
        }
      };

      // alpha * acc for CW columns of this thread's row, rounded to bf16 pairs.
      auto convert = [&](const uint32_t (&r)[CW], uint32_t (&o)[CW / 2]) {
#pragma unroll
        for (int j = 0; j < CW; j += 2) {
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(alpha * __uint_as_float(r[j]), alpha * __uint_as_float(r[j + 1]));
          o[j / 2] = *reinterpret_cast<const uint32_t*>(&h2);
        }
      };
      // alpha * acc + beta * C in fp32, rounded once to bf16 pairs (C in D's layout).
      auto convert_c = [&](int c, const uint32_t (&r)[CW], uint32_t (&o)[CW / 2]) {
        const int64_t col0 = n0 + c;
#pragma unroll
        for (int j = 0; j < CW; j += 2) {
          float c0 = 0.f, c1 = 0.f;
          if (row_ok) {
            if (!row_major) {
              if (col0 + j < p.n) c0 = __bfloat162float(p.c[(col0 + j) * p.ldc + row]);
              if (col0 + j + 1 < p.n) c1 = __bfloat162float(p.c[(col0 + j + 1) * p.ldc + row]);
            } else {
              const __nv_bfloat16* crow = p.c + row * p.ldc + col0;
              if (col0 + j < p.n) c0 = __bfloat162float(crow[j]);
              if (col0 + j + 1 < p.n) c1 = __bfloat162float(crow[j + 1]);
            }
          }
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(fmaf(beta, c0, alpha * __uint_as_float(r[j])),
                                                         fmaf(beta, c1, alpha * __uint_as_float(r[j + 1])));
          o[j / 2] = *reinterpret_cast<const uint32_t*>(&h2);
        }
      };

      // Write CW columns (tile column offset c) of this thread's row.
      auto emit = [&](int c, const uint32_t (&o)[CW / 2]) {
        const int64_t col0 = n0 + c;
        if (nbuf > 0) {
          const uint32_t buf = stg_grp + (nbuf == 2 ? (chunk_no & 1u) : 0u) * p.stg_bytes;
          // The TMA store that last read this buffer must be done reading it.
          if (issuer) {
            if (nbuf == 2) bulk_wait_group_read<1>(); else bulk_wait_group_read<0>();
          }
          named_bar_sync(bar_id, 128);
          if ((int)lane < q_rows) {
            if (!row_major) {
              // [CW columns][BM rows]: each store instruction fills one column's 64-byte run.
#pragma unroll
              for (int j = 0; j < CW; ++j)
                st_shared_u16(buf + (uint32_t)((j * BM + r_loc) * 2), (uint16_t)(j % 2 == 0 ? (o[j / 2] & 0xFFFFu) : (o[j / 2] >> 16)));
            } else {
              // [BM rows][CW columns] in the 64-byte (CW 32) or 32-byte (CW 16) TMA swizzle:
              // 16-byte vector v of row r sits at vector v ^ ((r >> 1) & 3) (CW 32) or
              // v ^ ((r >> 2) & 1) (CW 16), which spreads a warp's rows over all banks.
              const uint32_t rbase = buf + (uint32_t)(r_loc * CW * 2);
              const uint32_t sw = CW == 32 ? (((uint32_t)r_loc >> 1) & 3u) : (((uint32_t)r_loc >> 2) & 1u);
#pragma unroll
              for (int v = 0; v < CW / 8; ++v)
                st_shared_v4(rbase + (((uint32_t)v ^ sw) << 4), o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
            }
          }
          fence_proxy_async_shared();
          named_bar_sync(bar_id, 128);
          if (issuer) {
            if (!row_major) tma_store_2d(&tmap_d, buf, (int32_t)m0, (int32_t)col0);
            else tma_store_2d(&tmap_d, buf, (int32_t)col0, (int32_t)m0);
            bulk_commit_group();
          }
          if (p.n_d_peer > 0) {
            // Fused gather (column-major D only): the staged block again, as 16-byte
            // stores of 8 rows each, into every peer destination.
            const int vpc = BM / 8;
            for (int v = (int)gtid; v < CW * vpc; v += 128) {
              const int j = v / vpc, r8 = (v - j * vpc) * 8;
              const int64_t col = col0 + j, rr = m0 + r8;
              if (col >= p.n || rr >= p.m) continue;
              const uint4 val = ld_shared_v4(buf + (uint32_t)((j * BM + r8) * 2));
              for (int gp = 0; gp < p.n_d_peer; ++gp) {
                __nv_bfloat16* dst = p.d_peer[gp] + col * p.ldd + rr;
                if (rr + 8 <= p.m) {
                  *reinterpret_cast<uint4*>(dst) = val;
                } else {
                  const uint32_t wv[4] = {val.x, val.y, val.z, val.w};
                  uint16_t* d16 = reinterpret_cast<uint16_t*>(dst);
                  for (int e = 0; e < (int)(p.m - rr); ++e)
                    d16[e] = (uint16_t)(e % 2 == 0 ? (wv[e / 2] & 0xFFFFu) : (wv[e / 2] >> 16));
                }
              }
            }
          }
          ++chunk_no;
        } else if (row_ok) {
          if (!row_major) {
            uint16_t* dst = reinterpret_cast<uint16_t*>(p.d + row) + col0 * p.ldd;
#pragma unroll
            for (int j = 0; j < CW; ++j)
              if (col0 + j < p.n) dst[j * p.ldd] = (uint16_t)(j % 2 == 0 ? (o[j / 2] & 0xFFFFu) : (o[j / 2] >> 16));
            for (int gp = 0; gp < p.n_d_peer; ++gp) {   // fused gather: the same block into each peer D
              uint16_t* pdst = reinterpret_cast<uint16_t*>(p.d_peer[gp] + row) + col0 * p.ldd;
#pragma unroll
              for (int j = 0; j < CW; ++j)
                if (col0 + j < p.n) pdst[j * p.ldd] = (uint16_t)(j % 2 == 0 ? (o[j / 2] & 0xFFFFu) : (o[j / 2] >> 16));
            }
          } else {
            __nv_bfloat16* drow = p.d + row * p.ldd + col0;
#pragma unroll
            for (int v = 0; v < CW / 8; ++v) {
              if (col0 + 8 * v + 8 <= p.n) {
                *reinterpret_cast<uint4*>(drow + 8 * v) = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
              } else {
                uint16_t* d16 = reinterpret_cast<uint16_t*>(drow);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  if (col0 + 8 * v + e < p.n)
                    d16[8 * v + e] = (uint16_t)(e % 2 == 0 ? (o[4 * v + e / 2] & 0xFFFFu) : (o[4 * v + e / 2] >> 16));
              }
            }
          }
        }
      };

      auto tmem_chunk = [&](uint32_t taddr, uint32_t (&r)[CW]) {
        if constexpr (CW == 32) tmem_ld32(taddr, r); else tmem_ld16(taddr, r);
        tmem_ld_wait();
      };

      if constexpr (COLS % 32 == 0) {
        if ((BN <= 256 || GEMM_WIDE_EARLY_RELEASE) && p.num_acc == 1 && !ov && beta == 0.f) {
          // Single accumulator (the tile fills TMEM): drain it into registers
          // as packed bf16 pairs, release it at once so the next tile's MMAs
          // start, then write D while that mainloop runs.
          uint32_t pk[COLS / 2];
#pragma unroll
          for (int cc = 0; cc < COLS; cc += 32) {
            uint32_t r[32], o[16];
            tmem_chunk(t_row + (uint32_t)(c_begin + cc), r);
            convert(r, o);
#pragma unroll
            for (int j = 0; j < 16; ++j) pk[cc / 2 + j] = o[j];
          }
          release_acc();
#pragma unroll
          for (int cc = 0; cc < COLS; cc += 32) {
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = pk[cc / 2 + j];
            emit(c_begin + cc, o);
          }
          if (warp == 2) TRACE_EVENT(3u, 2u, acc);
          if (++acc == p.num_acc) { acc = 0; acc_phase ^= 1u; }
          continue;
        }
      }
      // Chunk by chunk: the accumulator is released right after its last
      // chunk has been read from TMEM, before that chunk is written out.  With
      // overlapped positions the columns the other position shares are read
      // first (the tail of position 0, the head of position 1) and the
      // accumulator is released as soon as they are in registers.
      constexpr int NCH = COLS / CW;
      const int ov_ch = ov / CW;
      const int first = (ov && cur_pos == 0) ? NCH - ov_ch : 0;
      const int release_after = ov ? ov_ch - 1 : NCH - 1;
      int i0 = 0;
      if (ov_ch == 2) {
        // Both shared chunks into registers with one wait, then release the
        // accumulator before either is converted and stored: the next tile's
        // MMAs wait only for these two TMEM reads.
        const int ca = (first % NCH) * CW, cb = ((first + 1) % NCH) * CW;
        uint32_t ra[CW], rb[CW], o[CW / 2];
        if constexpr (CW == 32) {
          tmem_ld32(t_row + (uint32_t)(c_begin + ca), ra);
          tmem_ld32(t_row + (uint32_t)(c_begin + cb), rb);
        } else {
          tmem_ld16(t_row + (uint32_t)(c_begin + ca), ra);
          tmem_ld16(t_row + (uint32_t)(c_begin + cb), rb);
        }
        tmem_ld_wait();
        release_acc();
        if (beta != 0.f) convert_c(c_begin + ca, ra, o); else convert(ra, o);
        emit(c_begin + ca, o);
        if (beta != 0.f) convert_c(c_begin + cb, rb, o); else convert(rb, o);
        emit(c_begin + cb, o);
        i0 = 2;
      }
#pragma unroll 1
      for (int i = i0; i < NCH; ++i) {
        const int ci = first + i < NCH ? first + i : first + i - NCH;
        const int cc = ci * CW;
        uint32_t r[CW], o[CW / 2];
        tmem_chunk(t_row + (uint32_t)(c_begin + cc), r);
        if (i == release_after) release_acc();
        if (beta != 0.f) convert_c(c_begin + cc, r, o); else convert(r, o);
        emit(c_begin + cc, o);
      }
      if (warp == 2) TRACE_EVENT(3u, 2u, acc);
      if (++acc == p.num_acc) { acc = 0; acc_phase ^= 1u; }
    }
    // Every TMA store of this group must have completed before the CTA exits.
    if (issuer && nbuf > 0) bulk_wait_group<0>();
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  tc_fence_before();
  if constexpr (CG == 2) { cluster_arrive(); cluster_wait(); } else { __syncthreads(); }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, (uint32_t)p.tmem_cols);
  }
  if (p.clock_out && threadIdx.x == 0) {
    // Every CTA adds its own cycles and nanoseconds: the ratio is the launch's
    // mean SM clock, weighted by how long each CTA ran.
    atomicAdd(p.clock_out, (unsigned long long)(clock64() - clk0));
    atomicAdd(p.clock_out + 1, (unsigned long long)(globaltimer_ns() - ns0));
  }
}

// ----------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

struct Resolved {
  int dt, cg, bm, bn, tile_k, atoms, stages, max_stages, cluster_m;
  uint32_t a_atom_bytes, b_atom_bytes, sf_stage_bytes, stage_bytes;
  int64_t smem_bytes;
  int tmem_cols, num_acc, threads, sf_slots;
  int acc_overlap;                  // columns the two accumulator positions share (0 = disjoint)
  uint32_t row_bytes;
  int cw, stg_bufs;                 // epilogue chunk width; staging buffers per group (0 = direct stores)
  uint32_t stg_bytes, stg_offset;
  float alpha_eff;                  // alpha * scale_a * scale_b
  int num_m_units, num_n_units, num_units, num_k_blocks;
  int grid, num_sms, raster_group;
  char reason[128];
};

int next_pow2_cols(int c) {
  int r = 32;
  while (r < c) r <<= 1;
  return r;
}

bool supported_bn(int cg, int bn) {
  if (cg == 1) return bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 192 || bn == 256;
  return bn == 64 || bn == 128 || bn == 192 || bn == 256 || bn == 512;
}

#define FAIL(...) do { snprintf(r.reason, sizeof(r.reason), __VA_ARGS__); return GEMM_ERR_CANNOT_IMPLEMENT; } while (0)

int resolve(const GemmArgs* a, Resolved& r) {
  memset(&r, 0, sizeof(r));
  if (!a) { snprintf(r.reason, sizeof(r.reason), "null args"); return GEMM_ERR_BAD_ARGS; }
  if (a->struct_size != sizeof(GemmArgs)) {
    snprintf(r.reason, sizeof(r.reason), "GemmArgs.struct_size %u != %zu", a->struct_size, sizeof(GemmArgs));
    return GEMM_ERR_BAD_ARGS;
  }
  if (a->dtype < 0 || a->dtype > 2) FAIL("unknown dtype %d", a->dtype);
  r.dt = a->dtype;
  if (a->m <= 0 || a->n <= 0 || a->k <= 0) FAIL("empty problem %lld x %lld x %lld", (long long)a->m, (long long)a->n, (long long)a->k);
  if (a->m > INT32_MAX / 2 || a->n > INT32_MAX / 2 || a->k > INT32_MAX / 2) FAIL("dimension too large");
  if (!a->a || !a->b || !a->d) { snprintf(r.reason, sizeof(r.reason), "null A/B/D pointer"); return GEMM_ERR_BAD_ARGS; }
  if (r.dt == 2 && (!a->sfa || !a->sfb)) { snprintf(r.reason, sizeof(r.reason), "NVFP4 needs sfa and sfb"); return GEMM_ERR_BAD_ARGS; }

  r.cg = a->cta_group == 0 ? 1 : a->cta_group;
  if (r.cg != 1 && r.cg != 2) FAIL("cta_group must be 1 or 2");
  r.cluster_m = a->cluster_m == 0 ? r.cg : a->cluster_m;
  if (r.cluster_m != r.cg) FAIL("cluster_m %d unsupported (must equal cta_group)", r.cluster_m);
  r.bm = 128 * r.cg;
  if (r.cg == 1 && a->tile_m == 64) {
    if (r.dt == 2) FAIL("tile_m 64 unsupported for NVFP4 (scale atoms are 128 rows)");
    r.bm = 64;
  }
  if (a->tile_m != 0 && a->tile_m != r.bm)
    FAIL("tile_m %d unsupported for cta_group %d (need %d%s)", a->tile_m, r.cg, r.bm, r.cg == 1 ? " or 64" : "");
  r.bn = a->tile_n == 0 ? 256 : a->tile_n;
  if (!supported_bn(r.cg, r.bn)) FAIL("tile_n %d unsupported for cta_group %d", r.bn, r.cg);
  const int ae = atom_elems(r.dt);
  r.tile_k = a->tile_k == 0 ? ae : a->tile_k;
  // A stage narrower than one 128-byte swizzle row uses the 64- or 32-byte
  // swizzle with one atom; wider stages are whole 128-byte atoms.
  const int mma_k = ae / 4;   // K elements of one MMA (32 bytes)
  if (r.tile_k < ae && r.dt != 2 && (r.tile_k == mma_k || r.tile_k == 2 * mma_k)) {
    r.row_bytes = (uint32_t)(r.tile_k / mma_k) * 32u;
    r.atoms = 1;
  } else {
    if (r.tile_k % ae != 0)
      FAIL("tile_k %d must be a multiple of %d (one 128-byte swizzle atom)%s", r.tile_k, ae,
           r.dt == 2 ? "" : ", or one or two MMA K steps");
    r.row_bytes = 128u;
    r.atoms = r.tile_k / ae;
    if (r.atoms != 1 && r.atoms != 2 && r.atoms != 4)
      FAIL("tile_k %d must be 1, 2 or 4 128-byte swizzle atoms (%d, %d or %d)", r.tile_k, ae, 2 * ae, 4 * ae);
  }

  // Element size in bytes (NVFP4: half a byte) and alignment (128-bit, as the reference's Alignment{A,B,D}).
  const int64_t bits = r.dt == 0 ? 16 : (r.dt == 1 ? 8 : 4);
  if (a->lda < a->k || a->ldb < a->k) FAIL("lda/ldb must be >= k");
  if (a->d_layout != GEMM_LAYOUT_COL_MAJOR && a->d_layout != GEMM_LAYOUT_ROW_MAJOR) FAIL("unknown d_layout %d", a->d_layout);
  const bool d_rm = a->d_layout == GEMM_LAYOUT_ROW_MAJOR;
  if (a->ldd < (d_rm ? a->n : a->m)) FAIL("ldd must be >= %s", d_rm ? "n (row-major D)" : "m");
  if (a->beta != 0.f) {
    if (!a->c) { snprintf(r.reason, sizeof(r.reason), "beta != 0 needs C"); return GEMM_ERR_BAD_ARGS; }
    if (a->ldc < (d_rm ? a->n : a->m)) FAIL("ldc must be >= %s", d_rm ? "n (row-major C)" : "m");
    if ((a->ldc * 16) % 128 != 0) FAIL("ldc must be a multiple of 8");
    if ((uintptr_t)a->c & 15) FAIL("C must be 16-byte aligned");
  }
  r.alpha_eff = a->alpha * (a->scale_a != 0.f ? a->scale_a : 1.f) * (a->scale_b != 0.f ? a->scale_b : 1.f);
  if ((a->lda * bits) % 128 != 0 || (a->ldb * bits) % 128 != 0) FAIL("lda/ldb rows must be 16-byte multiples");
  if ((a->ldd * 16) % 128 != 0) FAIL("ldd must be a multiple of 8");
  if (((uintptr_t)a->a | (uintptr_t)a->b | (uintptr_t)a->d) & 15) FAIL("A/B/D must be 16-byte aligned");
  if ((a->k * bits) % 128 != 0) FAIL("k must be a multiple of %lld", (long long)(128 / bits));
  if (r.dt == 2) {
    if (a->k % r.tile_k != 0) FAIL("NVFP4 needs k %% tile_k == 0");
    if (a->m % r.bm != 0 || a->n % r.bn != 0) FAIL("NVFP4 needs m %% %d == 0 and n %% tile_n == 0", r.bm);
    if (r.bn != 128 && r.bn != 256) FAIL("NVFP4 needs tile_n 128 or 256 (scale atoms are 128 rows)");
    if (((uintptr_t)a->sfa | (uintptr_t)a->sfb) & 15) FAIL("sfa/sfb must be 16-byte aligned");
  }

  r.a_atom_bytes = (uint32_t)(r.bm / r.cg) * r.row_bytes;
  r.b_atom_bytes = (uint32_t)(r.bn / r.cg) * r.row_bytes;
  r.sf_stage_bytes = 0;
  if (r.dt == 2) {
    const int b_blocks = r.bn / 128;   // every CTA (also of a pair) stages the whole tile's B scales
    r.sf_stage_bytes = (uint32_t)(r.atoms * 4 * 512 * (1 + b_blocks));
  }
  r.stage_bytes = (uint32_t)r.atoms * (r.a_atom_bytes + r.b_atom_bytes) + r.sf_stage_bytes;
  const int64_t fixed = 1024 /* alignment slack */ + kBarrierBytes;
  r.max_stages = (int)((kSmemLimit - fixed) / r.stage_bytes);
  if (r.max_stages > kMaxStages) r.max_stages = kMaxStages;
  if (r.max_stages < 1) FAIL("one stage (%u B) exceeds shared memory", r.stage_bytes);
  r.stages = a->stages == 0 ? r.max_stages : a->stages;
  if (r.stages < 1) FAIL("stages must be >= 1");
  if (r.stages > r.max_stages) FAIL("stages %d exceed shared memory (max %d at %u B/stage)", r.stages, r.max_stages, r.stage_bytes);
  r.smem_bytes = fixed + (int64_t)r.stages * r.stage_bytes;
  // Epilogue staging: per group of 4 epilogue warps, one or two buffers of
  // (rows per CTA) x CW bf16 after the ring and barriers, when they fit; else
  // the epilogue stores D directly from registers.  The stage count (and so
  // can_implement) never depends on it.
  {
    const int groups = epi_warps_for(r.bn) / 4;
    r.cw = (r.bn / groups) % 32 == 0 ? 32 : 16;
    r.stg_bytes = (uint32_t)((r.bm / r.cg) * r.cw * 2);
    const int64_t ring_end = ((int64_t)r.stages * r.stage_bytes + kBarrierBytes + 1023) / 1024 * 1024;
    r.stg_offset = (uint32_t)ring_end;
    r.stg_bufs = 0;
    if (!(a->flags & GEMM_FLAG_DIRECT_EPILOGUE))
      for (int nb = 2; nb >= 1 && r.stg_bufs == 0; --nb)
        if (1024 + ring_end + (int64_t)groups * nb * r.stg_bytes <= kSmemLimit) r.stg_bufs = nb;
    if (r.stg_bufs > 0) r.smem_bytes = 1024 + ring_end + (int64_t)groups * r.stg_bufs * r.stg_bytes;
  }
  // One CTA per SM: the persistent schedule assumes it, and a second resident
  // CTA would only stall in tcgen05.alloc until the first frees its columns.
  if (r.smem_bytes < kMinSmemPerCta) r.smem_bytes = kMinSmemPerCta;

  int sf_cols = 0;   // TMEM columns of one stage's scale factors
  if (r.dt == 2) {
    const int nsf = r.atoms * 4;
    sf_cols = nsf * 4 + nsf * ((r.bn + 127) / 128) * 4;
  }
  // Two accumulator buffers when they fit (the epilogue then overlaps the
  // next tile's mainloop), else one.  NVFP4 scale factors then take as many
  // per-stage slots (up to 4, at most the stage count) as the columns left allow.
  r.num_acc = 2 * r.bn + sf_cols <= 512 ? 2 : 1;
  r.acc_overlap = 0;
  if (r.num_acc == 1 && sf_cols > 0 && r.bn == 256 && kAccOverlap > 0 && 2 * r.bn - kAccOverlap + sf_cols <= 512) {
    // NVFP4 256-wide tile: the second accumulator position starts kAccOverlap
    // columns before the first one ends, which leaves the top columns for the
    // scale factors.  The epilogue reads the shared columns first and then
    // releases the accumulator, so the next tile's MMAs overlap the rest of it.
    r.acc_overlap = kAccOverlap;
  }
  const int acc_cols = r.acc_overlap ? 2 * r.bn - r.acc_overlap : r.num_acc * r.bn;
  r.sf_slots = 1;
  if (sf_cols > 0) {
    r.sf_slots = (512 - acc_cols) / sf_cols;
    if (r.sf_slots > 4) r.sf_slots = 4;
    if (r.sf_slots > r.stages) r.sf_slots = r.stages;
    if (r.sf_slots < 1) r.sf_slots = 1;
  }
  const int cols = acc_cols + r.sf_slots * sf_cols;
  if (cols > 512) FAIL("TMEM: %d columns needed (accumulator + scales) > 512", cols);
  r.tmem_cols = next_pow2_cols(cols);
  r.threads = threads_for(r.bn);

  r.num_m_units = (int)((a->m + r.bm - 1) / r.bm);
  r.num_n_units = (int)((a->n + r.bn - 1) / r.bn);
  r.num_units = r.num_m_units * r.num_n_units;
  r.num_k_blocks = (int)((a->k + r.tile_k - 1) / r.tile_k);
  r.raster_group = a->raster_group != 0 ? a->raster_group : 1;
  if (r.raster_group > r.num_m_units) r.raster_group = r.num_m_units;
  if (-r.raster_group > r.num_n_units) r.raster_group = -r.num_n_units;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&r.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    r.num_sms = 148;
    cudaGetLastError();
  }
  int pairs = r.num_sms / r.cg;
  if (a->max_ctas > 0) pairs = a->max_ctas / r.cg > 0 ? a->max_ctas / r.cg : 1;
  if (pairs > r.num_units) pairs = r.num_units;
  r.grid = pairs * r.cg;
  return GEMM_OK;
}
#undef FAIL

bool encode_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType t, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, uint32_t swizzle_bytes) {
  const CUtensorMapSwizzle swz = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                               : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                               : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult res = g_encode(m, t, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                          GEMM_L2_PROMOTION, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS;
}

// Scale-factor tensor map: dims (128 x uint32 = one 512-byte atom, K/64 atoms,
// row blocks of 128), no swizzle; box (128, nsf atoms, row blocks).
bool encode_sf_3d(CUtensorMap* m, const void* ptr, uint64_t kblocks, uint64_t row_blocks, uint32_t box_kb,
                  uint32_t box_rb) {
  cuuint64_t dims[3] = {128, kblocks, row_blocks};
  cuuint64_t strides[2] = {512, kblocks * 512};
  cuuint32_t box[3] = {128, box_kb, box_rb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult res = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS;
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, KernelParams);

template <int DT, int CG, int BN>
KernelFn kernel_ptr() { return gemm_sm100a_kernel<DT, CG, BN>; }

template <int DT, int CG>
KernelFn pick_bn(int bn) {
  if constexpr (CG == 1) {
    switch (bn) {
      case 16: return kernel_ptr<DT, CG, 16>();
      case 32: return kernel_ptr<DT, CG, 32>();
      case 64: return kernel_ptr<DT, CG, 64>();
      case 128: return kernel_ptr<DT, CG, 128>();
      case 192: return kernel_ptr<DT, CG, 192>();
      case 256: return kernel_ptr<DT, CG, 256>();
    }
  } else {
    switch (bn) {
      case 64: return kernel_ptr<DT, CG, 64>();
      case 128: return kernel_ptr<DT, CG, 128>();
      case 192: return kernel_ptr<DT, CG, 192>();
      case 256: return kernel_ptr<DT, CG, 256>();
      case 512:
        if constexpr (DT != 2) return kernel_ptr<DT, CG, 512>();
        break;
    }
  }
  return nullptr;
}

// Each kernel's dynamic shared-memory limit is raised to the 227 KiB maximum
// once per device (launches then pass their own size), so a launch makes no
// attribute call; that keeps launches cheap and capturable in CUDA graphs.
std::mutex g_attr_mu;
struct AttrSet { KernelFn fn; int dev; };
AttrSet g_attr_set[1024];
int g_attr_n = 0;

bool ensure_smem_attr(KernelFn fn, int dev) {
  std::lock_guard<std::mutex> lock(g_attr_mu);
  for (int i = 0; i < g_attr_n; ++i)
    if (g_attr_set[i].fn == fn && g_attr_set[i].dev == dev) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (g_attr_n < 1024) g_attr_set[g_attr_n++] = {fn, dev};
  return true;
}

KernelFn pick_kernel(int dt, int cg, int bn) {
  switch (dt * 2 + (cg - 1)) {
    case 0: return pick_bn<0, 1>(bn);
    case 1: return pick_bn<0, 2>(bn);
    case 2: return pick_bn<1, 1>(bn);
    case 3: return pick_bn<1, 2>(bn);
    case 4: return pick_bn<2, 1>(bn);
    case 5: return pick_bn<2, 2>(bn);
  }
  return nullptr;
}

}  // namespace

extern "C" int gemm_sm100a_query(const GemmArgs* args, GemmInfo* info) {
  Resolved r;
  const int rc = resolve(args, r);
  if (info) {
    memset(info, 0, sizeof(*info));
    info->struct_size = sizeof(GemmInfo);
    info->tile_m = r.bm; info->tile_n = r.bn; info->tile_k = r.tile_k; info->stages = r.stages;
    info->cta_group = r.cg; info->cluster_m = r.cluster_m; info->max_stages = r.max_stages;
    info->smem_bytes_per_stage = r.stage_bytes; info->smem_bytes = r.smem_bytes;
    info->tmem_columns = r.tmem_cols; info->grid_ctas = r.grid; info->num_tiles = r.num_units;
    info->num_sms = r.num_sms; info->can_implement = rc == GEMM_OK;
    memcpy(info->reason, r.reason, sizeof(info->reason));
    info->epilogue_staging_buffers = r.stg_bufs;
  }
  return rc;
}

// One launch; `peers` (n_peers <= kMaxGatherPeers) are extra D destinations
// already validated by the caller.
static int launch_impl(const GemmArgs* args, void* const* peers, int n_peers, void* stream) {
  StreamDeviceGuard guard(reinterpret_cast<cudaStream_t>(stream));
  if (!guard.ok) return GEMM_ERR_LAUNCH;
  Resolved r;
  int rc = resolve(args, r);
  if (rc != GEMM_OK) return rc;
  if (!get_encode()) return GEMM_ERR_LAUNCH;
  const GemmArgs& a = *args;

  CUtensorMap tma_a, tmb_b;
  const bool bf = r.dt == 0;
  const CUtensorMapDataType t = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const int64_t eb_num = r.dt == 0 ? 2 : 1, eb_den = r.dt == 2 ? 2 : 1;   // bytes per element = num/den
  const uint64_t inner_k = (uint64_t)(r.dt == 2 ? a.k / 2 : a.k);       // tensor-map elements along K
  const uint32_t box_inner = bf ? r.row_bytes / 2 : r.row_bytes;
  if (!encode_2d(&tma_a, a.a, t, inner_k, (uint64_t)a.m, (uint64_t)(a.lda * eb_num / eb_den), box_inner,
                 (uint32_t)(r.bm / r.cg), r.row_bytes))
    return GEMM_ERR_CANNOT_IMPLEMENT;
  if (!encode_2d(&tmb_b, a.b, t, inner_k, (uint64_t)a.n, (uint64_t)(a.ldb * eb_num / eb_den), box_inner,
                 (uint32_t)((r.bn > 256 ? 256 : r.bn) / r.cg), r.row_bytes))
    return GEMM_ERR_CANNOT_IMPLEMENT;

  // NVFP4 pair kernel: scale factors through 3-D maps (uint32 x 128 = one
  // 512-byte atom, K/64 atoms per row block, row blocks), one stage's atoms
  // per box: SFA one row block, SFB the tile's BN/128 row blocks.
  CUtensorMap tm_sfa, tm_sfb;
  memset(&tm_sfa, 0, sizeof(tm_sfa));
  memset(&tm_sfb, 0, sizeof(tm_sfb));
  if (r.dt == 2 && r.cg == 2) {
    const uint32_t nsf = (uint32_t)r.atoms * 4u;
    if (!encode_sf_3d(&tm_sfa, a.sfa, (uint64_t)(a.k / 64), (uint64_t)(a.m / 128), nsf, 1u) ||
        !encode_sf_3d(&tm_sfb, a.sfb, (uint64_t)(a.k / 64), (uint64_t)(a.n / 128), nsf, (uint32_t)(r.bn / 128)))
      return GEMM_ERR_CANNOT_IMPLEMENT;
  }

  // D for the staged epilogue's TMA stores: box = the CTA's rows x one CW-column
  // chunk; column-major unswizzled, row-major in the 64- / 32-byte swizzle the
  // epilogue writes its staging rows in.
  CUtensorMap tm_d;
  memset(&tm_d, 0, sizeof(tm_d));
  if (r.stg_bufs > 0) {
    const bool d_rm = a.d_layout == GEMM_LAYOUT_ROW_MAJOR;
    const uint32_t rows = (uint32_t)(r.bm / r.cg);
    const bool okd = d_rm ? encode_2d(&tm_d, a.d, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)a.n, (uint64_t)a.m,
                                      (uint64_t)a.ldd * 2u, (uint32_t)r.cw, rows, r.cw == 32 ? 64u : 32u)
                          : encode_2d(&tm_d, a.d, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)a.m, (uint64_t)a.n,
                                      (uint64_t)a.ldd * 2u, rows, (uint32_t)r.cw, 0u);
    if (!okd) return GEMM_ERR_CANNOT_IMPLEMENT;
  }

  KernelParams p;
  memset(&p, 0, sizeof(p));
  p.m = (int32_t)a.m; p.n = (int32_t)a.n; p.k = (int32_t)a.k;
  p.num_m_units = r.num_m_units; p.num_n_units = r.num_n_units; p.num_units = r.num_units;
  p.num_k_blocks = r.num_k_blocks; p.atoms = r.atoms; p.stages = r.stages;
  p.raster_group = r.raster_group; p.tmem_cols = r.tmem_cols;
  p.stage_bytes = r.stage_bytes; p.a_atom_bytes = r.a_atom_bytes; p.b_atom_bytes = r.b_atom_bytes;
  p.row_bytes = r.row_bytes;
  p.cta_rows = r.bm / r.cg;
  p.sf_stage_bytes = r.sf_stage_bytes;
  p.idesc = make_idesc(r.dt, r.bm, r.bn > 256 ? 256 : r.bn);
  p.num_acc = r.num_acc;
  p.acc_overlap = r.acc_overlap;
  p.alpha = r.alpha_eff;
  p.beta = a.beta;
  p.c = reinterpret_cast<const __nv_bfloat16*>(a.c);
  p.ldc = a.ldc;
  p.d_row_major = a.d_layout == GEMM_LAYOUT_ROW_MAJOR ? 1 : 0;
  p.stg_bufs = r.stg_bufs;
  p.stg_offset = r.stg_offset;
  p.stg_bytes = r.stg_bytes;
  p.d = reinterpret_cast<__nv_bfloat16*>(a.d);
  p.ldd = a.ldd;
  p.status = a.status;
  p.timeout_ns = (uint64_t)(a.timeout_ms ? a.timeout_ms : 4000u) * 1000000ull;
  p.flags = a.flags;
  p.sfa = reinterpret_cast<const uint8_t*>(a.sfa);
  p.sfb = reinterpret_cast<const uint8_t*>(a.sfb);
  p.sf_kblocks = (int32_t)(a.k / 64);
  p.sf_slots = r.sf_slots;
  p.n_d_peer = n_peers;
  for (int i = 0; i < n_peers; ++i) p.d_peer[i] = reinterpret_cast<__nv_bfloat16*>(peers[i]);
  p.l2_prefetch = a.l2_prefetch < 0 ? 0 : (a.l2_prefetch == 0 ? kDefaultL2Prefetch : a.l2_prefetch);
  p.clock_out = a.clock_out;

  KernelFn fn = pick_kernel(r.dt, r.cg, r.bn);
  if (!fn) return GEMM_ERR_CANNOT_IMPLEMENT;
  if (!ensure_smem_attr(fn, guard.dev)) return GEMM_ERR_LAUNCH;

  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)r.grid, 1, 1);
  cfg.blockDim = dim3((unsigned)r.threads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)r.smem_bytes;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)r.cg;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, tma_a, tmb_b, tm_sfa, tm_sfb, tm_d, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return GEMM_ERR_LAUNCH;
  }
  return GEMM_OK;
}

extern "C" int gemm_sm100a_launch(const GemmArgs* args, void* stream) {
  return launch_impl(args, nullptr, 0, stream);
}

namespace {

using PFN_memGetAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
PFN_memGetAddressRange g_addr_range = nullptr;
std::once_flag g_addr_range_once;

// True when [ptr, ptr + bytes) lies inside one device allocation.  The range
// is queried in the caller's context (which also holds mappings opened from
// other processes by CUDA IPC), else with the owning device current (its
// primary context), after which the caller's device is restored.
bool block_inside_allocation(const void* ptr, size_t bytes, int owner, int current) {
  std::call_once(g_addr_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_addr_range = reinterpret_cast<PFN_memGetAddressRange>(fn);
  });
  if (!g_addr_range) return false;
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS && owner != current) {
    if (cudaSetDevice(owner) != cudaSuccess) { cudaGetLastError(); return false; }
    r = g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
    cudaSetDevice(current);
  }
  if (r != CUDA_SUCCESS) return false;
  const uintptr_t p = reinterpret_cast<uintptr_t>(ptr);
  return p >= base && bytes <= size && p - base <= size - bytes;
}

}  // namespace

extern "C" int gemm_sm100a_launch_gather(const GemmArgs* args, void* const* peer_d, int32_t n_peers,
                                         void* stream) {
  if (n_peers < 0 || n_peers > kMaxGatherPeers || (n_peers > 0 && !peer_d)) return GEMM_ERR_BAD_ARGS;
  if (args && args->struct_size == sizeof(GemmArgs) && n_peers > 0 && args->d_layout != GEMM_LAYOUT_COL_MAJOR)
    return GEMM_ERR_CANNOT_IMPLEMENT;   // the gather writes column-major D blocks
  StreamDeviceGuard guard(reinterpret_cast<cudaStream_t>(stream));
  if (!guard.ok) return GEMM_ERR_LAUNCH;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GEMM_ERR_LAUNCH;
  {
    Resolved r;
    const int rc = resolve(args, r);
    if (rc != GEMM_OK) return rc;
  }
  // Bytes of the m x n column-major block at stride ldd that every destination must hold.
  const size_t block_bytes = ((size_t)(args->n - 1) * (size_t)args->ldd + (size_t)args->m) * 2u;
  if (n_peers > 0) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, args->d) != cudaSuccess || at.type != cudaMemoryTypeDevice ||
        !block_inside_allocation(args->d, block_bytes, at.device, dev)) {
      cudaGetLastError();
      return GEMM_ERR_BAD_ARGS;
    }
  }
  for (int i = 0; i < n_peers; ++i) {
    // Every destination must be device memory this GPU can store to, large
    // enough for the whole block; enable peer access where it is another
    // GPU's memory, so a bad pointer or a short buffer is an error here and
    // never a fault in the kernel.
    if (!peer_d[i] || (reinterpret_cast<uintptr_t>(peer_d[i]) & 15)) return GEMM_ERR_BAD_ARGS;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, peer_d[i]) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      return GEMM_ERR_BAD_ARGS;
    }
    if (!block_inside_allocation(peer_d[i], block_bytes, at.device, dev)) {
      cudaGetLastError();
      return GEMM_ERR_BAD_ARGS;
    }
    if (at.device != dev) {
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, dev, at.device) != cudaSuccess || !can) { cudaGetLastError(); return GEMM_ERR_BAD_ARGS; }
      const cudaError_t e = cudaDeviceEnablePeerAccess(at.device, 0);
      if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) { cudaGetLastError(); return GEMM_ERR_LAUNCH; }
      cudaGetLastError();   // clear "already enabled"
    }
  }
  return launch_impl(args, peer_d, n_peers, stream);
}

extern "C" int gemm_sm100a_read_status(const int32_t* status, void* stream, int32_t* detail) {
  StreamDeviceGuard guard(reinterpret_cast<cudaStream_t>(stream));
  if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) {
    cudaGetLastError();
    return GEMM_ERR_LAUNCH;
  }
  if (!status) { if (detail) *detail = 0; return GEMM_OK; }
  int32_t v = 0;
  if (cudaMemcpy(&v, status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return GEMM_ERR_LAUNCH;
  }
  if (detail) *detail = v;
  return v == 0 ? GEMM_OK : GEMM_ERR_TIMEOUT;
}

extern "C" const char* gemm_sm100a_strerror(int code) {
  switch (code) {
    case GEMM_OK: return "ok";
    case GEMM_ERR_CANNOT_IMPLEMENT: return "cannot implement (shape, alignment, knob or shared-memory limit)";
    case GEMM_ERR_LAUNCH: return "CUDA launch or driver error";
    case GEMM_ERR_TIMEOUT: return "device wait timed out";
    case GEMM_ERR_BAD_ARGS: return "bad arguments";
  }
  return "unknown error";
}

extern "C" int gemm_sm100a_version(void) { return 200; }

#if GEMM_TRACE
// Trace builds only: copy CTA 0's event log (4 regions of 16384 entries, one
// per role) to `out` and clear it.  Returns the number of entries copied.
extern "C" int gemm_sm100a_trace_read(unsigned long long* out, int max) {
  const int n = max < (int)(4 * kTraceRegion) ? max : (int)(4 * kTraceRegion);
  if (cudaMemcpyFromSymbol(out, g_trace_log, (size_t)n * sizeof(unsigned long long)) != cudaSuccess) return -1;
  static unsigned long long zeros[4 * kTraceRegion];
  cudaMemcpyToSymbol(g_trace_log, zeros, sizeof(zeros));
  return n;
}
#endif
